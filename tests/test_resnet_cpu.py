"""ResNet parity on CPU: the fp32 restatement against the reference model's own outputs, and a
torch emulation of the device layout (padded pixel space, one row shift per 3x3 tap, packed
K-major weights with folded BatchNorm) against the fp32 restatement."""
import os

import numpy as np
import torch

from conftest import REPO

GOLDEN = os.path.join(REPO, "tests", "golden", "resnet_small.npz")


def _fixture():
    z = np.load(GOLDEN)
    sd = {k[3:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("sd/")}
    return sd, torch.from_numpy(z["x"]), z["policy"], z["value"]


def test_fp32_restatement_matches_reference_model():
    from omoknuni_quantum_b200.resnet import reference_forward_fp32
    sd, x, pol, val = _fixture()
    p, v = reference_forward_fp32(sd, x)
    np.testing.assert_allclose(p.numpy(), pol, rtol=0, atol=2e-6)
    np.testing.assert_allclose(v.numpy(), val, rtol=0, atol=2e-6)


def emulate_device_forward(conv_w, conv_b, head, spec, x):
    """The device algorithm in fp32 torch: activations [B*P, C] in the padded pixel space."""
    S, C, HW = spec.board_size, spec.filters, spec.hw
    P = (S + 1) ** 2
    B = x.shape[0]
    inp = torch.zeros(B, S + 1, S + 1, 64)
    inp[:, :S, :S, :spec.input_channels] = x.permute(0, 2, 3, 1)
    a = inp.reshape(B * P, 64)
    pad = torch.zeros(S + 1, S + 1, dtype=torch.bool)
    pad[S, :] = True
    pad[:, S] = True
    pad = pad.reshape(-1).repeat(B)

    def conv(a, w, b, res=None):
        cin = a.shape[1]
        w = w.reshape(C, 9, cin)
        out = torch.zeros(a.shape[0], C)
        for tap in range(9):
            off = (tap // 3 - 1) * (S + 1) + (tap % 3 - 1)
            src = torch.zeros_like(a)
            lo, hi = max(0, -off), min(a.shape[0], a.shape[0] - off)
            src[lo:hi] = a[lo + off:hi + off]
            out += src @ w[:, tap, :].T
        out = out + b
        if res is not None:
            out = out + res
        out = torch.relu(out)
        out[pad] = 0
        return out

    nw = C * 9 * 64
    h = conv(a, conv_w[:nw].float(), conv_b[:C])
    off_w, off_b = nw, C
    for i in range(spec.num_blocks):
        t = conv(h, conv_w[off_w:off_w + C * 9 * C].float(), conv_b[off_b:off_b + C])
        off_w += C * 9 * C; off_b += C
        h = conv(t, conv_w[off_w:off_w + C * 9 * C].float(), conv_b[off_b:off_b + C], res=h)
        off_w += C * 9 * C; off_b += C
    real = h.reshape(B, S + 1, S + 1, C)[:, :S, :S, :].reshape(B, HW, C)
    Hp, Hv, A = spec.fc_policy_hidden, spec.fc_value_hidden, spec.num_actions
    o = 0
    w1 = head[o:o + 3 * C].reshape(3, C); o += 3 * C
    b1 = head[o:o + 3]; o += 3
    fc1p = head[o:o + 2 * HW * Hp].reshape(2 * HW, Hp); o += 2 * HW * Hp
    b1p = head[o:o + Hp]; o += Hp
    fc2p = head[o:o + Hp * A].reshape(Hp, A); o += Hp * A
    b2p = head[o:o + A]; o += A
    fc1v = head[o:o + HW * Hv].reshape(HW, Hv); o += HW * Hv
    b1v = head[o:o + Hv]; o += Hv
    fc2v = head[o:o + Hv]; o += Hv
    b2v = head[o]
    h3 = torch.relu(real @ w1.T + b1)                      # [B, HW, 3]
    pin = h3[:, :, :2].permute(0, 2, 1).reshape(B, 2 * HW)
    hp = torch.relu(pin @ fc1p + b1p)
    pol = torch.softmax(hp @ fc2p + b2p, dim=1)
    hv = torch.relu(h3[:, :, 2] @ fc1v + b1v)
    val = torch.tanh(hv @ fc2v + b2v)
    return pol, val


def test_device_layout_emulation_matches_fp32_forward():
    from omoknuni_quantum_b200.resnet import pack_parameters, reference_forward_fp32, spec_from_state_dict
    sd, x, _, _ = _fixture()
    spec = spec_from_state_dict(sd, 15)
    conv_w, conv_b, head = pack_parameters(sd, spec)
    # emulate with the unrounded weights: repack in fp32 to isolate the layout from bf16 rounding
    w32 = torch.cat([t.reshape(-1) for t in _pack_fp32(sd, spec)])
    p_ref, v_ref = reference_forward_fp32(sd, x)
    p, v = emulate_device_forward(w32, conv_b, head, spec, x)
    np.testing.assert_allclose(p.numpy(), p_ref.numpy(), rtol=0, atol=1e-5)
    np.testing.assert_allclose(v.numpy(), v_ref.numpy(), rtol=0, atol=1e-5)
    assert conv_w.dtype == torch.bfloat16 and conv_w.numel() == w32.numel()


def _pack_fp32(sd, spec):
    from omoknuni_quantum_b200.resnet import IN_PAD, _fold
    out = []

    def pk(w, cin_pad):
        k = torch.zeros(w.shape[0], 3, 3, cin_pad)
        k[..., :w.shape[1]] = w.permute(0, 2, 3, 1)
        return k.reshape(w.shape[0], -1)
    out.append(pk(_fold(sd, "conv_input", "bn_input")[0], IN_PAD))
    for i in range(spec.num_blocks):
        for c, n in (("conv1", "bn1"), ("conv2", "bn2")):
            out.append(pk(_fold(sd, f"residual_blocks.{i}.{c}", f"residual_blocks.{i}.{n}")[0], spec.filters))
    return out


def test_flops_per_position_config1():
    from omoknuni_quantum_b200.resnet import ResNetSpec
    s = ResNetSpec(num_blocks=10, filters=128, fc_value_hidden=128)
    # trunk of benchmark config 1 (10 x 128, 15x15): ~1.34 GFLOP per position
    assert 1.30e9 < s.flops_per_position() < 1.36e9
