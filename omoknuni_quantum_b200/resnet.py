"""ResNet policy/value evaluator on B200 (tcgen05 bf16 implicit-GEMM trunk, fused epilogues).

Architecture and parameter names follow the reference's ResNetModel
(python/mcts/neural_networks/resnet_model.py:26-271): input 3x3 conv + BN + ReLU, residual
blocks (conv-BN-ReLU-conv-BN-add-ReLU), policy head (1x1 conv to 2 channels, BN, ReLU,
FC(2HW -> fc_policy_hidden), ReLU, FC(-> actions), log_softmax) and value head (1x1 conv to 1
channel, BN, ReLU, FC(HW -> fc_value_hidden), ReLU, FC(-> 1), tanh). A reference ``state_dict``
loads unchanged. The evaluator returns probabilities, as ResNetEvaluator does
(resnet_evaluator.py:254-257: exp of the log-softmax).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Dict

import torch
import torch.nn.functional as F

from . import _lib
from .engine import WaveEngine, _stream_ptr

BN_EPS = 1e-5
IN_PAD = 64


def in_pad(input_channels: int) -> int:
    """Input channels padded to one 64-channel K block, or two for more than 64 planes (chess)."""
    return IN_PAD if input_channels <= IN_PAD else 2 * IN_PAD


@dataclass(frozen=True)
class ResNetSpec:
    board_size: int = 15
    input_channels: int = 19
    num_blocks: int = 10
    filters: int = 128
    num_actions: int = 225
    fc_policy_hidden: int = 256
    fc_value_hidden: int = 256

    @property
    def hw(self) -> int:
        return self.board_size ** 2

    def flops_per_position(self) -> int:
        """Dense multiply-add FLOPs of one forward (2 per MAC), conv trunk + heads."""
        HW, C, Cin = self.hw, self.filters, self.input_channels
        trunk = 2 * HW * 9 * (Cin * C + 2 * self.num_blocks * C * C)
        heads = 2 * HW * C * 3 + 2 * (2 * HW * self.fc_policy_hidden + self.fc_policy_hidden * self.num_actions
                                      + HW * self.fc_value_hidden + self.fc_value_hidden)
        return trunk + heads


def spec_from_state_dict(sd: Dict[str, torch.Tensor], board_size: int) -> ResNetSpec:
    nb = len({k.split(".")[1] for k in sd if k.startswith("residual_blocks.")})
    return ResNetSpec(board_size=board_size, input_channels=sd["conv_input.weight"].shape[1],
                      num_blocks=nb, filters=sd["conv_input.weight"].shape[0],
                      num_actions=sd["policy_head.fc2.weight"].shape[0],
                      fc_policy_hidden=sd["policy_head.fc1.weight"].shape[0],
                      fc_value_hidden=sd["value_head.fc1.weight"].shape[0])


def init_state_dict(spec: ResNetSpec, seed: int = 0) -> Dict[str, torch.Tensor]:
    """Seeded random weights in the reference's state_dict layout, initialised the way
    ResNetModel._initialize_weights / the head initialisers do (resnet_model.py:72-88,
    125-137, 219-244): He-normal (fan_in, ReLU) convolutions, BN weight ~ N(1, 0.02),
    Xavier-normal linear layers (policy fc2 gain 0.1), small-normal value head."""
    g = torch.Generator().manual_seed(seed)
    C, Cin, HW, A = spec.filters, spec.input_channels, spec.hw, spec.num_actions
    Hp, Hv = spec.fc_policy_hidden, spec.fc_value_hidden
    sd: Dict[str, torch.Tensor] = {}

    def he(shape):
        fan_in = shape[1] * shape[2] * shape[3]
        return torch.randn(shape, generator=g) * math.sqrt(2.0 / fan_in)

    def xavier(shape, gain=1.0):
        return torch.randn(shape, generator=g) * gain * math.sqrt(2.0 / (shape[0] + shape[1]))

    def bn(prefix, n):
        sd[prefix + ".weight"] = 1.0 + 0.02 * torch.randn(n, generator=g)
        sd[prefix + ".bias"] = torch.zeros(n)
        sd[prefix + ".running_mean"] = torch.zeros(n)
        sd[prefix + ".running_var"] = torch.ones(n)
        sd[prefix + ".num_batches_tracked"] = torch.zeros((), dtype=torch.long)

    sd["conv_input.weight"] = he((C, Cin, 3, 3)) + 0.01 * torch.randn((C, Cin, 3, 3), generator=g)
    bn("bn_input", C)
    for i in range(spec.num_blocks):
        sd[f"residual_blocks.{i}.conv1.weight"] = he((C, C, 3, 3))
        bn(f"residual_blocks.{i}.bn1", C)
        sd[f"residual_blocks.{i}.conv2.weight"] = he((C, C, 3, 3))
        bn(f"residual_blocks.{i}.bn2", C)
    sd["policy_head.conv.weight"] = he((2, C, 1, 1))
    bn("policy_head.bn", 2)
    sd["policy_head.fc1.weight"] = xavier((Hp, 2 * HW))
    sd["policy_head.fc1.bias"] = torch.zeros(Hp)
    sd["policy_head.fc2.weight"] = xavier((A, Hp), gain=0.1)
    sd["policy_head.fc2.bias"] = torch.zeros(A)
    sd["value_head.conv.weight"] = he((1, C, 1, 1))
    bn("value_head.bn", 1)
    sd["value_head.fc1.weight"] = xavier((Hv, HW))
    sd["value_head.fc1.bias"] = torch.zeros(Hv)
    sd["value_head.fc2.weight"] = xavier((1, Hv))
    sd["value_head.fc2.bias"] = torch.zeros(1)
    return sd


def _fold(sd, conv, bn):
    w = sd[conv + ".weight"].float()
    s = sd[bn + ".weight"].float() / torch.sqrt(sd[bn + ".running_var"].float() + BN_EPS)
    b = sd[bn + ".bias"].float() - sd[bn + ".running_mean"].float() * s
    return w * s.view(-1, *([1] * (w.dim() - 1))), b


def reference_forward_fp32(sd: Dict[str, torch.Tensor], x: torch.Tensor):
    """fp32 eval-mode forward of the reference architecture (the parity reference of the bf16
    kernels): returns (policy probabilities [B, A], value [B])."""
    def bn(t, p):
        return F.batch_norm(t, sd[p + ".running_mean"].float(), sd[p + ".running_var"].float(),
                            sd[p + ".weight"].float(), sd[p + ".bias"].float(), False, 0.0, BN_EPS)
    x = x.float()
    h = F.relu(bn(F.conv2d(x, sd["conv_input.weight"].float(), padding=1), "bn_input"))
    i = 0
    while f"residual_blocks.{i}.conv1.weight" in sd:
        p = f"residual_blocks.{i}."
        o = F.relu(bn(F.conv2d(h, sd[p + "conv1.weight"].float(), padding=1), p + "bn1"))
        o = bn(F.conv2d(o, sd[p + "conv2.weight"].float(), padding=1), p + "bn2")
        h = F.relu(o + h)
        i += 1
    B = h.shape[0]
    pp = F.relu(bn(F.conv2d(h, sd["policy_head.conv.weight"].float()), "policy_head.bn")).reshape(B, -1)
    pp = F.relu(F.linear(pp, sd["policy_head.fc1.weight"].float(), sd["policy_head.fc1.bias"].float()))
    logp = F.log_softmax(F.linear(pp, sd["policy_head.fc2.weight"].float(), sd["policy_head.fc2.bias"].float()), dim=1)
    vv = F.relu(bn(F.conv2d(h, sd["value_head.conv.weight"].float()), "value_head.bn")).reshape(B, -1)
    vv = F.relu(F.linear(vv, sd["value_head.fc1.weight"].float(), sd["value_head.fc1.bias"].float()))
    v = torch.tanh(F.linear(vv, sd["value_head.fc2.weight"].float(), sd["value_head.fc2.bias"].float()))
    return torch.exp(logp), v.reshape(B)


DTYPES = {"bf16": (_lib.OMQ_DTYPE_BF16, torch.bfloat16), "fp16": (_lib.OMQ_DTYPE_F16, torch.float16)}


def pack_parameters(sd: Dict[str, torch.Tensor], spec: ResNetSpec, dtype: str = "bf16"):
    """Fold BatchNorm and lay the parameters out as omq_resnet_load expects
    (conv_w in the net's 16-bit dtype, conv_b fp32, head fp32; see include/omq_b200.h)."""
    C = spec.filters
    ws, bs = [], []

    def pack_conv(w, cin_pad):
        cout, cin = w.shape[0], w.shape[1]
        k = torch.zeros(cout, 3, 3, cin_pad)
        k[..., :cin] = w.permute(0, 2, 3, 1)
        return k.reshape(cout, 9 * cin_pad)

    w, b = _fold(sd, "conv_input", "bn_input")
    ws.append(pack_conv(w, in_pad(spec.input_channels))); bs.append(b)
    for i in range(spec.num_blocks):
        p = f"residual_blocks.{i}."
        for c, n in (("conv1", "bn1"), ("conv2", "bn2")):
            w, b = _fold(sd, p + c, p + n)
            ws.append(pack_conv(w, C)); bs.append(b)
    conv_w = torch.cat([x.reshape(-1) for x in ws]).to(DTYPES[dtype][1])
    conv_b = torch.cat(bs).float()
    wp, bp = _fold(sd, "policy_head.conv", "policy_head.bn")
    wv, bv = _fold(sd, "value_head.conv", "value_head.bn")
    head = torch.cat([
        torch.cat([wp.reshape(2, C), wv.reshape(1, C)]).reshape(-1), torch.cat([bp, bv]),
        sd["policy_head.fc1.weight"].float().t().contiguous().reshape(-1), sd["policy_head.fc1.bias"].float(),
        sd["policy_head.fc2.weight"].float().t().contiguous().reshape(-1), sd["policy_head.fc2.bias"].float(),
        sd["value_head.fc1.weight"].float().t().contiguous().reshape(-1), sd["value_head.fc1.bias"].float(),
        sd["value_head.fc2.weight"].float().reshape(-1), sd["value_head.fc2.bias"].float(),
    ])
    return conv_w, conv_b, head


class ResNetEvaluator:
    """tcgen05 ResNet on one GPU. ``evaluate_batch(features)`` keeps the reference
    protocol (features [B, C, n, n] -> probabilities [B, A], values [B]); inside the device
    search the engine calls ``forward_queue`` instead, which packs the queued leaves on the
    device and writes the queue's result buffers without a host round trip.

    ``dtype`` is the 16-bit type of the weights, activations and dense-layer operands (fp32
    accumulation either way): "bf16" (default; the benchmark configs' type) or "fp16", the
    precision of the reference evaluator's autocast (resnet_evaluator.py:247-249). fp16 keeps 3
    more mantissa bits, which is what keeps a 20-block trunk within 2e-2 of an fp32 forward; like
    the reference's autocast it overflows above 65504."""

    def __init__(self, state_dict: Dict[str, torch.Tensor], board_size: int = 15,
                 max_batch: int = 4096, device=None, dtype: str = "bf16", trunk: str = "auto"):
        if not torch.cuda.is_available():
            raise RuntimeError("ResNetEvaluator needs a CUDA device (B200); there is no CPU fallback")
        if dtype not in DTYPES:
            raise ValueError(f"dtype must be one of {sorted(DTYPES)}")
        self.dtype = dtype
        if trunk not in ("auto", "per_layer"):
            raise ValueError("trunk is 'auto' (the whole-trunk kernel where it applies) or 'per_layer'")
        self.trunk = trunk
        self.spec = spec_from_state_dict(state_dict, board_size)
        self.state_dict = {k: v.detach().cpu() for k, v in state_dict.items()}
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.L = _lib.load()
        self._net = None
        self._max_batch = 0
        self.generation = 0     # bumped whenever the device net (and its buffers) is re-created
        self.profiling = False  # CUDA-event timing of forward calls on (no graph capture then)
        self._ensure(max_batch)
        self._return_torch_tensors = True

    @classmethod
    def from_module(cls, module: torch.nn.Module, **kw) -> "ResNetEvaluator":
        board = getattr(module, "board_size", 15)
        return cls(module.state_dict(), board_size=board, **kw)

    @classmethod
    def random(cls, spec: ResNetSpec, seed: int = 0, **kw) -> "ResNetEvaluator":
        return cls(init_state_dict(spec, seed), board_size=spec.board_size, **kw)

    def _ensure(self, max_batch: int) -> None:
        if self._net is not None and max_batch <= self._max_batch:
            return
        self.close()
        s = self.spec
        cfg = _lib.ResNetConfig(s.board_size, s.input_channels, s.num_blocks, s.filters, s.num_actions,
                                s.fc_policy_hidden, s.fc_value_hidden, int(max_batch), self.device.index or 0,
                                DTYPES[self.dtype][0], int(self.trunk == "per_layer"))
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(self.L.omq_resnet_create(ctypes.byref(cfg), ctypes.byref(h)), "omq_resnet_create")
            self._net = h
            self._max_batch = int(max_batch)
            self.generation += 1
            conv_w, conv_b, head = pack_parameters(self.state_dict, s, self.dtype)
            a, b, c = (ctypes.c_uint64() for _ in range(3))
            _lib.check(self.L.omq_resnet_param_sizes(h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c)),
                       "omq_resnet_param_sizes")
            if (a.value, b.value, c.value) != (conv_w.numel(), conv_b.numel(), head.numel()):
                raise RuntimeError("parameter packing does not match the native layout")
            self._params = [t.to(self.device).contiguous() for t in (conv_w, conv_b, head)]
            _lib.check(self.L.omq_resnet_load(h, *[ctypes.c_void_p(t.data_ptr()) for t in self._params],
                                              _stream_ptr()), "omq_resnet_load")

    def close(self):
        if getattr(self, "_net", None) is not None and self._net.value:
            self.L.omq_resnet_destroy(self._net)
        self._net = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def memory_bytes(self) -> int:
        b = ctypes.c_uint64()
        _lib.check(self.L.omq_resnet_memory(self._net, ctypes.byref(b)), "omq_resnet_memory")
        return int(b.value)

    @torch.no_grad()
    def evaluate_batch(self, features):
        x = torch.as_tensor(features).to(self.device, torch.float32).contiguous()
        B = x.shape[0]
        self._ensure(max(B, 1))
        policy = torch.empty(B, self.spec.num_actions, dtype=torch.float32, device=self.device)
        value = torch.empty(B, dtype=torch.float32, device=self.device)
        if B:
            _lib.check(self.L.omq_resnet_forward_features(self._net, ctypes.c_void_p(x.data_ptr()), B,
                                                          ctypes.c_void_p(policy.data_ptr()),
                                                          ctypes.c_void_p(value.data_ptr()), _stream_ptr()),
                       "omq_resnet_forward_features")
        return policy, value

    def forward_queue(self, engine: WaveEngine, queue: int) -> None:
        self._ensure(engine.queue_capacity)
        _lib.check(self.L.omq_resnet_forward_queue(self._net, engine._h, int(queue), _stream_ptr()),
                   "omq_resnet_forward_queue")

    def profile(self, capacity: int) -> None:
        """Time the convolution trunk of the next ``capacity`` forward calls with CUDA events."""
        _lib.check(self.L.omq_resnet_profile(self._net, int(capacity)), "omq_resnet_profile")
        self.profiling = int(capacity) > 0

    def profile_read(self, max_calls: int = 1 << 16):
        """(trunk_ms [calls], positions [calls]) of the profiled calls (synchronizes)."""
        import numpy as np
        n = ctypes.c_int32()
        ms = np.zeros(max_calls, np.float32)
        cnt = np.zeros(max_calls, np.int32)
        _lib.check(self.L.omq_resnet_profile_read(self._net, ctypes.byref(n), ms.ctypes.data,
                                                  cnt.ctypes.data, max_calls), "omq_resnet_profile_read")
        return ms[:n.value], cnt[:n.value]

    @property
    def conv_launches_per_call(self) -> int:
        """Trunk kernel launches per forward: 1 for the whole-trunk kernel (15x15 boards, 128
        filters), else one per conv."""
        n = ctypes.c_int32()
        _lib.check(self.L.omq_resnet_trunk_launches(self._net, ctypes.byref(n)), "omq_resnet_trunk_launches")
        return int(n.value)

    @property
    def fused_trunk(self) -> bool:
        return self.conv_launches_per_call == 1

    def trunk_flops_per_position(self) -> int:
        s = self.spec
        return 2 * s.hw * 9 * (s.input_channels * s.filters + 2 * s.num_blocks * s.filters * s.filters)

    def error(self) -> int:
        e = ctypes.c_int32()
        _lib.check(self.L.omq_resnet_error(self._net, ctypes.byref(e), _stream_ptr()), "omq_resnet_error")
        return int(e.value)
