"""The ResNet forward that allocates nothing (omq_resnet_forward_noalloc), called through the
C ABI the way a caller that must not let the library allocate would call it: every input and
output buffer belongs to the caller, and the library uses only its fixed built-in scratch array.
Such callers are processes whose own allocator owns the device heap, or latency-critical threads
where a cudaMalloc would synchronise the device. Its results must match the allocating entry
point (omq_resnet_forward_features) and the fp32 restatement of the reference model on two calls
in a row, the second with a smaller batch so that leftovers of the first call in the shared
scratch cannot leak into it. Every game shape and both filter counts go through the fixed
scratch, and each shape's documented batch limit is enforced."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-2  # the tolerance of the other ResNet GPU tests

# (board size, input planes, actions) of Gomoku, Go and chess
SHAPES = {"gomoku": (15, 19, 225), "go": (19, 17, 362), "chess": (8, 119, 4672)}
SCRATCH = 8 << 20


def _limit(board, planes, filters):
    """Positions per call that the fixed 8 MiB scratch holds: the packed input plus three
    activation buffers per padded (n+1)^2 grid, bf16, and 1 KiB kept for the error word."""
    pad = 64 if planes <= 64 else 128
    return (SCRATCH - 1024) // ((board + 1) ** 2 * (pad + 3 * filters) * 2)


def _features(n, board, planes, seed):
    g = np.random.default_rng(seed)
    f = (g.random((n, planes, board, board)) < 0.25).astype(np.float32)
    f[:, -1] = g.integers(0, 2, (n, 1, 1))
    return torch.from_numpy(f).cuda()


@pytest.mark.parametrize("filters", [128, 256])
@pytest.mark.parametrize("game", ["gomoku", "go", "chess"])
def test_noalloc_forward_matches_allocating_forward(game, filters):
    from omoknuni_quantum_b200 import _lib
    from omoknuni_quantum_b200.resnet import (ResNetEvaluator, ResNetSpec, init_state_dict, pack_parameters,
                                              reference_forward_fp32)
    board, planes, actions = SHAPES[game]
    spec = ResNetSpec(board_size=board, input_channels=planes, num_blocks=2, filters=filters,
                      num_actions=actions, fc_value_hidden=128)
    sd = init_state_dict(spec, seed=11)
    limit = _limit(board, planes, filters)
    ref = ResNetEvaluator(sd, board_size=board, max_batch=limit + 1)
    L = _lib.load()
    conv_w, conv_b, head = (t.cuda().contiguous() for t in pack_parameters(sd, spec))
    dev = torch.cuda.current_device()
    cfg = _lib.ResNetConfig(board, planes, spec.num_blocks, filters, actions, spec.fc_policy_hidden,
                            spec.fc_value_hidden, 0, dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def call(x, p, v):
        return L.omq_resnet_forward_noalloc(ctypes.byref(cfg), ctypes.c_void_p(conv_w.data_ptr()),
                                            ctypes.c_void_p(conv_b.data_ptr()),
                                            ctypes.c_void_p(head.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                            x.shape[0], ctypes.c_void_p(p.data_ptr()),
                                            ctypes.c_void_p(v.data_ptr()), stream)

    for n, seed in ((limit, 1), (max(1, limit // 4), 2)):
        x = _features(n, board, planes, seed)
        p = torch.full((n, actions), float("nan"), device="cuda")
        v = torch.full((n,), float("nan"), device="cuda")
        _lib.check(call(x, p, v), "omq_resnet_forward_noalloc")
        err = ctypes.c_int32(-1)
        _lib.check(L.omq_resnet_noalloc_error(dev, ctypes.byref(err), stream), "omq_resnet_noalloc_error")
        assert err.value == _lib.OMQ_OK
        pr, vr = ref.evaluate_batch(x)
        assert torch.isfinite(p).all() and torch.isfinite(v).all()
        assert (p - pr).abs().max().item() < TOL and (v - vr).abs().max().item() < TOL
        pf, vf = reference_forward_fp32(sd, x.cpu())
        assert (p.cpu() - pf).abs().max().item() < TOL and (v.cpu() - vf).abs().max().item() < TOL

    # one position more than the fixed scratch holds is refused with a clear message
    x = _features(limit + 1, board, planes, 3)
    st = call(x, torch.empty(limit + 1, actions, device="cuda"), torch.empty(limit + 1, device="cuda"))
    assert st == _lib.OMQ_BAD_ARG
    assert f"scratch limit of {limit}".encode() in L.omq_last_error()


def test_noalloc_forward_in_fp16_matches_allocating_forward():
    """The fixed-scratch forward with fp16 weights and activations (omq_resnet_config.dtype =
    OMQ_DTYPE_F16) equals the allocating fp16 forward, on two calls in a row."""
    from omoknuni_quantum_b200 import _lib
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, ResNetSpec, init_state_dict, pack_parameters
    spec = ResNetSpec(num_blocks=2, filters=128, fc_value_hidden=128)
    sd = init_state_dict(spec, seed=12)
    ref = ResNetEvaluator(sd, max_batch=64, dtype="fp16")
    L = _lib.load()
    conv_w, conv_b, head = (t.cuda().contiguous() for t in pack_parameters(sd, spec, "fp16"))
    dev = torch.cuda.current_device()
    cfg = _lib.ResNetConfig(15, 19, spec.num_blocks, 128, 225, spec.fc_policy_hidden, spec.fc_value_hidden, 0, dev,
                            _lib.OMQ_DTYPE_F16)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for n, seed in ((30, 4), (9, 5)):
        x = _features(n, 15, 19, seed)
        p = torch.full((n, 225), float("nan"), device="cuda")
        v = torch.full((n,), float("nan"), device="cuda")
        _lib.check(L.omq_resnet_forward_noalloc(ctypes.byref(cfg), ctypes.c_void_p(conv_w.data_ptr()),
                                                ctypes.c_void_p(conv_b.data_ptr()), ctypes.c_void_p(head.data_ptr()),
                                                ctypes.c_void_p(x.data_ptr()), n, ctypes.c_void_p(p.data_ptr()),
                                                ctypes.c_void_p(v.data_ptr()), stream), "omq_resnet_forward_noalloc")
        pr, vr = ref.evaluate_batch(x)
        assert (p - pr).abs().max().item() < TOL and (v - vr).abs().max().item() < TOL


def test_noalloc_rejects_a_device_that_does_not_exist():
    from omoknuni_quantum_b200 import _lib
    L = _lib.load()
    err = ctypes.c_int32(0)
    st = L.omq_resnet_noalloc_error(torch.cuda.device_count() + 3, ctypes.byref(err), None)
    assert st == _lib.OMQ_BAD_ARG
    assert b"out of range" in L.omq_last_error()
