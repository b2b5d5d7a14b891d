"""The ResNet forward that allocates nothing (omq_resnet_forward_noalloc), called through the
C ABI the way a caller that must not let the library allocate would call it: every input and
output buffer belongs to the caller, and the library uses only its fixed built-in scratch array.
Such callers are processes whose own allocator owns the device heap, or latency-critical threads
where a cudaMalloc would synchronise the device. Its results must match the allocating entry
point (omq_resnet_forward_features) on two calls in a row, the second with a smaller batch so
that leftovers of the first call in the shared scratch cannot leak into it."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-2  # the tolerance of the other ResNet GPU tests


def _features(n, seed):
    g = np.random.default_rng(seed)
    f = np.zeros((n, 19, 15, 15), np.float32)
    f[:, 0] = g.random((n, 15, 15)) < 0.3
    f[:, 1] = g.integers(1, 3, (n, 1, 1))
    f[:, 2].reshape(n, -1)[np.arange(n), g.integers(0, 225, n)] = 1
    return torch.from_numpy(f).cuda()


def test_noalloc_forward_matches_allocating_forward():
    from omoknuni_quantum_b200 import _lib
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, ResNetSpec, init_state_dict, pack_parameters
    spec = ResNetSpec(num_blocks=3, filters=128, fc_value_hidden=128)
    sd = init_state_dict(spec, seed=11)
    ref = ResNetEvaluator(sd, max_batch=64)
    L = _lib.load()
    conv_w, conv_b, head = (t.cuda().contiguous() for t in pack_parameters(sd, spec))
    cfg = _lib.ResNetConfig(15, 19, spec.num_blocks, spec.filters, 225, spec.fc_policy_hidden,
                            spec.fc_value_hidden, 0, torch.cuda.current_device())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def call(x, p, v):
        return L.omq_resnet_forward_noalloc(ctypes.byref(cfg), ctypes.c_void_p(conv_w.data_ptr()),
                                            ctypes.c_void_p(conv_b.data_ptr()),
                                            ctypes.c_void_p(head.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                            x.shape[0], ctypes.c_void_p(p.data_ptr()),
                                            ctypes.c_void_p(v.data_ptr()), stream)

    for n, seed in ((30, 1), (7, 2)):
        x = _features(n, seed)
        p = torch.full((n, 225), float("nan"), device="cuda")
        v = torch.full((n,), float("nan"), device="cuda")
        _lib.check(call(x, p, v), "omq_resnet_forward_noalloc")
        torch.cuda.synchronize()
        pr, vr = ref.evaluate_batch(x)
        assert torch.isfinite(p).all() and torch.isfinite(v).all()
        assert (p - pr).abs().max().item() < TOL and (v - vr).abs().max().item() < TOL

    # a batch beyond the fixed scratch is refused with a clear message
    x = _features(37, 3)
    st = call(x, torch.empty(37, 225, device="cuda"), torch.empty(37, device="cuda"))
    assert st == _lib.OMQ_BAD_ARG
    assert b"scratch limit of 36" in L.omq_last_error()
