"""ResNet on the B200: tcgen05 bf16 kernels against the fp32 restatement of the reference model
(tolerance 2e-2 absolute on policy probabilities and values), batch invariance, and the
device leaf-queue path against the host protocol path."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-2

# the fp32 reference forward runs on the GPU: keep its convolutions and matmuls in true fp32
torch.backends.cudnn.allow_tf32 = False
torch.backends.cuda.matmul.allow_tf32 = False


def _features(n, seed=0):
    """Reference-layout features of random legal-looking positions: occupancy, player plane,
    last move."""
    g = np.random.default_rng(seed)
    f = np.zeros((n, 19, 15, 15), np.float32)
    for i in range(n):
        occ = g.random((15, 15)) < g.uniform(0.05, 0.5)
        f[i, 0] = occ
        f[i, 1] = g.integers(1, 3)
        ys, xs = np.nonzero(occ)
        if len(ys):
            j = g.integers(len(ys))
            f[i, 2, ys[j], xs[j]] = 1
    return torch.from_numpy(f)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("blocks,filters,hv", [(10, 128, 128), (2, 256, 256)])
def test_forward_matches_fp32_reference(blocks, filters, hv, dtype):
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, ResNetSpec, init_state_dict, reference_forward_fp32
    spec = ResNetSpec(num_blocks=blocks, filters=filters, fc_value_hidden=hv)
    sd = init_state_dict(spec, seed=7)
    ev = ResNetEvaluator(sd, max_batch=512, dtype=dtype)
    x = _features(333, seed=blocks)
    p, v = ev.evaluate_batch(x.cuda())
    torch.cuda.synchronize()
    assert ev.error() == 0
    sd_gpu = {k: t.cuda() for k, t in sd.items()}
    pr, vr = reference_forward_fp32(sd_gpu, x.cuda())
    dp = (p - pr).abs().max().item()
    dv = (v - vr).abs().max().item()
    assert torch.isfinite(p).all() and torch.isfinite(v).all()
    assert dp < TOL and dv < TOL, (dp, dv)
    # the policy is a distribution
    assert torch.allclose(p.sum(1), torch.ones_like(p[:, 0]), atol=1e-4)


def _calibrate_bn(sd, x):
    """Running statistics of every BatchNorm set to the batch statistics of `x` as it flows
    through the net (what a trained checkpoint carries). Without them a 20-block He-initialised
    trunk grows its activations ~2x per block and every value saturates at +-1, which would make a
    tolerance check vacuous."""
    import torch.nn.functional as F
    from omoknuni_quantum_b200.resnet import BN_EPS
    sd = dict(sd)

    def bn(t, p):
        sd[p + ".running_mean"] = t.mean((0, 2, 3))
        sd[p + ".running_var"] = t.var((0, 2, 3))
        return F.batch_norm(t, sd[p + ".running_mean"], sd[p + ".running_var"], sd[p + ".weight"],
                            sd[p + ".bias"], False, 0.0, BN_EPS)
    h = F.relu(bn(F.conv2d(x, sd["conv_input.weight"], padding=1), "bn_input"))
    i = 0
    while f"residual_blocks.{i}.conv1.weight" in sd:
        p = f"residual_blocks.{i}."
        o = F.relu(bn(F.conv2d(h, sd[p + "conv1.weight"], padding=1), p + "bn1"))
        h = F.relu(bn(F.conv2d(o, sd[p + "conv2.weight"], padding=1), p + "bn2") + h)
        i += 1
    bn(F.conv2d(h, sd["policy_head.conv.weight"]), "policy_head.bn")
    bn(F.conv2d(h, sd["value_head.conv.weight"]), "value_head.bn")
    return sd


def _rounded_forward(sd, x, dt):
    """The fp32 forward with the trunk's weights (BatchNorm folded) and every activation the
    kernels store rounded to the 16-bit type `dt`: the error that rounding alone causes, with no
    kernel involved."""
    import torch.nn.functional as F
    from omoknuni_quantum_b200.resnet import _fold
    q = lambda t: t.to(dt).float()
    w, b = _fold(sd, "conv_input", "bn_input")
    h = q(F.relu(F.conv2d(q(x), q(w), padding=1) + b.view(1, -1, 1, 1)))
    i = 0
    while f"residual_blocks.{i}.conv1.weight" in sd:
        p = f"residual_blocks.{i}."
        w1, b1 = _fold(sd, p + "conv1", p + "bn1")
        w2, b2 = _fold(sd, p + "conv2", p + "bn2")
        o = q(F.relu(F.conv2d(h, q(w1), padding=1) + b1.view(1, -1, 1, 1)))
        h = q(F.relu(F.conv2d(o, q(w2), padding=1) + b2.view(1, -1, 1, 1) + h))
        i += 1
    B = h.shape[0]
    wp, bp = _fold(sd, "policy_head.conv", "policy_head.bn")
    wv, bv = _fold(sd, "value_head.conv", "value_head.bn")
    pp = F.relu(F.conv2d(h, wp) + bp.view(1, -1, 1, 1)).reshape(B, -1)
    pp = F.relu(F.linear(pp, sd["policy_head.fc1.weight"], sd["policy_head.fc1.bias"]))
    lp = F.log_softmax(F.linear(pp, sd["policy_head.fc2.weight"], sd["policy_head.fc2.bias"]), 1)
    vv = F.relu(F.conv2d(h, wv) + bv.view(1, -1, 1, 1)).reshape(B, -1)
    vv = F.relu(F.linear(vv, sd["value_head.fc1.weight"], sd["value_head.fc1.bias"]))
    v = torch.tanh(F.linear(vv, sd["value_head.fc2.weight"], sd["value_head.fc2.bias"]))
    return lp.exp(), v.reshape(B)


def _deep_case(game):
    from omoknuni_quantum_b200.resnet import ResNetSpec, init_state_dict
    n, planes, acts = {"gomoku": (15, 19, 225), "go": (19, 17, 362), "chess": (8, 119, 4672)}[game]
    hv = 128 if game == "gomoku" else 256
    spec = ResNetSpec(board_size=n, input_channels=planes, num_blocks=20, filters=256, num_actions=acts,
                      fc_value_hidden=hv)
    g = np.random.default_rng(21)
    x = torch.from_numpy((g.random((300, planes, n, n)) < 0.25).astype(np.float32)).cuda()
    x[:, -1] = torch.from_numpy(g.integers(0, 2, (300, 1, 1)).astype(np.float32)).cuda()
    sd = {k: t.cuda() for k, t in init_state_dict(spec, seed=9).items()}
    with torch.no_grad():
        sd = _calibrate_bn(sd, x[:128])
    # a peaked policy: logits of a few units (the initialiser's fc2 gain of 0.1 gives ~0.01)
    sd["policy_head.fc2.weight"] = sd["policy_head.fc2.weight"] * (30.0 * (acts / 225) ** 0.5)
    return n, acts, sd, x


@pytest.mark.parametrize("game", ["gomoku", "go", "chess"])
def test_deep_20x256_fp16_forward_matches_fp32_reference(game):
    """The model of configs 2-4 at full depth (20 blocks x 256 filters, 41 convolutions) in fp16,
    the reference evaluator's autocast precision, against the fp32 forward within the 2e-2 gate,
    on a few hundred positions of each game's shape, with BatchNorm statistics that keep the
    values inside (-1, 1) and the policy far from uniform."""
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, reference_forward_fp32
    n, acts, sd, x = _deep_case(game)
    ev = ResNetEvaluator({k: t.cpu() for k, t in sd.items()}, board_size=n, max_batch=300, dtype="fp16")
    p, v = ev.evaluate_batch(x)
    torch.cuda.synchronize()
    assert ev.error() == 0
    with torch.no_grad():
        pr, vr = reference_forward_fp32(sd, x)
    # the check means something: values spread inside (-1, 1), policies far from uniform
    assert vr.std().item() > 0.1 and (vr.abs() < 0.99).float().mean().item() > 0.9
    assert pr.max(1).values.median().item() > 5.0 / acts
    dp = (p - pr).abs().max().item()
    dv = (v - vr).abs().max().item()
    assert torch.isfinite(p).all() and torch.isfinite(v).all()
    assert dp < TOL and dv < TOL, (dp, dv)


@pytest.mark.parametrize("game", ["gomoku", "go", "chess"])
def test_deep_20x256_bf16_forward_error_is_the_rounding_error(game):
    """The same model in bf16 (the benchmark configs' type). bf16 keeps 8 significant bits, and
    over 41 convolutions the rounding of weights and stored activations alone moves the outputs
    by several 1e-2 from fp32 (measured by `_rounded_forward`, no kernel involved). The kernels
    must add no error of their own beyond that: their deviation from fp32 stays within 1.5x the
    rounding-only deviation (plus 5e-3)."""
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, reference_forward_fp32
    n, acts, sd, x = _deep_case(game)
    ev = ResNetEvaluator({k: t.cpu() for k, t in sd.items()}, board_size=n, max_batch=300, dtype="bf16")
    p, v = ev.evaluate_batch(x)
    torch.cuda.synchronize()
    assert ev.error() == 0
    with torch.no_grad():
        pr, vr = reference_forward_fp32(sd, x)
        pq, vq = _rounded_forward(sd, x, torch.bfloat16)
    ep, ev_ = (pq - pr).abs().max().item(), (vq - vr).abs().max().item()
    dp, dv = (p - pr).abs().max().item(), (v - vr).abs().max().item()
    assert torch.isfinite(p).all() and torch.isfinite(v).all()
    assert dp <= 1.5 * ep + 5e-3 and dv <= 1.5 * ev_ + 5e-3, (dp, ep, dv, ev_)


def test_forward_is_batch_invariant():
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, ResNetSpec
    ev = ResNetEvaluator.random(ResNetSpec(num_blocks=3, filters=128), seed=3, max_batch=512)
    x = _features(257, seed=5).cuda()
    p1, v1 = ev.evaluate_batch(x)
    perm = torch.randperm(257, generator=torch.Generator().manual_seed(0)).cuda()
    p2, v2 = ev.evaluate_batch(x[perm])
    assert torch.equal(p1[perm], p2) and torch.equal(v1[perm], v2)
    p3, v3 = ev.evaluate_batch(x[:5])
    assert torch.equal(p1[:5], p3) and torch.equal(v1[:5], v3)
    # a call large enough for the heads' 256-wide tiles (small calls take 128-wide fc1 tiles)
    big = ResNetEvaluator(ev.state_dict, max_batch=12000)
    xb = torch.cat([x, _features(12000 - 257, seed=6).cuda()])
    p4, v4 = big.evaluate_batch(xb)
    assert torch.equal(p1, p4[:257]) and torch.equal(v1, v4[:257])


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_queue_path_equals_protocol_path(dtype):
    """forward_queue (device packing from the tree) == evaluate_batch on the engine's reference
    feature tensor: identical trees."""
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, ResNetSpec
    from omoknuni_quantum_b200.roots import random_roots
    ev = ResNetEvaluator.random(ResNetSpec(num_blocks=2, filters=128), seed=1, max_batch=1024, dtype=dtype)

    class Protocol:
        def evaluate_batch(self, f):
            return ev.evaluate_batch(f)

    roots = torch.from_numpy(random_roots(4, 3)).cuda()
    e1 = WaveEngine(3, capacity=60000, max_wave_size=64)
    e1.search(roots, 192, evaluator=ev)
    e2 = WaveEngine(3, capacity=60000, max_wave_size=64)
    e2.search(roots, 192, evaluator=Protocol())
    for r in range(3):
        a, b = e1.export_tree(r), e2.export_tree(r)
        for k in a:
            assert np.array_equal(a[k], b[k]), (r, k)


def test_distinct_handles_from_concurrent_host_threads():
    """Engines and networks are thread-safe across distinct handles: two host threads, each with
    its own ResNet and search engine on its own stream, give the results of a sequential run."""
    import threading
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, ResNetSpec
    from omoknuni_quantum_b200.roots import random_root
    spec = ResNetSpec(num_blocks=2, filters=128)
    boards = [np.stack([random_root(90 + 4 * t + i) for i in range(4)]) for t in range(2)]

    def run(t, out):
        with torch.cuda.stream(torch.cuda.Stream()):
            ev = ResNetEvaluator.random(spec, seed=11, max_batch=1024)
            eng = WaveEngine(4, capacity=60000, max_wave_size=64)
            for _ in range(3):
                eng.search(torch.from_numpy(boards[t]).cuda(), 192, evaluator=ev)
            out[t] = eng.root_visits().cpu().numpy()
            torch.cuda.current_stream().synchronize()

    seq = {}
    for t in range(2):
        run(t, seq)
    par = {}
    th = [threading.Thread(target=run, args=(t, par)) for t in range(2)]
    for x in th:
        x.start()
    for x in th:
        x.join()
    for t in range(2):
        assert np.array_equal(seq[t], par[t]), t


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_whole_trunk_kernel_equals_per_layer_convs(dtype):
    """The whole-trunk kernel (15x15 boards, 128 filters: one launch per forward, activations in
    a per-CTA scratch) gives the same policies and values, bit for bit, as one conv launch per
    layer, on batches below, at and above one position per CTA pair."""
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, ResNetSpec, init_state_dict
    sd = init_state_dict(ResNetSpec(num_blocks=4, filters=128, fc_value_hidden=128), seed=8)
    fused = ResNetEvaluator(sd, max_batch=2000, dtype=dtype)
    layered = ResNetEvaluator(sd, max_batch=2000, dtype=dtype, trunk="per_layer")
    assert fused.conv_launches_per_call == 1 and layered.conv_launches_per_call == 9
    for n, seed in ((1, 21), (150, 22), (297, 23), (2000, 24)):
        x = _features(n, seed=seed).cuda()
        pf, vf = fused.evaluate_batch(x)
        pl, vl = layered.evaluate_batch(x)
        assert torch.equal(pf, pl) and torch.equal(vf, vl), n
    assert fused.error() == 0 and layered.error() == 0
    # 19x19 and 256 filters keep the per-layer kernel
    big = ResNetEvaluator(init_state_dict(ResNetSpec(num_blocks=1, filters=256, fc_value_hidden=128), seed=1),
                          max_batch=8)
    assert big.conv_launches_per_call == 3
