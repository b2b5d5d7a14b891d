"""GPU parity of the device wave search against the reference fixtures and the oracle.

Bit-exact: visit counts, value sums, priors, virtual-loss counts, parent ids, parent actions,
the implied children table, the root policy and the final move.
"""
import hashlib

import numpy as np
import pytest
import torch

from golden_cases import ReplayEvaluator, children_table, digest, float_names, load, load_float, names

pytestmark = pytest.mark.gpu


def _engine(g, trees=1, **kw):
    from omoknuni_quantum_b200.engine import WaveEngine
    return WaveEngine(trees, capacity=int(g["capacity"]), max_wave_size=int(g["wave"]),
                      c_puct=float(g["c_puct"]), virtual_loss=float(g["virtual_loss"]),
                      enable_virtual_loss=bool(g["enable_vl"]), **kw)


def _assert_tree_matches(t, g):
    assert t["visits"].shape[0] == int(g["num_nodes"])
    for k in ("visits", "value_sums", "priors", "virtual_loss", "parent", "action"):
        assert digest(t[k]) == str(g["sha_" + k]), k
    assert digest(children_table(t["parent"], t["action"])) == str(g["sha_children"])


@pytest.mark.parametrize("name", names())
def test_search_matches_reference_fixture(name):
    g = load(name)
    eng = _engine(g)
    boards = torch.from_numpy(g["board"][None]).cuda()
    eng.search(boards, int(g["sims"]))
    t = eng.export_tree(0)
    _assert_tree_matches(t, g)
    visits = eng.root_visits()[0].cpu().numpy()
    pol = eng.policy_from_visits(visits)
    assert np.array_equal(pol, g["policy"])
    assert int(np.argmax(pol)) == int(g["final_move"])


def test_multi_tree_lockstep_matches_oracle(oracle_lib):
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.roots import random_roots
    R, sims, wave = 6, 300, 64
    roots = random_roots(11, R)
    roots[2] = 0                                  # an empty root in the same batch
    eng = WaveEngine(R, capacity=120000, max_wave_size=wave)
    eng.search(torch.from_numpy(roots).cuda(), sims)
    visits = eng.root_visits().cpu().numpy()
    for r in range(R):
        o = oracle_lib.Oracle(120000).search(roots[r], sims, wave)
        t = eng.export_tree(r)
        assert np.array_equal(t["visits"], o.visits)
        assert np.array_equal(t["value_sums"], o.value_sums)
        assert np.array_equal(t["parent"], o.parent) and np.array_equal(t["action"], o.action)
        assert np.array_equal(eng.policy_from_visits(visits[r]), o.policy)


def _edge_roots():
    """A root that already holds five in a row, a board with three empty cells and no five (runs
    of at most two in every direction), a random root and the empty board."""
    from omoknuni_quantum_b200.roots import random_roots
    r = random_roots(23, 4)
    r[0, 7, 2:7] = 1                              # five for black, and one more white stone
    r[0, 3, 3] = 2
    y, x = np.mgrid[0:15, 0:15]
    full = (1 + ((x // 2 + y) % 2)).astype(np.int8)
    full[0, 0] = full[7, 7] = full[14, 5] = 0
    r[1] = full
    r[3] = 0
    return r


@pytest.mark.parametrize("sims,wave", [(300, 64), (5, 64), (64, 64)])
def test_edge_roots_and_short_searches_match_oracle(oracle_lib, sims, wave):
    """Roots the reference searches without special cases (a decided board: every child is
    terminal; a nearly full board: children reach the full board), and searches shorter than one
    wave or exactly one wave, against the oracle."""
    from omoknuni_quantum_b200.engine import WaveEngine
    roots = _edge_roots()
    eng = WaveEngine(4, capacity=80000, max_wave_size=wave)
    eng.search(torch.from_numpy(roots).cuda(), sims)
    visits = eng.root_visits().cpu().numpy()
    assert visits[1].sum() == sims and np.count_nonzero(visits[1]) <= 3
    for r in range(4):
        o = oracle_lib.Oracle(80000).search(roots[r], sims, wave)
        t = eng.export_tree(r)
        for k, ok in (("visits", o.visits), ("value_sums", o.value_sums), ("priors", o.priors),
                      ("parent", o.parent), ("action", o.action)):
            assert np.array_equal(t[k], ok), (r, k)
        assert np.array_equal(eng.policy_from_visits(visits[r]), o.policy)


class _RecordingTorchEvaluator:
    """A float-valued evaluator on the GPU (fixed random linear policy/value heads on the
    features). Records every output keyed by the feature bytes so that the oracle can replay
    exactly the same evaluator outputs."""

    def __init__(self, seed=0):
        g = torch.Generator().manual_seed(seed)
        self.wp = (torch.randn(19 * 225, 225, generator=g) * 0.05).cuda()
        self.wv = (torch.randn(19 * 225, generator=g) * 0.05).cuda()
        self.table = {}

    def evaluate_batch(self, feats):
        x = feats.reshape(feats.shape[0], -1)
        logits = x @ self.wp
        pol = torch.softmax(logits, dim=1)
        val = torch.tanh(x @ self.wv)
        fc = feats.cpu().numpy().astype(np.float32)
        pc, vc = pol.cpu().numpy(), val.cpu().numpy()
        for i in range(fc.shape[0]):
            self.table[hashlib.sha256(fc[i].tobytes()).digest()] = (pc[i].copy(), vc[i])
        return pol, val

    def replay(self, feats):
        n = feats.shape[0]
        p = np.zeros((n, 225), np.float32)
        v = np.zeros(n, np.float32)
        for i in range(n):
            p[i], v[i] = self.table[hashlib.sha256(np.ascontiguousarray(feats[i], np.float32).tobytes()).digest()]
        return p, v


def test_float_evaluator_replay_is_bit_exact(oracle_lib):
    """Same evaluator outputs -> identical trees, W included (fp32 sums in the reference's
    per-simulation order)."""
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.roots import random_root
    board = random_root(21)
    ev = _RecordingTorchEvaluator()
    eng = WaveEngine(1, capacity=150000, max_wave_size=128)
    eng.search(torch.from_numpy(board[None]).cuda(), 640, evaluator=ev)
    t = eng.export_tree(0)
    o = oracle_lib.Oracle(150000).search(board, 640, 128, evaluator=ev.replay)
    assert o.result["boundary_ties"] == 0
    assert np.array_equal(t["parent"], o.parent) and np.array_equal(t["action"], o.action)
    assert np.array_equal(t["priors"], o.priors)
    assert np.array_equal(t["visits"], o.visits)
    assert np.array_equal(t["value_sums"], o.value_sums)


def test_generic_evaluator_path_equals_builtin_synthetic(oracle_lib):
    """The reference evaluator protocol (features -> evaluate_batch) gives the same tree as the
    built-in synthetic kernel, and the device features equal the oracle's feature tensors."""
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.roots import random_root
    board = random_root(5)

    class NumpySynth:
        def evaluate_batch(self, f):
            return oracle_lib.synth_eval(f.cpu().numpy())

    e1 = WaveEngine(1, capacity=80000, max_wave_size=64)
    e1.search(torch.from_numpy(board[None]).cuda(), 256, evaluator=NumpySynth())
    e2 = WaveEngine(1, capacity=80000, max_wave_size=64)
    e2.search(torch.from_numpy(board[None]).cuda(), 256)
    a, b = e1.export_tree(0), e2.export_tree(0)
    for k in a:
        assert np.array_equal(a[k], b[k]), k


def test_tree_full_raises():
    from omoknuni_quantum_b200._lib import TreeFullError
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.roots import random_root
    eng = WaveEngine(1, capacity=5000, max_wave_size=256)
    with pytest.raises(TreeFullError, match="Tree full"):
        eng.search(torch.from_numpy(random_root(0)[None]).cuda(), 800)


def test_virtual_loss_is_reverted_every_wave():
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.roots import random_root
    eng = WaveEngine(1, capacity=100000, max_wave_size=128)
    eng.begin(torch.from_numpy(random_root(3)[None]).cuda())
    eng.root_expand()
    for _ in range(3):
        eng.wave(128)
        t = eng.export_tree(0)
        assert (t["virtual_loss"] == 0).all()
        assert t["visits"][0] == t["visits"][t["parent"] == 0].sum()


def test_selfplay_moves_match_oracle(oracle_lib):
    """Each move's policy in batched device self-play equals the oracle's search of that board."""
    from omoknuni_quantum_b200.selfplay import BatchedSelfPlay
    sp = BatchedSelfPlay(4, num_simulations=96, wave_size=32, capacity=40000, seed=3)
    recs = sp.play(3)
    for r in recs:
        for ex in r.examples:
            o = oracle_lib.Oracle(40000).search(ex["state"], 96, 32)
            assert np.array_equal(ex["policy"], o.policy)


def test_root_dirichlet_noise_replays_bit_exact_in_oracle(oracle_lib):
    """With eps > 0 every wave mixes a fresh Dirichlet vector into the root priors. Replaying the
    vector each device wave drew makes the oracle's tree identical; the vectors are proper
    distributions over the root's children, differ between waves, and repeat for a fixed seed."""
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.roots import random_root
    board = random_root(8)
    eps, wave, waves = 0.25, 64, 4

    def run(seed):
        eng = WaveEngine(1, capacity=60000, max_wave_size=wave, dirichlet_alpha=0.3,
                         dirichlet_epsilon=eps, noise_seed=seed)
        eng.begin(torch.from_numpy(board[None]).cuda())
        eng.root_expand()
        noise = []
        for _ in range(waves):
            eng.wave(wave)
            noise.append(eng.root_noise()[0].cpu().numpy())
        return eng, noise

    eng, noise = run(123)
    o = oracle_lib.Oracle(60000)
    assert o.begin(board, o.config(waves * wave, wave)) == 0
    for nz in noise:
        assert o.wave(wave, root_noise=nz, eps=eps) == 0
    t, ot = eng.export_tree(0), o.export()
    for k in ("visits", "value_sums", "priors", "parent", "action"):
        assert np.array_equal(t[k], getattr(ot, k)), k
    legal = board.reshape(-1) == 0
    for nz in noise:
        assert abs(nz.sum() - 1.0) < 1e-5 and (nz >= 0).all() and (nz[~legal] == 0).all()
    assert not np.array_equal(noise[0], noise[1])
    _, again = run(123)
    _, other = run(124)
    assert all(np.array_equal(a, b) for a, b in zip(noise, again))
    assert not np.array_equal(noise[0], other[0])
    # without noise the same waves reproduce the noiseless oracle
    e0 = WaveEngine(1, capacity=60000, max_wave_size=wave, dirichlet_epsilon=0.0)
    e0.search(torch.from_numpy(board[None]).cuda(), waves * wave)
    o0 = oracle_lib.Oracle(60000).search(board, waves * wave, wave)
    assert np.array_equal(e0.export_tree(0)["visits"], o0.visits)


def test_cuda_graph_waves_equal_plain_waves():
    """WaveEngine.search(graphs=True) replays a captured wave: identical trees to the plain
    launches, for several searches in a row and a partial last wave; the launch counter counts
    each replay's kernels once."""
    from omoknuni_quantum_b200 import _lib
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, ResNetSpec
    from omoknuni_quantum_b200.roots import random_root
    ev = ResNetEvaluator.random(ResNetSpec(num_blocks=2, filters=128), seed=5, max_batch=512)
    b = torch.from_numpy(np.stack([random_root(70 + i) for i in range(2)])).cuda()
    plain, graph = WaveEngine(2, capacity=80000, max_wave_size=64), WaveEngine(2, capacity=80000, max_wave_size=64)
    for sims in (200, 256, 200):
        n0 = _lib.kernel_launches()
        plain.search(b, sims, ev)
        n_plain = _lib.kernel_launches() - n0
        n0 = _lib.kernel_launches()
        graph.search(b, sims, ev, graphs=True)
        n_graph = _lib.kernel_launches() - n0
        for r in range(2):
            a, c = plain.export_tree(r), graph.export_tree(r)
            for k in ("parent", "action", "priors", "visits", "value_sums", "terminal"):
                assert np.array_equal(a[k], c[k]), (sims, k)
        # the one-call search (omq_search) reads the tree headers with one copy at its end; the
        # host-sequenced graph path checks them with one k_status launch
        assert n_graph == n_plain + 1, (n_graph, n_plain)
    assert len(graph._graphs) == 1


def test_bounded_wait_times_out_and_context_stays_usable(oracle_lib):
    """A device wait that can never complete (an mbarrier nothing arrives on) gives up after its
    limit and reports OMQ_TIMEOUT through device memory; the context then runs a normal search."""
    import ctypes
    import time
    from omoknuni_quantum_b200 import _lib
    from omoknuni_quantum_b200.engine import WaveEngine, _stream_ptr
    from omoknuni_quantum_b200.roots import random_root
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    t0 = time.perf_counter()
    _lib.check(_lib.load().omq_selftest_wait_timeout(20_000_000, ctypes.c_void_p(status.data_ptr()),
                                                     _stream_ptr()), "omq_selftest_wait_timeout")
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(status.item()) == 3            # OMQ_TIMEOUT
    assert 0.015 < dt < 5.0
    board = random_root(77)
    eng = WaveEngine(1, capacity=40000, max_wave_size=64)
    eng.search(torch.from_numpy(board[None]).cuda(), 128)
    o = oracle_lib.Oracle(40000).search(board, 128, 64)
    assert np.array_equal(eng.export_tree(0)["visits"], o.visits)


def test_warmup_and_update_with_move(oracle_lib):
    from omoknuni_quantum_b200 import MCTS, MCTSConfig, SyntheticEvaluator
    from omoknuni_quantum_b200.roots import random_root
    m = MCTS(MCTSConfig(num_simulations=192, max_wave_size=64, dirichlet_epsilon=0.0,
                        initial_tree_nodes=60000), SyntheticEvaluator())
    m.warmup(2, 64)
    assert m.get_statistics()["total_searches"] == 0
    b = random_root(88)
    p = m.search(b)
    assert np.array_equal(p, oracle_lib.Oracle(60000).search(b, 192, 64).policy)
    m.update_with_move(int(np.argmax(p)))


@pytest.mark.parametrize("n", [9, 19])
def test_gomoku_other_board_sizes_match_oracle(oracle_lib, n):
    """Gomoku on 9x9 and 19x19 (MCTSConfig.board_size): device trees equal the oracle's, and the
    ResNet on the (n+1)^2 padded grid matches the fp32 reference forward."""
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, ResNetSpec, init_state_dict, reference_forward_fp32
    from omoknuni_quantum_b200.roots import random_root
    boards = np.stack([random_root(300 + i, stones=10, board_size=n) for i in range(3)])
    eng = WaveEngine(3, board_size=n, capacity=100000, max_wave_size=64)
    eng.search(torch.from_numpy(boards).cuda(), 256)
    for r in range(3):
        o = oracle_lib.Oracle(100000, n).search(boards[r], 256, 64)
        t = eng.export_tree(r)
        for k in ("parent", "action", "priors", "visits", "value_sums", "terminal"):
            assert np.array_equal(t[k], getattr(o, k)), (n, r, k)
    spec = ResNetSpec(board_size=n, num_blocks=2, filters=128, num_actions=n * n)
    sd = init_state_dict(spec, seed=4)
    ev = ResNetEvaluator(sd, board_size=n, max_batch=256)
    g = np.random.default_rng(n)
    x = torch.zeros(100, 19, n, n)
    x[:, 0] = torch.from_numpy((g.random((100, n, n)) < 0.3).astype(np.float32))
    x[:, 1] = 1.0
    p, v = ev.evaluate_batch(x.cuda())
    pr, vr = reference_forward_fp32({k: t.cuda() for k, t in sd.items()}, x.cuda())
    assert (p - pr).abs().max().item() < 2e-2 and (v - vr).abs().max().item() < 2e-2


def test_backup_sign_convention_on_device():
    """test_mcts_phases_detailed.py:578-616 on the device through the evaluator protocol."""
    from omoknuni_quantum_b200.engine import WaveEngine

    class Const:
        def evaluate_batch(self, x):
            n = x.shape[0]
            return torch.full((n, 225), 1.0 / 225, device=x.device), torch.full((n,), 0.5, device=x.device)

    eng = WaveEngine(1, capacity=20000, max_wave_size=1)
    eng.search(torch.zeros(1, 15, 15, dtype=torch.int8).cuda(), 1, evaluator=Const())
    t = eng.export_tree(0)
    leaf = int(np.nonzero(t["visits"][1:])[0].max()) + 1
    child = int(t["parent"][leaf])
    assert t["parent"][child] == 0
    assert (t["value_sums"][0], t["value_sums"][child], t["value_sums"][leaf]) == (0.5, -0.5, 0.5)


@pytest.mark.parametrize("name", float_names())
def test_search_matches_reference_with_float_evaluator(name):
    """The reference searched with a float evaluator (an fp32 ResNet, outputs recorded per
    position); the engine fed the same outputs through the evaluator protocol builds the same tree
    bit for bit: priors (normalised with torch's CPU summation order), visit counts, value sums,
    the CSR layout, the root policy and the final move."""
    from omoknuni_quantum_b200.engine import WaveEngine
    g = load_float(name)
    ev = ReplayEvaluator(g)
    eng = WaveEngine(1, capacity=int(g["capacity"]), max_wave_size=int(g["wave"]))
    eng.search(torch.from_numpy(g["board"][None]).cuda(), int(g["sims"]), evaluator=ev)
    assert ev.misses == 0
    t = eng.export_tree(0)
    assert t["visits"].shape[0] == int(g["num_nodes"])
    for k in ("visits", "value_sums", "priors", "virtual_loss", "parent", "action"):
        assert digest(t[k]) == str(g["sha_" + k]), k
    assert digest(children_table(t["parent"], t["action"])) == str(g["sha_children"])
    pol = eng.policy_from_visits(eng.root_visits()[0].cpu().numpy())
    assert np.array_equal(pol, g["policy"]) and int(np.argmax(pol)) == int(g["final_move"])


def test_device_prior_sum_is_torchs_order():
    """The warp sum behind the prior normalisation equals torch.sum on the CPU bit for bit at
    every length up to 600 and at sampled lengths up to 5,000 (the 16-row cascade included)."""
    import ctypes
    from omoknuni_quantum_b200 import _lib
    rng = np.random.default_rng(3)
    lengths = list(range(0, 601)) + [int(n) for n in rng.integers(601, 5001, 200)]
    vals = [(rng.random(n) ** 3 * rng.choice([1e-3, 1.0, 3e4])).astype(np.float32) for n in lengths]
    offs = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    x = torch.from_numpy(np.concatenate(vals)).cuda()
    o = torch.from_numpy(offs).cuda()
    out = torch.full((len(lengths),), float("nan"), device="cuda")
    L = _lib.load()
    _lib.check(L.omq_selftest_prior_sum(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(o.data_ptr()),
                                        len(lengths), ctypes.c_void_p(out.data_ptr()),
                                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
               "omq_selftest_prior_sum")
    got = out.cpu().numpy()
    want = np.array([torch.from_numpy(v).sum().item() if len(v) else 0.0 for v in vals], np.float32)
    bad = [n for n, a, b in zip(lengths, got, want) if a != b]
    assert not bad, bad[:10]


@pytest.mark.parametrize("game,dtype", [("gomoku", "bf16"), ("go", "bf16"), ("chess", "bf16"), ("gomoku", "fp16")])
def test_one_call_search_equals_stepwise_search(game, dtype):
    """omq_search / omq_search_go / omq_search_chess (one C-ABI call: begin, root expansion and
    every wave with the tensor-core ResNet on the leaf queues) build the same trees as the same
    search sequenced step by step from the host (begin, root_expand, wave, ...)."""
    import ctypes
    from omoknuni_quantum_b200 import _lib
    from omoknuni_quantum_b200.engine import WaveEngine, _stream_ptr
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, ResNetSpec
    R, sims, wave = 3, 200, 64
    if game == "go":
        from omoknuni_quantum_b200.go import random_roots as go_roots
        hist, meta = go_roots(4, R, moves=40, board_size=19)
        boards, meta = torch.from_numpy(hist).cuda(), torch.from_numpy(meta)
        spec = ResNetSpec(board_size=19, input_channels=17, num_blocks=2, filters=256, num_actions=362)
        n = 19
    elif game == "chess":
        from omoknuni_quantum_b200.chess import random_position
        ps = [random_position(40 + i) for i in range(R)]
        boards = np.stack([p.root_records() for p in ps])
        meta = np.array([len(p.prior) for p in ps], np.int32)
        spec = ResNetSpec(board_size=8, input_channels=119, num_blocks=2, filters=128, num_actions=4672)
        n = 8
    else:
        from omoknuni_quantum_b200.roots import random_roots
        boards, meta = torch.from_numpy(random_roots(8, R)).cuda(), None
        spec = ResNetSpec(num_blocks=2, filters=128)
        n = 15
    ev = ResNetEvaluator.random(spec, seed=4, max_batch=R * wave, dtype=dtype)
    engines = [WaveEngine(R, board_size=n, capacity=80000, max_wave_size=wave, game=game)
               for _ in range(2)]
    a, b = engines
    # one call through the C ABI
    L = _lib.load()
    if game == "chess":
        rec, npr = a._chess_roots(boards, meta)
        st = L.omq_search_chess(a._h, ev._net, ctypes.c_void_p(rec.data_ptr()), ctypes.c_void_p(npr.data_ptr()),
                                sims, _stream_ptr())
    elif game == "go":
        h, m = a._go_roots(boards, meta)
        k, kc = a._go_keys(None)
        st = L.omq_search_go(a._h, ev._net, ctypes.c_void_p(h.data_ptr()), ctypes.c_void_p(m.data_ptr()),
                             ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(kc.data_ptr()), sims, _stream_ptr())
    else:
        st = L.omq_search(a._h, ev._net, ctypes.c_void_p(boards.data_ptr()), sims, _stream_ptr())
    _lib.check(st, "omq_search")
    # the same search step by step
    b.begin(boards, meta)
    b.root_expand(ev)
    done = 0
    while done < sims:
        w = min(wave, sims - done)
        b.wave(w, ev)
        done += w
    b.check_status()
    for r in range(R):
        ta, tb = a.export_tree(r), b.export_tree(r)
        assert ta["visits"].shape[0] > 1
        for key in ta:
            assert np.array_equal(ta[key], tb[key]), (r, key)
