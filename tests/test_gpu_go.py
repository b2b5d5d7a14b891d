"""GPU parity of the device Go search (config 3's game) against the oracle's Go search.

Bit-exact on the same roots: tree shape (parent, action), visit counts, value sums, priors,
terminal flags and the root policy, with the built-in synthetic evaluator and with a float
evaluator whose outputs are replayed (which also proves the 17-plane features identical: the
replay table is keyed by the feature bytes)."""
import hashlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _roots(seed, count, moves, n):
    from omoknuni_quantum_b200.go import random_roots
    return random_roots(seed, count, moves=moves, board_size=n)


def _compare(eng, r, o):
    t = eng.export_tree(r)
    assert t["visits"].shape == o.visits.shape
    for k in ("parent", "action", "priors", "visits", "value_sums", "terminal"):
        assert np.array_equal(t[k], getattr(o, k)), k


@pytest.mark.parametrize("n,moves,sims,wave,cap", [(9, 30, 300, 64, 150000), (19, 60, 512, 128, 400000),
                                                  (13, 120, 200, 32, 150000)])
def test_go_search_matches_oracle(oracle_lib, n, moves, sims, wave, cap):
    from omoknuni_quantum_b200.engine import WaveEngine
    hist, meta = _roots(7 + n, 4, moves, n)
    eng = WaveEngine(4, board_size=n, capacity=cap, max_wave_size=wave, game="go")
    eng.search(torch.from_numpy(hist).cuda(), sims, meta=torch.from_numpy(meta))
    visits = eng.root_visits().cpu().numpy()
    for r in range(4):
        o = oracle_lib.Oracle(cap, n).search_go(hist[r], int(meta[r, 0]), sims, wave,
                                               ko=int(meta[r, 1]), passes=int(meta[r, 2]))
        assert o.result["status"] == 0
        _compare(eng, r, o)
        assert np.array_equal(eng.policy_from_visits(visits[r]), o.policy)


def test_go_ko_pass_and_terminal_roots(oracle_lib):
    """Roots with a live ko point, one pass already made (a pass child ends the game), and a
    finished game (two passes: no children)."""
    from omoknuni_quantum_b200.engine import WaveEngine, go_meta
    from omoknuni_quantum_b200.go import GoPosition
    n = 7
    g = GoPosition(n)
    for a in (1 * 7 + 1, 1 * 7 + 2, 0 * 7 + 2, 0 * 7 + 3, 2 * 7 + 2, 2 * 7 + 3, 3 * 7 + 0, 1 * 7 + 4):
        g.play(a)
    g.play(1 * 7 + 3)             # black captures the white stone at (1,2): white faces a ko
    roots = [g.copy()]
    p = g.copy(); p.play(p.pass_action); roots.append(p)
    q = p.copy(); q.play(q.pass_action); roots.append(q)
    hist = np.stack([x.history_planes() for x in roots])
    meta = np.stack([x.meta() for x in roots])
    eng = WaveEngine(3, board_size=n, capacity=60000, max_wave_size=32, game="go")
    eng.search(torch.from_numpy(hist).cuda(), 160, meta=torch.from_numpy(meta))
    for r, x in enumerate(roots):
        o = oracle_lib.Oracle(60000, n).search_go(hist[r], x.to_move, 160, 32, ko=x.ko, passes=x.passes)
        _compare(eng, r, o)
    t2 = eng.export_tree(2)
    assert t2["visits"].shape[0] == 1 and t2["visits"][0] == 160  # terminal root
    t1 = eng.export_tree(1)
    pass_child = np.flatnonzero((t1["parent"] == 0) & (t1["action"] == n * n))
    assert len(pass_child) == 1 and t1["terminal"][pass_child[0]] == 1


class _RecordingGoEvaluator:
    def __init__(self, n, seed=0):
        g = torch.Generator().manual_seed(seed)
        C = n * n
        self.wp = (torch.randn(17 * C, C + 1, generator=g) * 0.05).cuda()
        self.wv = (torch.randn(17 * C, generator=g) * 0.05).cuda()
        self.table = {}
        self.A = C + 1

    def evaluate_batch(self, feats):
        x = feats.reshape(feats.shape[0], -1)
        pol = torch.softmax(x @ self.wp, dim=1)
        val = torch.tanh(x @ self.wv)
        fc, pc, vc = feats.cpu().numpy().astype(np.float32), pol.cpu().numpy(), val.cpu().numpy()
        for i in range(fc.shape[0]):
            self.table[hashlib.sha256(fc[i].tobytes()).digest()] = (pc[i].copy(), vc[i])
        return pol, val

    def replay(self, feats):
        n = feats.shape[0]
        p = np.zeros((n, self.A), np.float32)
        v = np.zeros(n, np.float32)
        for i in range(n):
            p[i], v[i] = self.table[hashlib.sha256(np.ascontiguousarray(feats[i], np.float32).tobytes()).digest()]
        return p, v


def test_go_float_evaluator_replay_and_features(oracle_lib):
    from omoknuni_quantum_b200.engine import WaveEngine
    n = 9
    hist, meta = _roots(31, 1, 40, n)
    ev = _RecordingGoEvaluator(n)
    eng = WaveEngine(1, board_size=n, capacity=80000, max_wave_size=64, game="go")
    eng.search(torch.from_numpy(hist).cuda(), 320, evaluator=ev, meta=torch.from_numpy(meta))
    o = oracle_lib.Oracle(80000, n).search_go(hist[0], int(meta[0, 0]), 320, 64, ko=int(meta[0, 1]),
                                             passes=int(meta[0, 2]), evaluator=ev.replay)
    _compare(eng, 0, o)


def test_go_features_of_root_match_host_history():
    """The root's 17 planes: own/opponent stones over the 8 history boards and the colour plane."""
    from omoknuni_quantum_b200.engine import WaveEngine
    n = 9
    hist, meta = _roots(2, 1, 25, n)
    eng = WaveEngine(1, board_size=n, capacity=20000, max_wave_size=16, game="go")
    eng.begin(torch.from_numpy(hist).cuda(), meta=torch.from_numpy(meta))
    f = eng.queue_features(0).cpu().numpy()[0]
    me = int(meta[0, 0])
    for k in range(8):
        assert np.array_equal(f[k], (hist[0, k] == me).astype(np.float32))
        assert np.array_equal(f[8 + k], (hist[0, k] == 3 - me).astype(np.float32))
    assert (f[16] == (1.0 if me == 1 else 0.0)).all()


def _go_spec(blocks=2, filters=256):
    from omoknuni_quantum_b200.resnet import ResNetSpec
    return ResNetSpec(board_size=19, input_channels=17, num_blocks=blocks, filters=filters,
                      num_actions=362, fc_policy_hidden=256, fc_value_hidden=256)


@pytest.mark.parametrize("filters", [256, 128])
def test_go_resnet_matches_fp32_reference(filters):
    """ResNet at config 3's shapes (17 planes of 19x19, 362 actions, value FC 361->256->1) on
    the padded 20x20 pixel grid, against the fp32 reference model: 2e-2 absolute."""
    from omoknuni_quantum_b200.go import random_position
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, init_state_dict, reference_forward_fp32
    spec = _go_spec(filters=filters)
    sd = init_state_dict(spec, seed=11)
    ev = ResNetEvaluator(sd, board_size=19, max_batch=512)
    feats = []
    for i in range(300):
        g = random_position(100 + i % 7, moves=10 + (i * 13) % 150, board_size=19)
        h, me = g.history_planes(), g.to_move
        f = np.zeros((17, 19, 19), np.float32)
        f[:8] = h == me
        f[8:16] = h == 3 - me
        f[16] = 1.0 if me == 1 else 0.0
        feats.append(f)
    x = torch.from_numpy(np.stack(feats)).cuda()
    p, v = ev.evaluate_batch(x)
    torch.cuda.synchronize()
    assert ev.error() == 0
    pr, vr = reference_forward_fp32({k: t.cuda() for k, t in sd.items()}, x)
    dp, dv = (p - pr).abs().max().item(), (v - vr).abs().max().item()
    assert dp < 2e-2 and dv < 2e-2, (dp, dv)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_go_resnet_queue_path_equals_protocol_path(dtype):
    """forward_queue packs the 17 planes on the device straight from the tree; the result equals
    evaluate_batch on the engine's fp32 feature tensor (identical trees)."""
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.resnet import ResNetEvaluator
    ev = ResNetEvaluator.random(_go_spec(), seed=2, max_batch=1024, dtype=dtype)

    class Protocol:
        def evaluate_batch(self, f):
            return ev.evaluate_batch(f)

    hist, meta = _roots(9, 3, 60, 19)
    h, m = torch.from_numpy(hist).cuda(), torch.from_numpy(meta)
    e1 = WaveEngine(3, board_size=19, capacity=120000, max_wave_size=64, game="go")
    e1.search(h, 192, evaluator=ev, meta=m)
    e2 = WaveEngine(3, board_size=19, capacity=120000, max_wave_size=64, game="go")
    e2.search(h, 192, evaluator=Protocol(), meta=m)
    for r in range(3):
        a, b = e1.export_tree(r), e2.export_tree(r)
        for k in a:
            assert np.array_equal(a[k], b[k]), k


def test_go_root_noise_replays_in_oracle_and_tree_full(oracle_lib):
    """Root Dirichlet noise over the Go root's children (pass included) replays bit-exact in the
    oracle; a too-small capacity raises TreeFullError."""
    from omoknuni_quantum_b200._lib import TreeFullError
    from omoknuni_quantum_b200.engine import WaveEngine
    n = 9
    hist, meta = _roots(44, 1, 30, n)
    eng = WaveEngine(1, board_size=n, capacity=60000, max_wave_size=32, game="go",
                     dirichlet_alpha=0.03, dirichlet_epsilon=0.25, noise_seed=9)
    eng.begin(torch.from_numpy(hist).cuda(), meta=torch.from_numpy(meta))
    eng.root_expand()
    o = oracle_lib.Oracle(60000, n)
    assert o.begin_go(hist[0], int(meta[0, 0]), o.config(96, 32), ko=int(meta[0, 1]),
                      passes=int(meta[0, 2])) == 0
    for _ in range(3):
        eng.wave(32)
        nz = eng.root_noise()[0].cpu().numpy()
        assert nz.shape == (n * n + 1,) and abs(nz.sum() - 1) < 1e-5
        assert o.wave(32, root_noise=nz, eps=0.25) == 0
    t, ot = eng.export_tree(0), o.export()
    for k in ("visits", "value_sums", "priors", "parent", "action"):
        assert np.array_equal(t[k], getattr(ot, k)), k
    small = WaveEngine(1, board_size=n, capacity=500, max_wave_size=64, game="go")
    with pytest.raises(TreeFullError):
        small.search(torch.from_numpy(hist).cuda(), 256, meta=torch.from_numpy(meta))


def test_go_selfplay_moves_match_oracle(oracle_lib):
    """Each move's policy in batched device Go self-play equals the oracle's search of that
    position (history planes, side to move, ko and passes carried between moves)."""
    from omoknuni_quantum_b200.selfplay import BatchedSelfPlay
    sp = BatchedSelfPlay(3, game="go", board_size=7, num_simulations=64, wave_size=16,
                         capacity=30000, seed=2)
    recs = sp.play(6)
    for r in recs:
        for i, ex in enumerate(r.examples):
            from omoknuni_quantum_b200.go import GoPosition
            g = GoPosition(7)
            for a in r.moves[:i]:
                g.play(a)
            assert np.array_equal(g.history_planes(), ex["state"])
            o = oracle_lib.Oracle(30000, 7).search_go(g.history_planes(), g.to_move, 64, 16,
                                                     ko=g.ko, passes=g.passes)
            assert np.array_equal(ex["policy"], o.policy)


def _superko_root(ply):
    """The reference double-ko game (tests/golden/go_superko.npz, game 0) replayed to `ply`."""
    import os
    from omoknuni_quantum_b200.go import GoPosition
    z = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "go_superko.npz"))
    g = GoPosition(int(z["g0_n"]))
    for a in z["g0_moves"][:ply]:
        g.play(int(a))
    return g, int(z["superko_ply"])


def test_go_superko_refusal_on_device_matches_oracle(oracle_lib):
    """At the double-ko position the reference refuses B's ko capture (1,2): the device root has
    no such child when the game's keys are passed, has it without them or with superko off, and
    every tree equals the oracle's."""
    from omoknuni_quantum_b200.engine import WaveEngine
    g, ply = _superko_root(20)
    assert ply == 20 and not g.is_legal(11)
    hist, meta, keys = g.history_planes(), g.meta(), g.root_keys()
    for superko, ks, child in ((True, keys, False), (True, None, True), (False, keys, True)):
        eng = WaveEngine(1, board_size=9, capacity=60000, max_wave_size=32, game="go", go_superko=superko)
        eng.search(torch.from_numpy(hist[None]).cuda(), 128, meta=torch.from_numpy(meta[None]),
                   keys=None if ks is None else [ks])
        t = eng.export_tree(0)
        assert bool(((t["parent"] == 0) & (t["action"] == 11)).any()) == child
        o = oracle_lib.Oracle(60000, 9).search_go(hist, g.to_move, 128, 32, ko=g.ko, passes=g.passes,
                                                 superko=superko, keys=() if ks is None else ks)
        _compare(eng, 0, o)


def test_go_superko_random_roots_with_game_keys(oracle_lib):
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.go import random_position
    ps = [random_position(600 + i, moves=50, board_size=9) for i in range(3)]
    eng = WaveEngine(3, board_size=9, capacity=80000, max_wave_size=64, game="go")
    eng.search(torch.from_numpy(np.stack([p.history_planes() for p in ps])).cuda(), 256,
               meta=torch.from_numpy(np.stack([p.meta() for p in ps])), keys=[p.root_keys() for p in ps])
    for r, p in enumerate(ps):
        o = oracle_lib.Oracle(80000, 9).search_go(p.history_planes(), p.to_move, 256, 64, ko=p.ko,
                                                 passes=p.passes, keys=p.root_keys())
        _compare(eng, r, o)


@pytest.mark.parametrize("rules", ["japanese", "korean"])
def test_go_repetition_terminal_on_device_matches_oracle(oracle_lib, rules):
    """Japanese / Korean rules: one move before the cycle's third repetition, that move's child is
    terminal on the device (root keys of every move, side to move included) and the trees equal
    the oracle's; a root three moves earlier must find it inside the tree the same way."""
    import os
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.go import GoPosition
    z = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "go_rulesets.npz"))
    gi = [i for i in range(int(z["games"])) if str(z[f"g{i}_rules"]) == rules][0]
    moves = z[f"g{gi}_moves"]
    last = len(moves) - 1                       # the ply where the reference reports terminal
    for ply in (last - 1, last - 3):
        g = GoPosition(9, rules=rules)
        for a in moves[:ply]:
            g.play(int(a))
        eng = WaveEngine(1, board_size=9, capacity=60000, max_wave_size=32, game="go", go_rules=rules)
        eng.search(torch.from_numpy(g.history_planes()[None]).cuda(), 256,
                   meta=torch.from_numpy(g.meta()[None]), keys=[g.root_keys()])
        o = oracle_lib.Oracle(60000, 9).search_go(g.history_planes(), g.to_move, 256, 32, ko=g.ko,
                                                 passes=g.passes, superko=False, cycle=True,
                                                 keys=g.root_keys())
        _compare(eng, 0, o)
        if ply == last - 1:
            t = eng.export_tree(0)
            child = np.flatnonzero((t["parent"] == 0) & (t["action"] == int(moves[ply])))
            assert len(child) == 1 and t["terminal"][child[0]] == 1
