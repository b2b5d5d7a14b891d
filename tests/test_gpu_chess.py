"""GPU parity of the device chess search (config 4's game) against the oracle's chess search.

Bit-exact on the same roots: tree shape, visit counts, value sums, priors, terminal flags and the
root policy, with the built-in synthetic evaluator and with a float evaluator replayed by feature
bytes (which proves the 119 planes identical). Roots cover random playouts, castling, en passant,
promotions, a repetition about to complete, the fifty-move edge, checkmate, stalemate and
insufficient material. The ResNet runs at config 4's shapes (119 planes padded to 128 channels,
8x8 on the 9x9 padded grid, 4672 actions)."""
import hashlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _special_roots():
    from omoknuni_quantum_b200.chess import ChessPosition
    out = []
    for fen in ["r3k2r/pppq1ppp/2n2n2/3pp3/3PP3/2N2N2/PPPQ1PPP/R3K2R w KQkq - 0 1",
                "rnbqkbnr/ppp1p1pp/8/3pPp2/8/8/PPPP1PPP/RNBQKBNR w KQkq f6 0 3",
                "8/PPP4k/8/8/8/8/4Kppp/8 w - - 0 1",
                "4k3/8/8/8/8/8/8/R3K2R w KQ - 98 90",
                "6k1/5ppp/8/8/8/8/5PPP/3R2K1 w - - 0 1",      # back-rank mate in one
                "7k/5Q2/6K1/8/8/8/8/8 b - - 0 1",             # stalemate (terminal root)
                "8/8/4k3/8/8/4K3/8/6N1 w - - 0 1"]:           # insufficient material
        out.append(ChessPosition(fen))
    p = ChessPosition()
    g1f3, g8f6, f3g1, f6g8 = (62 << 6) | 45, (6 << 6) | 21, (45 << 6) | 62, (21 << 6) | 6
    for m in [g1f3, g8f6, f3g1, f6g8, g1f3, g8f6, f3g1]:
        p.play(m)                                   # ...Ng8 now repeats the start placement a third time
    out.append(p)
    return out


def _run(positions, sims, wave, evaluator="synthetic", cap=120000):
    from omoknuni_quantum_b200.engine import WaveEngine
    rec = np.stack([p.root_records() for p in positions])
    npr = np.array([len(p.prior) for p in positions], np.int32)
    eng = WaveEngine(len(positions), board_size=8, capacity=cap, max_wave_size=wave, game="chess")
    eng.search(rec, sims, evaluator=evaluator, meta=npr)
    return eng


def _oracle(oracle_lib, p, sims, wave, cap=120000, evaluator=None):
    o = oracle_lib.Oracle(cap, 8)
    return o.search_chess(p.record(), sims, wave, prior=p.prior, evaluator=evaluator)


def _compare(eng, r, o):
    t = eng.export_tree(r)
    assert t["visits"].shape == o.visits.shape
    for k in ("parent", "action", "priors", "visits", "value_sums", "terminal"):
        assert np.array_equal(t[k], getattr(o, k)), k


def test_chess_random_roots_match_oracle(oracle_lib):
    from omoknuni_quantum_b200.chess import random_position
    ps = [random_position(40 + i) for i in range(4)]
    eng = _run(ps, 400, 64)
    visits = eng.root_visits().cpu().numpy()
    for r, p in enumerate(ps):
        o = _oracle(oracle_lib, p, 400, 64)
        assert o.result["status"] == 0
        _compare(eng, r, o)
        assert np.array_equal(eng.policy_from_visits(visits[r]), o.policy)


def test_chess_special_roots_match_oracle(oracle_lib):
    ps = _special_roots()
    eng = _run(ps, 256, 32)
    for r, p in enumerate(ps):
        _compare(eng, r, _oracle(oracle_lib, p, 256, 32))
    # stalemate and insufficient-material roots are terminal: no children
    for r in (5, 6):
        t = eng.export_tree(r)
        assert t["visits"].shape[0] == 1 and t["terminal"][0] == 1
    # the repetition root: some knight move back to the start position is found terminal
    t = eng.export_tree(7)
    assert t["terminal"].sum() >= 1


class _RecordingChessEvaluator:
    def __init__(self, seed=0):
        g = torch.Generator().manual_seed(seed)
        self.wp = (torch.randn(119 * 64, 4672, generator=g) * 0.02).cuda()
        self.wv = (torch.randn(119 * 64, generator=g) * 0.05).cuda()
        self.table = {}

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
        p = np.zeros((n, 4672), np.float32)
        v = np.zeros(n, np.float32)
        for i in range(n):
            p[i], v[i] = self.table[hashlib.sha256(np.ascontiguousarray(feats[i], np.float32).tobytes()).digest()]
        return p, v


def test_chess_float_evaluator_replay_and_features(oracle_lib):
    from omoknuni_quantum_b200.chess import random_position
    p = random_position(77)
    ev = _RecordingChessEvaluator()
    eng = _run([p], 192, 32, evaluator=ev, cap=30000)
    o = _oracle(oracle_lib, p, 192, 32, cap=30000, evaluator=ev.replay)
    _compare(eng, 0, o)


def test_chess_root_features_match_oracle(oracle_lib):
    from omoknuni_quantum_b200.chess import random_position
    from omoknuni_quantum_b200.engine import WaveEngine
    p = random_position(9)
    eng = WaveEngine(1, board_size=8, capacity=20000, max_wave_size=16, game="chess")
    eng.begin(p.root_records()[None], meta=np.array([len(p.prior)], np.int32))
    f = eng.queue_features(0).cpu().numpy()[0]
    want = oracle_lib.chess_features([p.record()] + p.prior[:7])
    assert np.array_equal(f, want)


def _chess_spec(filters=256, blocks=2):
    from omoknuni_quantum_b200.resnet import ResNetSpec
    return ResNetSpec(board_size=8, input_channels=119, num_blocks=blocks, filters=filters,
                      num_actions=4672, fc_policy_hidden=256, fc_value_hidden=256)


@pytest.mark.parametrize("filters", [256, 128])
def test_chess_resnet_matches_fp32_reference(oracle_lib, filters):
    from omoknuni_quantum_b200.chess import random_position
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, init_state_dict, reference_forward_fp32
    sd = init_state_dict(_chess_spec(filters), seed=5)
    ev = ResNetEvaluator(sd, board_size=8, max_batch=512)
    feats = []
    for i in range(200):
        p = random_position(300 + i)
        feats.append(oracle_lib.chess_features([p.record()] + p.prior[:7]))
    x = torch.from_numpy(np.stack(feats)).cuda()
    pol, val = ev.evaluate_batch(x)
    torch.cuda.synchronize()
    assert ev.error() == 0
    pr, vr = reference_forward_fp32({k: t.cuda() for k, t in sd.items()}, x)
    dp, dv = (pol - pr).abs().max().item(), (val - vr).abs().max().item()
    assert dp < 2e-2 and dv < 2e-2, (dp, dv)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_chess_resnet_queue_path_equals_protocol_path(dtype):
    from omoknuni_quantum_b200.chess import random_position
    from omoknuni_quantum_b200.resnet import ResNetEvaluator
    ev = ResNetEvaluator.random(_chess_spec(), seed=3, max_batch=1024, dtype=dtype)

    class Protocol:
        def evaluate_batch(self, f):
            return ev.evaluate_batch(f)

    ps = [random_position(500 + i) for i in range(3)]
    e1 = _run(ps, 192, 64, evaluator=ev, cap=40000)
    e2 = _run(ps, 192, 64, evaluator=Protocol(), cap=40000)
    for r in range(3):
        a, b = e1.export_tree(r), e2.export_tree(r)
        for k in a:
            assert np.array_equal(a[k], b[k]), k


def test_chess_root_noise_replays_in_oracle_and_tree_full(oracle_lib):
    from omoknuni_quantum_b200._lib import TreeFullError
    from omoknuni_quantum_b200.chess import random_position
    from omoknuni_quantum_b200.engine import WaveEngine
    p = random_position(12)
    rec = p.root_records()[None]
    npr = np.array([len(p.prior)], np.int32)
    eng = WaveEngine(1, board_size=8, capacity=40000, max_wave_size=32, game="chess",
                     dirichlet_alpha=0.3, dirichlet_epsilon=0.25, noise_seed=5)
    eng.begin(rec, meta=npr)
    eng.root_expand()
    o = oracle_lib.Oracle(40000, 8)
    assert o.begin_chess(p.record(), o.config(96, 32), prior=p.prior) == 0
    for _ in range(3):
        eng.wave(32)
        nz = eng.root_noise()[0].cpu().numpy()
        assert nz.shape == (4672,) and abs(nz.sum() - 1) < 1e-5
        assert o.wave(32, root_noise=nz, eps=0.25) == 0
    t, ot = eng.export_tree(0), o.export()
    for k in ("visits", "value_sums", "priors", "parent", "action"):
        assert np.array_equal(t[k], getattr(ot, k)), k
    small = WaveEngine(1, board_size=8, capacity=100, max_wave_size=64, game="chess")
    with pytest.raises(TreeFullError):
        small.search(rec, 256, meta=npr)


def test_chess_selfplay_moves_match_oracle(oracle_lib):
    from omoknuni_quantum_b200.chess import ChessPosition
    from omoknuni_quantum_b200.selfplay import BatchedSelfPlay
    sp = BatchedSelfPlay(3, game="chess", num_simulations=64, wave_size=16, capacity=30000, seed=3)
    recs = sp.play(5)
    for r in recs:
        p = ChessPosition()
        for i, ex in enumerate(r.examples):
            o = oracle_lib.Oracle(30000, 8).search_chess(p.record(), 64, 16, prior=p.prior)
            assert np.array_equal(ex["policy"], o.policy)
            p.play(p.action_to_move(r.moves[i]))


def _castles(p):
    return [m for m in p.legal_moves()
            if (p.sq[(m >> 6) & 63] & 7) == 6 and abs(((m >> 6) & 7) - (m & 7)) == 2]


def _chess960_roots(count=6):
    """Positions of the reference's Chess960 games (tests/golden/chess960.npz) at the first ply
    where the side to move can castle, plus two start positions; games replayed on the host."""
    import os
    from omoknuni_quantum_b200.chess import ChessPosition, chess960_fen
    z = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "chess960.npz"))
    out = [ChessPosition(chess960_fen(int(z["numbers"][0])), chess960=True),
           ChessPosition(chess960_fen(int(z["numbers"][1])), chess960=True)]
    go = z["game_off"]
    for g in range(len(go) - 1):
        p = ChessPosition(chess960_fen(int(z["numbers"][g])), chess960=True)
        for i in range(go[g], go[g + 1]):
            if _castles(p):
                out.append(p.copy())
                break
            if int(z["moves"][i]) < 0:
                break
            p.play(int(z["moves"][i]))
        if len(out) >= count:
            break
    return out


def test_chess960_roots_match_oracle(oracle_lib):
    """Chess960 castling (arbitrary king and rook files) on the device matches the oracle, which
    replays the reference engine's Chess960 games; the castling moves are root children."""
    ps = _chess960_roots()
    assert len(ps) >= 5
    eng = _run(ps, 384, 48)
    for r, p in enumerate(ps):
        _compare(eng, r, _oracle(oracle_lib, p, 384, 48))
        t = eng.export_tree(r)
        kids = set(int(a) for a, par in zip(t["action"], t["parent"]) if par == 0)
        assert all(p.move_to_action(m) in kids for m in _castles(p))
        assert len(kids) == len(p.legal_moves())
