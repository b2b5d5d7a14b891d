"""Self-play with the moves drawn and played on the device (omq_selfplay_move): the same games as
the host driver replaying the device's counter-based draws - moves, examples (position, visit
policy, root value, player, move number), game ends, winners and resignations - for the built-in
synthetic evaluator and the tensor-core ResNet, with and without subtree reuse."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _roots(G):
    from omoknuni_quantum_b200.roots import random_roots
    r = random_roots(77, G)
    r[1] = 0
    r[1, 7, 3:7] = 1                  # black to move with an open four
    r[1, 2, 2] = r[1, 3, 10] = r[1, 11, 4] = r[1, 12, 12] = 2
    return r


def _play(sampling, evaluator, reuse, resign):
    from omoknuni_quantum_b200.selfplay import BatchedSelfPlay
    kw = dict(num_simulations=96, wave_size=32, capacity=60000, seed=11, temperature_threshold=4,
              roots=_roots(6), subtree_reuse=reuse, evaluator=evaluator,
              resign_threshold=resign, resign_min_move=2)
    if sampling == "device":
        sp = BatchedSelfPlay(6, sampling="device", max_moves=16, **kw)
    else:
        sp = BatchedSelfPlay(6, sampling="host", rng="counter", **kw)
    recs = sp.play(7)
    sp.close()
    return recs


@pytest.mark.parametrize("evaluator,reuse,resign", [("synthetic", "none", -0.98), ("synthetic", "keep", 0.05),
                                                     ("resnet", "carry", -0.98)])
def test_device_selfplay_equals_host_replay(evaluator, reuse, resign):
    if evaluator == "resnet":
        from omoknuni_quantum_b200.resnet import ResNetEvaluator, ResNetSpec
        evaluator = ResNetEvaluator.random(ResNetSpec(num_blocks=2, filters=128), seed=2, max_batch=6 * 32)
    dev = _play("device", evaluator, reuse, resign)
    host = _play("host", evaluator, reuse, resign)
    assert sum(len(r.moves) for r in dev) > 6
    for a, b in zip(dev, host):
        assert a.moves == b.moves
        assert (a.finished, a.winner, a.resigned) == (b.finished, b.winner, b.resigned)
        assert len(a.examples) == len(b.examples) == len(a.moves)
        for x, y in zip(a.examples, b.examples):
            assert np.array_equal(x["state"], y["state"])
            assert np.array_equal(x["policy"], y["policy"])
            assert x["player"] == y["player"] and x["move_number"] == y["move_number"]
            assert np.float32(x["value_pred"]) == np.float32(y["value_pred"])
    if resign > 0:
        assert any(r.resigned for r in dev)


def _chess_roots():
    from omoknuni_quantum_b200.chess import ChessPosition, random_position
    r = [random_position(5 * 1_000_003 + i) for i in range(4)]
    r.append(ChessPosition("8/8/8/4k3/8/8/8/R3K3 w - - 99 80"))    # every move ends it: fifty moves
    r.append(ChessPosition("6k1/5ppp/8/8/8/8/5PPP/R5K1 w - - 0 30"))  # mate in one on the board
    return r


def _play_chess(sampling, reuse, resign):
    from omoknuni_quantum_b200.selfplay import BatchedSelfPlay
    kw = dict(num_simulations=64, wave_size=16, capacity=60000, seed=5, temperature_threshold=3,
              roots=_chess_roots(), subtree_reuse=reuse, evaluator="synthetic", game="chess",
              resign_threshold=resign, resign_min_move=2)
    if sampling == "device":
        sp = BatchedSelfPlay(6, sampling="device", max_moves=12, **kw)
    else:
        sp = BatchedSelfPlay(6, sampling="host", rng="counter", **kw)
    recs = sp.play(6)
    final = [p.root_records().tobytes() for p in sp.positions]
    sp.close()
    return recs, final


@pytest.mark.parametrize("reuse,resign", [("none", -0.98), ("keep", 0.05)])
def test_device_chess_selfplay_equals_host_replay(reuse, resign):
    """Chess games played by omq_selfplay_move_chess equal the host driver's (the reference
    engine's rules in chess.py): moves, examples (the 80-byte records), ends and the final root
    records with their repetition counts and earlier positions."""
    (dev, dfinal), (host, hfinal) = _play_chess("device", reuse, resign), _play_chess("host", reuse, resign)
    assert sum(len(r.moves) for r in dev) > 6
    assert dev[4].finished and dev[4].winner == 0 and len(dev[4].moves) == 1   # the fifty-move draw
    for a, b in zip(dev, host):
        assert a.moves == b.moves
        assert (a.finished, a.winner, a.resigned) == (b.finished, b.winner, b.resigned)
        assert len(a.examples) == len(b.examples) == len(a.moves)
        for x, y in zip(a.examples, b.examples):
            assert x["state"].tobytes() == y["state"].tobytes()
            assert np.array_equal(x["policy"], y["policy"])
            assert x["player"] == y["player"] and x["move_number"] == y["move_number"]
            assert np.float32(x["value_pred"]) == np.float32(y["value_pred"])
    assert dfinal == hfinal
    if resign > 0:
        assert any(r.resigned for r in dev)


def _go_roots(rules):
    from omoknuni_quantum_b200.go import GoPosition
    out = []
    for i in range(4):
        g = GoPosition(9, rules=rules)
        rng = np.random.default_rng(40 + i)
        for _ in range(24):
            cand = np.flatnonzero(g.legal_mask()[:-1])
            g.play(int(rng.choice(cand)))
        out.append(g)
    # white to move after a pass, and every point is a one-point eye of black's single group:
    # white can only pass, which ends the game (scored)
    g = GoPosition(9, rules=rules)
    g.board[:] = 1
    for y, x in ((1, 1), (1, 7), (7, 1), (7, 7), (4, 4)):
        g.board[y, x] = 0
    g.history = [g.board.copy()]
    g.to_move, g.passes = 2, 1
    out.append(g)
    out.append(GoPosition(9, rules=rules))                 # the empty board
    return out


def _play_go(sampling, rules, reuse, resign):
    from omoknuni_quantum_b200.selfplay import BatchedSelfPlay
    kw = dict(num_simulations=64, wave_size=16, capacity=60000, seed=9, temperature_threshold=3,
              roots=_go_roots(rules), board_size=9, subtree_reuse=reuse, evaluator="synthetic", game="go",
              resign_threshold=resign, resign_min_move=2)
    if sampling == "device":
        sp = BatchedSelfPlay(6, sampling="device", max_moves=12, **kw)
    else:
        sp = BatchedSelfPlay(6, sampling="host", rng="counter", **kw)
    recs = sp.play(7)
    final = [(p.history_planes().tobytes(), p.meta().tobytes(), list(p.keys), list(p.prisoners), p.repeated)
             for p in sp.positions]
    sp.close()
    return recs, final


@pytest.mark.parametrize("rules,reuse,resign", [("chinese", "none", -0.98), ("japanese", "keep", 0.05),
                                                ("korean", "carry", -0.98)])
def test_device_go_selfplay_equals_host_replay(rules, reuse, resign):
    """Go games played by omq_selfplay_move_go equal the host driver's (go.py, the reference
    engine's rules): moves, examples (the 8 history boards), ends, scores and the final
    positions (history, side to move, ko, passes, keys, prisoners)."""
    (dev, dfinal), (host, hfinal) = _play_go("device", rules, reuse, resign), _play_go("host", rules, reuse, resign)
    assert sum(len(r.moves) for r in dev) > 6
    # white's forced pass ends it: black's area 81 against komi 7.5; by territory 5 against 6.5
    assert dev[4].finished and dev[4].moves == [81] and dev[4].winner == (1 if rules == "chinese" else -1)
    for a, b in zip(dev, host):
        assert a.moves == b.moves
        assert (a.finished, a.winner, a.resigned) == (b.finished, b.winner, b.resigned)
        assert len(a.examples) == len(b.examples) == len(a.moves)
        for x, y in zip(a.examples, b.examples):
            assert np.array_equal(x["state"], y["state"])
            assert np.array_equal(x["policy"], y["policy"])
            assert x["player"] == y["player"] and x["move_number"] == y["move_number"]
            assert np.float32(x["value_pred"]) == np.float32(y["value_pred"])
    assert dfinal == hfinal
    if resign > 0:
        assert any(r.resigned for r in dev)
