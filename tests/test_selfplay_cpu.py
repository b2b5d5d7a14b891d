"""Self-play bookkeeping on CPU with a fake searcher: temperature sampling then arg-max,
legal moves, five detection, outcome values from each player's perspective, reproducibility."""
import numpy as np
import pytest

from omoknuni_quantum_b200.selfplay import BatchedSelfPlay, board_after, game_result


def _fake_search(boards):
    """Visits favour the lowest empty cell strongly, then the next ones (deterministic)."""
    out = np.zeros((boards.shape[0], 225), np.int64)
    for i, b in enumerate(boards):
        empty = np.nonzero(b.reshape(-1) == 0)[0]
        out[i, empty[:3]] = [50, 30, 20]
    return out


def test_selfplay_moves_values_and_determinism():
    sp = BatchedSelfPlay(3, search=_fake_search, temperature_threshold=2, seed=7)
    recs = sp.play(12)
    for r in recs:
        b = np.zeros((15, 15), np.int8)
        for m in r.moves:
            assert b.reshape(-1)[m] == 0
            b = board_after(b, m)
        assert len(r.examples) == len(r.moves)
        # after the temperature moves the arg-max (the lowest empty cell) is played
        assert r.moves[2] == min(np.nonzero(r.examples[2]["state"].reshape(-1) == 0)[0])
        assert all(abs(e["policy"].sum() - 1) < 1e-12 for e in r.examples)
    sp2 = BatchedSelfPlay(3, search=_fake_search, temperature_threshold=2, seed=7)
    assert [r.moves for r in sp2.play(12)] == [r.moves for r in recs]
    # arg-max play where black fills row 0 and white row 1: black's five ends the game at move 9
    def rows(boards):
        out = np.zeros((boards.shape[0], 225), np.int64)
        for i, b in enumerate(boards):
            row = 0 if int((b != 0).sum()) % 2 == 0 else 1
            out[i, row * 15 + int((b[row] != 0).sum())] = 1
        return out
    sp3 = BatchedSelfPlay(1, search=rows, temperature_threshold=0)
    r = sp3.play(20)[0]
    assert r.finished and r.winner == 1 and len(r.moves) == 9
    ex = r.training_examples()
    assert all(e.value == (r.winner if i % 2 == 0 else -r.winner) for i, e in enumerate(ex))


def test_game_result():
    b = np.zeros((15, 15), np.int8)
    assert game_result(b) is None
    b[3, 2:7] = 1
    b[9, 0:4] = 2
    assert game_result(b) == 1
    full = (1 + (np.add.outer(np.arange(15), 2 * np.arange(15)) % 4 >= 2)).astype(np.int8)
    assert game_result(full) == 0


def _uniform_legal_search(sp, game):
    def search(inputs):
        live = [p for p, r in zip(sp.positions, sp.records) if not r.finished]
        out = []
        for p in live:
            if game == "go":
                v = p.legal_mask().astype(np.int64)
            else:
                v = np.zeros(4672, np.int64)
                for m in p.legal_moves():
                    v[p.move_to_action(m)] = 1
            out.append(v)
        return np.stack(out)
    return search


def test_go_selfplay_plays_legal_games_and_scores_them():
    from omoknuni_quantum_b200.selfplay import BatchedSelfPlay
    sp = BatchedSelfPlay(3, game="go", board_size=7, seed=4)
    sp._search = _uniform_legal_search(sp, "go")
    recs = sp.play(120)
    assert len(recs) == 3
    for r in recs:
        assert len(r.moves) == len(r.examples) > 0
        assert all(ex["state"].shape == (8, 7, 7) and ex["policy"].shape == (50,) for ex in r.examples)
        assert [ex["player"] for ex in r.examples[:4]] == [1, 2, 1, 2]
        if r.finished:
            assert r.moves[-1] == 49 and r.moves[-2] == 49      # two passes end the game
            assert r.winner in (1, -1, 0)
    ex = sp.examples()
    assert len(ex) == sum(len(r.examples) for r in recs)


def test_go_area_score():
    from omoknuni_quantum_b200.go import GoPosition
    g = GoPosition(5, komi=0.5)
    g.board[:, 1] = 1                     # black wall: column 0 is black territory
    g.board[:, 3] = 2                     # white wall: column 4 is white territory, column 2 neutral
    assert g.score() == (10.0, 10.5)
    g.play(g.pass_action)
    g.play(g.pass_action)
    assert g.result() == 2


def test_chess_selfplay_plays_legal_games():
    from omoknuni_quantum_b200.selfplay import BatchedSelfPlay
    sp = BatchedSelfPlay(2, game="chess", seed=1, temperature_threshold=100)
    sp._search = _uniform_legal_search(sp, "chess")
    recs = sp.play(40)
    for r in recs:
        assert len(r.moves) == len(r.examples) > 0
        assert r.examples[0]["policy"].shape == (4672,) and r.examples[0]["player"] == 1
    # replaying the recorded actions from the start reproduces the final positions
    from omoknuni_quantum_b200.chess import ChessPosition
    for g, r in enumerate(recs):
        p = ChessPosition()
        for a in r.moves:
            p.play(p.action_to_move(a))
        assert p.fen() == sp.positions[g].fen()


def test_resignation_q_values_and_metrics():
    """SelfPlayGame's resignation (self_play_manager.py:350-393): after move resign_min_move + 1
    a root value below the threshold makes the player who just moved resign and lose; training
    values mix the root values with use_mcts_q_values; metrics as the reference's play_game."""
    def losing(boards):
        # black's root values are fine, white's are lost (< -0.98) from its own perspective
        vals = np.array([0.5 if int((b != 0).sum()) % 2 == 0 else -0.99 for b in boards])
        return _fake_search(boards), vals
    sp = BatchedSelfPlay(2, search=losing, temperature_threshold=0, seed=1, resign_min_move=4)
    recs = sp.play(20)
    for r in recs:
        assert r.finished and r.resigned
        # white moves at move numbers 1, 3, 5 ...: the first white move with move_count > 4
        assert len(r.moves) == 6 and r.winner == 1
        ex = r.training_examples()
        assert [e.value for e in ex] == [1.0, -1.0] * 3
        mixed = r.training_examples(use_mcts_q_values=True, q_value_weight=0.8)
        assert abs(mixed[0].value - (0.8 * 0.5 + 0.2 * 1.0)) < 1e-12
        assert abs(mixed[1].value - (0.8 * -0.99 + 0.2 * -1.0)) < 1e-12
        m = r.metrics()
        assert m["resigned"] and m["game_length"] == 6 and m["winner"] == 1
        assert m["value_accuracies"] == [1.0] * 6 and len(m["policy_entropies"]) == 6
    off = BatchedSelfPlay(2, search=losing, temperature_threshold=0, seed=1, enable_resign=False)
    assert not any(r.resigned for r in off.play(8))


def test_go_selfplay_engine_follows_the_rule_set(monkeypatch):
    """Japanese / Korean roots are searched by an engine built with that rule set (the device's
    repetition rule instead of superko), one engine per rule set; mixed batches are refused."""
    import torch
    from omoknuni_quantum_b200 import engine as engine_mod
    from omoknuni_quantum_b200.go import GoPosition
    built = []

    class FakeEngine:
        def __init__(self, R, **kw):
            built.append(kw.get("go_rules", "chinese"))
            self.R, self.n = R, kw["board_size"]

        def search(self, roots, sims, evaluator, **kw):
            self.masks = [np.ones(self.n * self.n + 1, bool) for _ in range(self.R)]
            self.meta = kw["meta"]

        def root_visits(self):
            v = np.zeros((self.R, self.n * self.n + 1), np.int64)
            v[:, 0] = 1                       # every game plays its first cell, then passes
            return torch.from_numpy(v)

        def root_nw(self):
            return torch.zeros(self.R, 2)

        def reroot(self, actions, keep=False):
            pass

    monkeypatch.setattr(engine_mod, "WaveEngine", FakeEngine)
    roots = [GoPosition(9, rules="japanese") for _ in range(2)]
    sp = BatchedSelfPlay(2, num_simulations=8, game="go", board_size=9, roots=roots,
                         enable_resign=False)
    sp.step()
    assert built == ["japanese"]
    mixed = [GoPosition(9, rules="japanese"), GoPosition(9)]
    sp2 = BatchedSelfPlay(2, num_simulations=8, game="go", board_size=9, roots=mixed)
    with pytest.raises(ValueError):
        sp2.step()


def test_counter_draws_are_visit_proportional_and_replayed_by_the_host_driver():
    """counter_choice (the device's draw, omq_selfplay_move) samples in proportion to the visit
    counts, uniformly when nothing was visited, and the host driver with rng="counter" plays
    exactly those draws."""
    from omoknuni_quantum_b200.selfplay import counter_choice, counter_draw
    visits = np.zeros(225, np.int64)
    visits[[3, 40, 200]] = [10, 30, 60]
    picks = np.bincount([counter_choice(visits, counter_draw(5, g, m)) for g in range(40) for m in range(250)],
                        minlength=225)
    assert picks.sum() == 10000 and set(np.nonzero(picks)[0]) == {3, 40, 200}
    assert np.allclose(picks[[3, 40, 200]] / 10000, [0.1, 0.3, 0.6], atol=0.02)
    assert 0 <= counter_choice(np.zeros(225, np.int64), counter_draw(1, 2, 3)) < 225
    assert counter_draw(1, 2, 3) == counter_draw(1, 2, 3) != counter_draw(1, 2, 4)
    sp = BatchedSelfPlay(3, search=_fake_search, temperature_threshold=3, seed=9, rng="counter")
    recs = sp.play(5)
    for g, r in enumerate(recs):
        for m in range(3):
            v = _fake_search(r.examples[m]["state"][None])[0]
            assert r.moves[m] == counter_choice(v, counter_draw(9, g, m))


def test_device_roots_round_trip_for_every_game():
    """The host side of device self-play: positions -> the engine's device root layout (boards,
    chess root records + earlier-position counts, Go history planes + side / ko / passes + game
    keys) -> positions again, unchanged; and the recorded-state decoders."""
    from omoknuni_quantum_b200.chess import ChessPosition, random_position as chess_random
    from omoknuni_quantum_b200.go import GoPosition
    from omoknuni_quantum_b200.selfplay import _ChessGame, _GoGame, _GomokuGame
    from omoknuni_quantum_b200.roots import random_roots

    gm = _GomokuGame(15)
    boards = list(random_roots(3, 4))
    d = gm.device_roots(boards)
    assert d["boards"].shape == (4, 225) and d["boards"].dtype == np.int8
    for g in range(4):
        assert np.array_equal(gm.device_position(d, g, boards[g], None), boards[g])
        assert np.array_equal(gm.device_state(d["boards"][g].view(np.uint8)), boards[g])

    cg = _ChessGame(8)
    pos = [chess_random(11 + i) for i in range(3)] + [ChessPosition()]
    d = cg.device_roots(pos)
    assert d["records"].shape == (4, 101 * 80) and list(d["nprior"]) == [min(len(p.prior), 100) for p in pos]
    for g, p in enumerate(pos):
        q = cg.device_position(d, g, p, None)
        assert q.root_records().tobytes() == p.root_records().tobytes()
        assert q.fen() == p.fen() and q.result() == p.result() and q.reps == p.reps
        assert cg.device_state(d["records"][g][:80]).tobytes() == p.record().tobytes()

    go = _GoGame(9)
    rng = np.random.default_rng(5)
    gpos = []
    for rules in ("chinese", "japanese", "korean"):
        p = GoPosition(9, rules=rules)
        for _ in range(15):
            p.play(int(rng.choice(np.flatnonzero(p.legal_mask()))))
        gpos.append(p)
    gpos.append(GoPosition(9))
    d = go.device_roots(gpos)
    assert d["keys"].dtype == np.int64 and list(d["nkeys"]) == [len(p.keys) for p in gpos]
    for g, p in enumerate(gpos):
        row = [0, 0, 0, 0, 0] + go.device_game(p)
        q = go.device_position(d, g, p, row)
        assert np.array_equal(q.history_planes(), p.history_planes())
        assert np.array_equal(q.meta(), p.meta()) and q.keys == p.keys
        assert q.prisoners == p.prisoners and q.repeated == p.repeated and q.rules == p.rules
        assert q.result() == p.result()
        assert np.array_equal(go.device_state(d["history"][g].reshape(-1)), p.history_planes())


def test_go_no_result_counts_as_a_draw():
    """A Japanese third repetition is the reference's "no result" (GameResult 4): no winner."""
    from omoknuni_quantum_b200.go import GoPosition
    from omoknuni_quantum_b200.selfplay import _GoGame
    p = GoPosition(9, rules="japanese")
    p.repeated = True
    assert p.result() == 4 and _GoGame(9).outcome(p) == 0
