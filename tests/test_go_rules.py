"""The oracle's Go rules replay the reference engine's games (tests/golden/go_rules.npz, made by
tests/golden/make_golden_go.py from GoState with superko off): every ply's legal mask and every
resulting board, with captures and kos, bit for bit."""
import os

import numpy as np

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "go_rules.npz")


def _games():
    g = np.load(GOLD)
    for i in range(int(g["games"])):
        n = int(g[f"g{i}_n"])
        yield (n, g[f"g{i}_boards"], g[f"g{i}_players"],
               np.unpackbits(g[f"g{i}_legal"], axis=1)[:, : n * n + 1].astype(bool), g[f"g{i}_moves"])


def test_go_oracle_replays_reference_games(oracle_lib):
    kos = captures = 0
    for n, boards, players, legal, moves in _games():
        ko = -1
        for t in range(len(moves)):
            assert np.array_equal(oracle_lib.go_legal(boards[t], players[t], ko), legal[t]), (n, t)
            res = oracle_lib.go_play(boards[t], players[t], int(moves[t]), ko)
            assert res is not None
            nb, ko = res
            kos += ko >= 0
            if t + 1 < len(moves):
                assert np.array_equal(nb, boards[t + 1]), (n, t)
                assert players[t + 1] == 3 - players[t]
                captures += int((boards[t] != 0).sum() + (moves[t] != n * n) - (nb != 0).sum())
    assert captures > 300 and kos > 0


def test_go_illegal_moves_and_ko(oracle_lib):
    b = np.zeros((5, 5), np.int8)
    b[0, 1] = b[1, 0] = 1                                # black stones around the corner (0,0)
    assert oracle_lib.go_play(b, 2, 0) is None          # white in the corner: suicide
    assert oracle_lib.go_play(b, 1, 0) is not None      # black filling its own eye is legal
    assert oracle_lib.go_play(b, 2, 1) is None          # occupied
    nb, ko = oracle_lib.go_play(b, 2, 25)               # pass: board unchanged
    assert np.array_equal(nb, b) and ko == -1
    # ko shape: white stone at (1,1) in atari, black captures it from (1,2)
    k = np.zeros((5, 5), np.int8)
    k[1, 0] = k[0, 1] = k[2, 1] = 1
    k[0, 2] = k[2, 2] = k[1, 3] = 2
    k[1, 1] = 2
    nb, ko = oracle_lib.go_play(k, 1, 1 * 5 + 2)
    assert nb[1, 1] == 0 and nb[1, 2] == 1 and ko == 1 * 5 + 1
    assert oracle_lib.go_play(nb, 2, ko, ko) is None    # immediate retake forbidden
    assert not oracle_lib.go_legal(nb, 2, ko)[ko]
    assert oracle_lib.go_legal(nb, 2, -1)[ko]           # legal once the ko point is cleared
    assert oracle_lib.go_play(nb, 2, 25, ko)[1] == -1   # pass clears the ko


def test_host_go_position_replays_reference_games():
    """The package's host-side Go position (root construction, moves between searches) follows
    the same reference games."""
    from omoknuni_quantum_b200.go import GoPosition
    for n, boards, players, legal, moves in _games():
        g = GoPosition(n)
        for t in range(len(moves)):
            assert np.array_equal(g.board, boards[t]) and g.to_move == players[t]
            if t % 7 == 0:  # the full mask is slow in pure Python; sample plies
                assert np.array_equal(g.legal_mask(), legal[t]), (n, t)
            g.play(int(moves[t]))


def test_go_roots_are_seeded_and_legal(oracle_lib):
    from omoknuni_quantum_b200.go import random_roots
    h, m = random_roots(3, 2, moves=60, board_size=9)
    h2, m2 = random_roots(3, 2, moves=60, board_size=9)
    assert np.array_equal(h, h2) and np.array_equal(m, m2)
    assert h.shape == (2, 8, 9, 9) and m.shape == (2, 3)
    assert (m[:, 0] == 1).all()                      # 60 moves: black to move
    for i in range(2):
        # consecutive history boards differ by one legal move each
        for k in range(7, 0, -1):
            prev, nxt = h[i, k], h[i, k - 1]
            mover = 1 if (60 - k) % 2 == 0 else 2
            a = np.flatnonzero((prev.reshape(-1) == 0) & (nxt.reshape(-1) == mover))
            assert len(a) == 1
            res = oracle_lib.go_play(prev, mover, int(a[0]))
            assert res is not None and np.array_equal(res[0], nxt)


def test_oracle_go_search_invariants(oracle_lib):
    """Oracle Go search: children of every expanded node are exactly the rules' legal moves (pass
    included, ascending), priors sum to 1, visits add up, double-pass children are terminal."""
    from omoknuni_quantum_b200.go import random_position
    g = random_position(5, moves=30, board_size=9)
    o = oracle_lib.Oracle(60000, 9)
    t = o.search_go(g.history_planes(), g.to_move, 256, 64, ko=g.ko, passes=g.passes)
    assert t.result["status"] == 0
    assert t.visits[0] == 256 and t.policy.shape == (82,)
    kids = t.parent == 0
    assert np.array_equal(np.sort(t.action[kids]), np.flatnonzero(g.legal_mask()))
    assert abs(t.priors[kids].sum() - 1.0) < 1e-5
    assert t.visits[0] == t.visits[kids].sum() + 0  # every simulation passes through a child
    # a pass child of a pass child is terminal
    pass_nodes = np.flatnonzero(t.action == 81)
    for c in pass_nodes:
        p = t.parent[c]
        assert bool(t.terminal[c]) == (p > 0 and t.action[p] == 81)


SUPERKO = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "go_superko.npz")


def _superko_games():
    g = np.load(SUPERKO)
    for i in range(int(g["games"])):
        n = int(g[f"g{i}_n"])
        yield (n, g[f"g{i}_boards"], g[f"g{i}_players"],
               np.unpackbits(g[f"g{i}_legal"], axis=1)[:, : n * n + 1].astype(bool), g[f"g{i}_moves"])


def test_go_superko_oracle_replays_reference_games(oracle_lib):
    """GoState with enforce_superko (the reference default): the oracle's legality with the game's
    position keys equals is_legal_move at every ply, including the double-ko refusal."""
    refused = 0
    for n, boards, players, legal, moves in _superko_games():
        ko, keys = -1, []
        for t in range(len(moves)):
            m = oracle_lib.go_legal_superko(boards[t], players[t], ko, keys)
            assert np.array_equal(m, legal[t]), (n, t)
            refused += int((oracle_lib.go_legal(boards[t], players[t], ko) & ~m).sum())
            nb, ko = oracle_lib.go_play(boards[t], players[t], int(moves[t]), ko)
            if moves[t] != n * n:
                keys.append(oracle_lib.go_key(nb, ko))
    assert refused >= 1


def test_go_superko_host_position_replays_reference_games(oracle_lib):
    from omoknuni_quantum_b200.go import GoPosition, position_key
    for n, boards, players, legal, moves in _superko_games():
        g = GoPosition(n)
        for t in range(len(moves)):
            assert np.array_equal(g.board, boards[t])
            if t % 5 == 0 or (n == 9 and 18 <= t <= 22):
                assert np.array_equal(g.legal_mask(), legal[t]), (n, t)
            g.play(int(moves[t]))
    # the host keys are the oracle's keys
    b = boards[-1]
    assert position_key(b, 5) == oracle_lib.go_key(b, 5) and position_key(b) == oracle_lib.go_key(b, -1)


RULESETS = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "go_rulesets.npz")


def test_go_rulesets_host_position_replays_reference_games():
    """Chinese / Japanese / Korean GoState games: legality (superko only under Chinese rules),
    the Japanese / Korean third-repetition terminal (no result / draw) and the scored results of
    games ended by two passes, ply by ply."""
    from omoknuni_quantum_b200.go import GoPosition
    z = np.load(RULESETS)
    seen = set()
    for i in range(int(z["games"])):
        rules, n = str(z[f"g{i}_rules"]), int(z[f"g{i}_n"])
        legal = np.unpackbits(z[f"g{i}_legal"], axis=1)[:, : n * n + 1].astype(bool)
        g = GoPosition(n, rules=rules)
        for t, mv in enumerate(z[f"g{i}_moves"]):
            assert np.array_equal(g.board, z[f"g{i}_boards"][t]) and g.to_move == z[f"g{i}_players"][t]
            assert g.is_terminal() == bool(z[f"g{i}_terminal"][t]), (rules, i, t)
            assert g.result() == int(z[f"g{i}_result"][t]), (rules, i, t)
            if t % 4 == 0 or t >= 18:
                assert np.array_equal(g.legal_mask(), legal[t]), (rules, i, t)
            if mv == -2:
                seen.add((rules, g.result()))
                break
            g.play(int(mv))
    assert ("japanese", 4) in seen and ("korean", 3) in seen
