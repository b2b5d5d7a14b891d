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
