"""Golden Go-rules fixture with positional superko ON (the reference's default GoState): games of
alphazero_py.GoState(n, 7.5, chinese_rules=True, enforce_superko=True) built from the reference
sources (`make -C oracle ref`). Game 0 sets up two kos and cycles through them (B takes ko 1,
W takes ko 2, B passes, W retakes ko 1, B retakes ko 2, W passes): B's capture of ko 1 would now
recreate an earlier (board, ko point), so GoState::isLegalMove (go_state.cpp:359-418) refuses it;
the game then continues with seeded random legal moves. Games 1-3 are seeded random games.
For every ply: board, side to move, legal mask (is_legal_move per point, pass always legal) and
the move played. Writes tests/golden/go_superko.npz. Runs only in the build container.
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle", "_ref"))
import alphazero_py as az  # noqa: E402

import numpy as np  # noqa: E402

sys.path.insert(0, HERE)
from make_golden_go import board_of  # noqa: E402


def record(s, n, moves_fn, plies):
    boards, players, legal, moves = [], [], [], []
    for t in range(plies):
        if s.is_terminal():
            break
        b = board_of(s, n)
        mask = np.zeros(n * n + 1, bool)
        mask[n * n] = True
        for m in range(n * n):
            mask[m] = s.is_legal_move(m)
        m = moves_fn(t, mask)
        boards.append(b)
        players.append(s.get_current_player())
        legal.append(mask)
        moves.append(n * n if m == -1 else m)
        s.make_move(m)
    return boards, players, legal, moves


def main():
    rec = {}
    n = 9
    B = [(0, 1), (1, 0), (2, 1), (5, 6), (6, 7), (7, 6), (6, 5)]
    W = [(0, 2), (1, 3), (2, 2), (1, 1), (5, 5), (6, 4), (7, 5)]
    script = []
    for b, w in zip(B, W):
        script += [b[0] * n + b[1], w[0] * n + w[1]]
    script += [11, 60, -1, 10, 59, -1]
    rng = np.random.default_rng(7)

    def scripted(t, mask):
        if t < len(script):
            return script[t]
        cand = np.flatnonzero(mask[:-1])
        return int(cand[rng.integers(len(cand))]) if len(cand) else -1

    games = [(n, scripted, 60)]
    for seed, size, plies in ((1, 9, 150), (2, 9, 150), (3, 13, 200)):
        r = np.random.default_rng(seed)

        def rnd(t, mask, r=r):
            cand = np.flatnonzero(mask[:-1])
            if len(cand) == 0 or r.random() < 0.02:
                return -1
            return int(cand[r.integers(len(cand))])
        games.append((size, rnd, plies))
    for gi, (size, fn, plies) in enumerate(games):
        s = az.GoState(size, 7.5, True, True)
        boards, players, legal, moves = record(s, size, fn, plies)
        rec[f"g{gi}_n"] = size
        rec[f"g{gi}_boards"] = np.array(boards, np.int8)
        rec[f"g{gi}_players"] = np.array(players, np.int8)
        rec[f"g{gi}_legal"] = np.packbits(np.array(legal), axis=1)
        rec[f"g{gi}_moves"] = np.array(moves, np.int16)
        print(f"game {gi}: {size}x{size}, {len(moves)} plies")
    rec["games"] = len(games)
    # the ply at which the superko refusal shows: after the setup and the 6-move cycle
    rec["superko_ply"] = len(script)
    path = os.path.join(HERE, "go_superko.npz")
    np.savez_compressed(path, **rec)
    print(path, os.path.getsize(path))


if __name__ == "__main__":
    main()
