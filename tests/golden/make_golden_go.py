"""Golden Go-rules fixture from the REFERENCE's C++ engine (alphazero_py.GoState, built from the
reference sources by `make -C oracle ref`): seeded random games with captures and kos, and for
every ply the board, the side to move, the legal-move mask and the move played.

Rules: GoState(board_size, 7.5, chinese_rules=True, enforce_superko=False) - captures, no
suicide, simple ko, pass always legal (src/games/go/go_state.cpp:227-420).
Writes tests/golden/go_rules.npz. Runs only in the build container.
"""
import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def board_of(state, n):
    """Board (0 empty, 1 black, 2 white; action = y * n + x) from the basic tensor
    representation: plane 0 holds the side to move's stones, plane 1 the opponent's.
    (GoState.to_string() crashes in this process layout, so it is not used.)"""
    t = np.array(state.get_basic_tensor_representation())
    cur = state.get_current_player()
    b = np.zeros((n, n), np.int8)
    b[t[0] > 0.5] = cur
    b[t[1] > 0.5] = 3 - cur
    return b


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("OMQ_REFERENCE"), required="OMQ_REFERENCE" not in os.environ)
    ap.parse_args()
    sys.path.insert(0, os.path.join(REPO, "oracle", "_ref"))
    import alphazero_py as az
    rec = {}
    games = [(9, 140, 1), (9, 140, 2), (9, 160, 3), (13, 220, 4), (19, 320, 5), (19, 320, 6)]
    for gi, (n, plies, seed) in enumerate(games):
        rng = np.random.default_rng(seed)
        s = az.GoState(n, 7.5, True, False)
        boards, players, legal, moves = [], [], [], []
        for _ in range(plies):
            if s.is_terminal():
                break
            b = board_of(s, n)
            # legality as make_move enforces it (GoState::isLegalMove, go_state.cpp:359-418);
            # getLegalMoves (:227-265) does not exclude the ko point when superko is off
            mask = np.zeros(n * n + 1, bool)
            mask[n * n] = True
            for m in range(n * n):
                mask[m] = s.is_legal_move(m)
            lm = [-1] + [m for m in range(n * n) if mask[m]]
            # play mostly next to existing stones to provoke captures and kos; pass rarely
            cand = [m for m in lm if m != -1]
            near = [m for m in cand if any(
                0 <= m // n + dy < n and 0 <= m % n + dx < n and b[m // n + dy, m % n + dx] != 0
                for dy, dx in ((1, 0), (-1, 0), (0, 1), (0, -1)))]
            if not cand or rng.random() < 0.02:
                m = -1
            elif near and rng.random() < 0.7:
                m = int(near[rng.integers(len(near))])
            else:
                m = int(cand[rng.integers(len(cand))])
            boards.append(b)
            players.append(s.get_current_player())
            legal.append(mask)
            moves.append(n * n if m == -1 else m)
            s.make_move(m)
        rec[f"g{gi}_n"] = n
        rec[f"g{gi}_boards"] = np.array(boards, np.int8)
        rec[f"g{gi}_players"] = np.array(players, np.int8)
        rec[f"g{gi}_legal"] = np.packbits(np.array(legal), axis=1)
        rec[f"g{gi}_moves"] = np.array(moves, np.int16)
        caps = int(sum((np.array(boards[i]) != 0).sum() + 1 - (np.array(boards[i + 1]) != 0).sum()
                       for i in range(len(boards) - 1) if moves[i] != n * n))
        print(f"game {gi}: {n}x{n}, {len(moves)} plies, captured stones {caps}")
    rec["games"] = len(games)
    path = os.path.join(HERE, "go_rules.npz")
    np.savez_compressed(path, **rec)
    print(path, os.path.getsize(path))


if __name__ == "__main__":
    main()
