"""Golden Chess960 fixture from the REFERENCE's C++ engine (alphazero_py.ChessState(True, "", k),
built from the reference sources by `make -C oracle ref`):
  * the start FEN of every position number 0..959 (Chess960::setupPosition; rook files in the
    castling field, Shredder style);
  * seeded random games (capture-biased) from start positions whose king stands on files c-f:
    per ply the FEN, the sorted legal moves (reference encoding), the terminal flag, the result
    and the move. With the king on the b- or g-file the reference's castling target (king file
    +-2, chess_rules.cpp:619-680) leaves the board, which no action encoding can express; those
    start positions are not played here.
Writes tests/golden/chess960.npz. Runs only in the build container.
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle", "_ref"))
import alphazero_py as az  # noqa: E402

import numpy as np  # noqa: E402

sys.path.insert(0, HERE)
from make_golden_chess import fen_of, _occupied  # noqa: E402


def result_code(r):
    return {"ONGOING": 0, "WIN_PLAYER1": 1, "WIN_PLAYER2": 2, "DRAW": 3}.get(r.name, 4)


def main():
    starts = [fen_of(az.ChessState(True, "", k)) for k in range(960)]
    king_file = [s.split()[0].split("/")[7].replace("1", "x").replace("2", "xx").replace("3", "xxx")
                 .replace("4", "xxxx").replace("5", "xxxxx").replace("6", "xxxxxx")
                 .replace("7", "xxxxxxx").replace("8", "xxxxxxxx").index("K") for s in starts]
    rng = np.random.default_rng(960)
    playable = [k for k in range(960) if 2 <= king_file[k] <= 5]
    picks = [int(k) for k in rng.choice(playable, size=14, replace=False)] + [518]
    fens, legal_flat, legal_off, term, res, moves, game_off, numbers = [], [], [0], [], [], [], [0], []
    for gi, k in enumerate(picks):
        s = az.ChessState(True, "", k)
        bias = 0.5 if gi % 2 else 0.2
        for t in range(120):
            f = fen_of(s)
            legal = sorted(int(a) for a in s.get_legal_moves())
            tm = bool(s.is_terminal())
            r = result_code(s.get_game_result())
            if tm or not legal:
                mv = -1
            else:
                mv = int(legal[rng.integers(len(legal))])
                occ = _occupied(f.split()[0])
                caps = [a for a in legal if occ[a & 63]]
                castles = [a for a in legal if abs((a & 63) % 8 - ((a >> 6) & 63) % 8) == 2
                           and f.split()[0].split("/")[7 if f.split()[1] == "w" else 0].find("K" if f.split()[1] == "w" else "k") >= 0]
                if castles and rng.random() < 0.5:
                    mv = int(castles[rng.integers(len(castles))])
                elif caps and rng.random() < bias:
                    mv = int(caps[rng.integers(len(caps))])
            fens.append(f)
            legal_flat.extend(legal)
            legal_off.append(len(legal_flat))
            term.append(tm)
            res.append(r)
            moves.append(mv)
            if mv < 0:
                break
            s.make_move(mv)
        game_off.append(len(fens))
        numbers.append(k)
    path = os.path.join(HERE, "chess960.npz")
    np.savez_compressed(path, starts=np.array(starts), fens=np.array(fens),
                        legal=np.array(legal_flat, np.int32), legal_off=np.array(legal_off, np.int64),
                        terminal=np.array(term), result=np.array(res, np.int8),
                        moves=np.array(moves, np.int32), game_off=np.array(game_off, np.int64),
                        numbers=np.array(numbers, np.int32))
    ncastle = sum(1 for f, m in zip(fens, moves) if m >= 0 and abs((m & 63) % 8 - ((m >> 6) & 63) % 8) == 2
                  and ((m >> 6) & 63) in (56, 57, 58, 59, 60, 61, 62, 63, 0, 1, 2, 3, 4, 5, 6, 7))
    print(f"{len(picks)} games, {len(fens)} plies, {sum(term)} terminal, ~{ncastle} king two-file moves; "
          f"{path} {os.path.getsize(path)} B")


if __name__ == "__main__":
    main()
