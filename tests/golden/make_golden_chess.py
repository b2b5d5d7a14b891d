"""Golden chess-rules fixture from the REFERENCE's C++ engine (alphazero_py.ChessState, built from
the reference sources by `make -C oracle ref`): for every ply of seeded games, the FEN (board,
side to move, castling rights, en-passant square, clocks), the sorted legal actions in the
reference's action encoding ((promotion << 12) | (from << 6) | to, chess_state.cpp:1474-1507),
the terminal flag, the game result and the move played.

Games: uniformly random games from the start position; capture-biased random games (they reach
sparse endgames); random games from positions rich in castling, promotion and en passant; a
forced threefold repetition; positions at the edge of the fifty-move rule; and the
insufficient-material cases of ChessRules::hasInsufficientMaterial (chess_rules.cpp:236-394).
Writes tests/golden/chess_rules.npz. Runs only in the build container.
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
# the reference module is imported before numpy: in the other order its to_string() crashes
sys.path.insert(0, os.path.join(REPO, "oracle", "_ref"))
import alphazero_py as az  # noqa: E402

import numpy as np  # noqa: E402

START = "rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1"
RICH = [
    "r3k2r/pppq1ppp/2n2n2/3pp3/3PP3/2N2N2/PPPQ1PPP/R3K2R w KQkq - 0 1",      # castling both ways
    "r3k2r/p1ppqpb1/bn2pnp1/3PN3/1p2P3/2N2Q1p/PPPBBPPP/R3K2R w KQkq - 0 1",   # tactical middlegame
    "8/PPP4k/8/8/8/8/4Kppp/8 w - - 0 1",                                     # promotions
    "rnbqkbnr/ppp1p1pp/8/3pPp2/8/8/PPPP1PPP/RNBQKBNR w KQkq f6 0 3",         # en passant available
    "8/2p5/3p4/KP5r/1R3p1k/8/4P1P1/8 w - - 0 1",                             # ep + pins
    "r3k2r/8/8/8/8/8/8/R3K2R w KQkq - 0 1",                                  # bare castling
    "4k3/8/8/8/8/8/8/R3K2R w KQ - 97 90",                                    # fifty-move edge
    "4k3/8/8/3q4/8/8/8/R3K2R w KQ - 0 1",                                    # castle through attack
]
INSUFFICIENT = [
    "8/8/4k3/8/8/4K3/8/8 w - - 0 1",          # K v K
    "8/8/4k3/8/8/4K3/8/6N1 w - - 0 1",        # KN v K
    "8/8/4k3/8/8/4K3/8/5B2 b - - 0 1",        # KB v K
    "8/8/2b1k3/8/8/4K3/8/5B2 w - - 0 1",      # KB v KB, bishops on opposite colours: not a draw
    "8/8/3bk3/8/8/4K3/8/5B2 w - - 0 1",       # KB v KB, same colour
    "8/8/4k3/8/8/4K3/8/5NN1 w - - 0 1",       # KNN v K
    "8/8/3nk3/8/8/4K3/8/6N1 w - - 0 1",       # KN v KN
    "8/8/3nk3/8/8/4K3/8/5B2 w - - 0 1",       # KN v KB
    "8/8/4k3/8/8/4K3/8/4BN2 w - - 0 1",       # KBN v K: not a draw
    "8/8/4k3/8/8/4K3/P7/8 w - - 0 1",         # KP v K: not a draw
]


def fen_of(state):
    for line in state.to_string().splitlines():
        if line.startswith("FEN: "):
            return line[5:].strip()
    raise RuntimeError("no FEN in to_string()")


def play(az, fen, plies, rng, capture_bias=0.0, forced=None):
    s = az.ChessState(False, fen) if fen != START else az.ChessState()
    rec = []
    for t in range(plies):
        f = fen_of(s)
        legal = sorted(int(a) for a in s.get_legal_moves())
        term = bool(s.is_terminal())
        res = int(s.get_game_result().value) if hasattr(s.get_game_result(), "value") else int(s.get_game_result())
        if term or not legal:
            rec.append((f, legal, term, res, -1))
            break
        if forced is not None and t < len(forced):
            mv = forced[t]
        else:
            mv = int(legal[rng.integers(len(legal))])
            if capture_bias > 0 and rng.random() < capture_bias:
                board = f.split()[0]
                occ = _occupied(board)
                caps = [a for a in legal if occ[a & 63]]
                if caps:
                    mv = int(caps[rng.integers(len(caps))])
        rec.append((f, legal, term, res, mv))
        s.make_move(mv)
    else:
        f = fen_of(s)
        rec.append((f, sorted(int(a) for a in s.get_legal_moves()), bool(s.is_terminal()),
                    int(s.get_game_result().value) if hasattr(s.get_game_result(), "value")
                    else int(s.get_game_result()), -1))
    return rec


def _occupied(board_fen):
    occ = []
    for row in board_fen.split("/"):
        for ch in row:
            if ch.isdigit():
                occ += [False] * int(ch)
            else:
                occ.append(True)
    return occ


def main():
    games = []
    rng = np.random.default_rng(2024)
    for g in range(6):
        games.append(play(az, START, 160, rng))
    for g in range(6):
        games.append(play(az, START, 300, rng, capture_bias=0.6))
    for fen in RICH:
        for _ in range(2):
            games.append(play(az, fen, 60, rng, capture_bias=0.3))
    # threefold: knights out and back twice (the start position occurs a third time)
    def act(sq_from, sq_to):
        return (sq_from << 6) | sq_to
    g1, f3, g8, f6 = 62, 45, 6, 21
    shuffle = [act(g1, f3), act(g8, f6), act(f3, g1), act(f6, g8)] * 2
    games.append(play(az, START, 12, rng, forced=shuffle))
    for fen in INSUFFICIENT:
        games.append(play(az, fen, 30, rng))
    fens, legal_flat, legal_off, term, res, moves, game_off = [], [], [0], [], [], [], [0]
    for gm in games:
        for f, legal, t, r, m in gm:
            fens.append(f)
            legal_flat.extend(legal)
            legal_off.append(len(legal_flat))
            term.append(t)
            res.append(r)
            moves.append(m)
        game_off.append(len(fens))
    path = os.path.join(HERE, "chess_rules.npz")
    np.savez_compressed(path, fens=np.array(fens), legal=np.array(legal_flat, np.int32),
                        legal_off=np.array(legal_off, np.int64), terminal=np.array(term),
                        result=np.array(res, np.int8), moves=np.array(moves, np.int32),
                        game_off=np.array(game_off, np.int64))
    print(f"{len(games)} games, {len(fens)} plies, {sum(term)} terminal; {path} {os.path.getsize(path)} B")


if __name__ == "__main__":
    main()
