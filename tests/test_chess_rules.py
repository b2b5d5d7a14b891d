"""The oracle's chess rules replay the reference engine's games (tests/golden/chess_rules.npz, made
by tests/golden/make_golden_chess.py from alphazero_py.ChessState): every ply's legal move list,
terminal flag and result, and every resulting position (board, side, castling rights, en-passant
square, clocks), bit for bit - including the engine's mirrored pawn-attack test and the
repetition rule over the game's positions."""
import os

import numpy as np

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "chess_rules.npz")


def _games():
    z = np.load(GOLD)
    go, off = z["game_off"], z["legal_off"]
    for g in range(len(go) - 1):
        yield [(str(z["fens"][i]), z["legal"][off[i]:off[i + 1]], bool(z["terminal"][i]),
                int(z["result"][i]), int(z["moves"][i])) for i in range(go[g], go[g + 1])]


def test_chess_oracle_replays_reference_games(oracle_lib):
    plies = terminal = 0
    for game in _games():
        pos = oracle_lib.chess_from_fen(game[0][0])
        seen = [pos]
        for t, (fen, legal, term, res, move) in enumerate(game):
            want = oracle_lib.chess_from_fen(fen)
            assert oracle_lib.chess_same(pos, want), (fen, t)
            assert pos["halfmove"] == want["halfmove"] and pos["fullmove"] == want["fullmove"], fen
            assert np.array_equal(oracle_lib.chess_legal(pos), legal), fen
            reps = sum(oracle_lib.chess_same(pos, q) for q in seen)
            assert oracle_lib.chess_terminal(pos, reps) == (term, res if term else 0), fen
            plies += 1
            terminal += term
            if move < 0:
                break
            pos = oracle_lib.chess_play(pos, move)
            seen.append(pos)
    assert plies > 2000 and terminal >= 15


def test_chess_action_encoding_round_trips(oracle_lib):
    """Every legal move of the fixture positions maps to a distinct action in [0, 4672) and back."""
    for game in list(_games())[:14]:
        for fen, legal, *_ in game[:40]:
            pos = oracle_lib.chess_from_fen(fen)
            acts = [oracle_lib.chess_action(pos, int(m)) for m in legal]
            assert all(0 <= a < 4672 for a in acts) and len(set(acts)) == len(acts)
            assert [oracle_lib.chess_move(pos, a) for a in acts] == [int(m) for m in legal]


def test_host_chess_position_replays_reference_games(oracle_lib):
    """The package's host-side chess position (roots, moves between searches) follows the same
    reference games: legal lists, terminal results, FENs and the 4672 encoding."""
    from omoknuni_quantum_b200.chess import ChessPosition
    games = list(_games())
    for gi, game in enumerate(games):
        pos = ChessPosition(game[0][0])
        for t, (fen, legal, term, res, move) in enumerate(game):
            assert pos.fen() == fen, (gi, t)
            if t % 5 == 0 or term or move < 0:
                assert pos.legal_moves() == [int(m) for m in legal], fen
                assert pos.result() == (res if term else 0), fen
                o = oracle_lib.chess_from_fen(fen)
                assert [pos.move_to_action(int(m)) for m in legal] == \
                    [oracle_lib.chess_action(o, int(m)) for m in legal]
            if move < 0:
                break
            pos.play(move)


def test_chess_roots_are_seeded_and_records_match_oracle(oracle_lib):
    from omoknuni_quantum_b200.chess import random_position, random_roots
    r1, n1 = random_roots(5, 3)
    r2, n2 = random_roots(5, 3)
    assert np.array_equal(r1, r2) and np.array_equal(n1, n2)
    p = random_position(5 * 1_000_003 + 1)
    o = oracle_lib.chess_from_fen(p.fen())
    assert oracle_lib.chess_same(o, r1[1, 0]) and r1[1, 0]["side"] == o["side"]
    assert 10 <= n1.min() and n1.max() <= 40
    # the prior positions are the game's, most recent first
    q = p.copy()
    assert np.array_equal(np.asarray(r1[1, 1]["sq"]), np.asarray(q.prior[0]["sq"]))


C960 = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "chess960.npz")


def _games960():
    z = np.load(C960)
    go, off = z["game_off"], z["legal_off"]
    for g in range(len(go) - 1):
        yield int(z["numbers"][g]), [(str(z["fens"][i]), z["legal"][off[i]:off[i + 1]], bool(z["terminal"][i]),
                                      int(z["result"][i]), int(z["moves"][i])) for i in range(go[g], go[g + 1])]


def test_chess960_start_positions_follow_the_reference_numbering():
    from omoknuni_quantum_b200.chess import chess960_fen
    starts = np.load(C960)["starts"]
    assert len(starts) == 960
    for k in range(960):
        assert chess960_fen(k) == str(starts[k]), k


def test_chess960_oracle_and_host_replay_reference_games(oracle_lib):
    """Chess960 games of the reference engine (kings starting on files c-f): legal moves incl.
    castling with arbitrary rook files, rights, terminal flags and resulting FENs, ply by ply."""
    from omoknuni_quantum_b200.chess import ChessPosition, chess960_fen
    castles = 0
    for number, game in _games960():
        pos = oracle_lib.chess_from_fen(game[0][0], chess960=True)
        host = ChessPosition(chess960_fen(number), chess960=True)
        seen = [pos]
        for t, (fen, legal, term, res, move) in enumerate(game):
            assert host.fen() == fen, (number, t)
            want = oracle_lib.chess_from_fen(fen, chess960=True)
            assert oracle_lib.chess_same(pos, want) and pos["castle"] == want["castle"], (number, t)
            assert np.array_equal(oracle_lib.chess_legal(pos), legal), (number, fen)
            if t % 3 == 0 or term:
                assert host.legal_moves() == [int(m) for m in legal], (number, fen)
            reps = sum(oracle_lib.chess_same(pos, q) for q in seen)
            assert oracle_lib.chess_terminal(pos, reps) == (term, res if term else 0), fen
            if move < 0:
                break
            frm, to = (move >> 6) & 63, move & 63
            castles += int((pos["sq"][frm] & 7) == 6 and abs(frm % 8 - to % 8) == 2)
            pos = oracle_lib.chess_play(pos, move)
            host.play(move)
            seen.append(pos)
    assert castles >= 10
