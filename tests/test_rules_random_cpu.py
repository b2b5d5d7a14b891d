"""Randomised cross-checks of the host game positions (root construction and self-play) against
the oracle's C++ rules: random legal games on small Go boards (captures, ko and positional
superko are exercised) and chess / Chess960 games, compared at every ply - legal moves,
the resulting position, and the superko keys."""
import numpy as np


def test_go_host_position_matches_oracle_on_random_games(oracle_lib):
    from omoknuni_quantum_b200.go import GoPosition, position_key
    refusals = captures = 0
    for n, seed in [(7, s) for s in range(6)] + [(9, s) for s in range(4)]:
        rng = np.random.default_rng(1000 * n + seed)
        g = GoPosition(n)
        for _ in range(4 * n * n):
            if g.is_terminal():
                break
            mask = g.legal_mask()
            plain = oracle_lib.go_legal(g.board, g.to_move, g.ko)
            orc = oracle_lib.go_legal_superko(g.board, g.to_move, g.ko, g.root_keys())
            assert np.array_equal(mask, orc), (n, seed)
            refusals += int(plain.sum() - orc.sum())
            # mostly stones, some passes
            cand = np.flatnonzero(mask[:-1])
            a = g.pass_action if len(cand) == 0 or rng.random() < 0.03 else int(rng.choice(cand))
            if a != g.pass_action:
                nb, nko = oracle_lib.go_play(g.board, g.to_move, a, g.ko)
                before = int((g.board != 0).sum())
            g.play(a)
            if a != g.pass_action:
                assert np.array_equal(g.board, nb) and g.ko == nko
                assert position_key(g.board, g.ko) == oracle_lib.go_key(g.board, g.ko)
                captures += int(before + 1 - (g.board != 0).sum())
    # positional-superko refusals beyond simple ko are rare in random play; the reference-game
    # fixtures of test_go_rules.py pin them
    assert captures > 50


def test_chess_host_position_matches_oracle_on_random_games(oracle_lib):
    from omoknuni_quantum_b200.chess import ChessPosition, chess960_fen
    starts = [(None, False)] + [(chess960_fen(k), True) for k in (7, 100, 333, 518, 700)]
    for i, (fen, c960) in enumerate(starts):
        rng = np.random.default_rng(500 + i)
        p = ChessPosition(fen, chess960=True) if c960 else ChessPosition()
        o = oracle_lib.chess_from_fen(p.fen(), chess960=c960)
        for ply in range(120):
            legal = sorted(int(m) for m in p.legal_moves())
            assert legal == sorted(int(m) for m in oracle_lib.chess_legal(o)), (i, ply, p.fen())
            if not legal or p.result() != 0:
                break
            m = legal[int(rng.integers(len(legal)))]
            p.play(m)
            o = oracle_lib.chess_play(o, m)
            want = oracle_lib.chess_from_fen(p.fen(), chess960=c960)
            assert oracle_lib.chess_same(o, want) and o["castle"] == want["castle"] and o["ep"] == want["ep"], (i, ply)


def test_go_fast_legal_mask_equals_trial_moves():
    """GoPosition.legal_mask's shortcut (empty neighbour, no capture, not ko) agrees with the full
    trial move on every cell of random positions, with and without superko keys."""
    from omoknuni_quantum_b200.go import GoPosition
    for n, seed in [(9, 1), (9, 2), (13, 3), (19, 4)]:
        rng = np.random.default_rng(seed)
        for superko in (True, False):
            g = GoPosition(n, superko=superko)
            for _ in range(3 * n * n // 2):
                slow = np.array([g._try(a) is not None for a in range(n * n)] + [True])
                assert np.array_equal(g.legal_mask(), slow)
                cand = np.flatnonzero(slow[:-1])
                if len(cand) == 0:
                    break
                g.play(int(cand[rng.integers(len(cand))]))
