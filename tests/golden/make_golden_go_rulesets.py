"""Golden Go fixture for the reference's rule sets: alphazero_py.GoState(n, GoRuleSet.X) for
CHINESE (superko, area scoring, komi 7.5), JAPANESE and KOREAN (no superko, third repetition ends
the game with no result / a draw, territory + prisoners scoring, komi 6.5), built from the
reference sources (`make -C oracle ref`). Games: the double-ko cycle played until the rules stop
it, and seeded random games whose passes become likely late, so that games end by two passes and
get scored. For every ply: board, side to move, legal mask (is_legal_move), move, terminal flag
and GameResult. Writes tests/golden/go_rulesets.npz. Runs only in the build container.
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

RULES = {"chinese": az.GoRuleSet.CHINESE, "japanese": az.GoRuleSet.JAPANESE, "korean": az.GoRuleSet.KOREAN}


def result_code(r):
    return {"ONGOING": 0, "WIN_PLAYER1": 1, "WIN_PLAYER2": 2, "DRAW": 3}.get(r.name, 4)


def play(rules, n, fn, plies):
    s = az.GoState(n, RULES[rules])
    boards, players, legal, moves, term, res = [], [], [], [], [], []
    for t in range(plies + 1):
        b = board_of(s, n)
        mask = np.zeros(n * n + 1, bool)
        mask[n * n] = True
        for m in range(n * n):
            mask[m] = s.is_legal_move(m)
        boards.append(b)
        players.append(s.get_current_player())
        legal.append(mask)
        term.append(bool(s.is_terminal()))
        res.append(result_code(s.get_game_result()))
        if term[-1] or t == plies:
            moves.append(-2)
            break
        m = fn(t, mask)
        moves.append(n * n if m == -1 else m)
        s.make_move(m)
    return boards, players, legal, moves, term, res


def main():
    n = 9
    B = [(0, 1), (1, 0), (2, 1), (5, 6), (6, 7), (7, 6), (6, 5)]
    W = [(0, 2), (1, 3), (2, 2), (1, 1), (5, 5), (6, 4), (7, 5)]
    cyc = []
    for b, w in zip(B, W):
        cyc += [b[0] * n + b[1], w[0] * n + w[1]]
    cyc += [11, 60, -1, 10, 59, -1] * 4

    def scripted(t, mask):
        return cyc[t] if t < len(cyc) and (cyc[t] == -1 or mask[cyc[t]]) else -1

    rec = {}
    games = []
    for rules in ("japanese", "korean", "chinese"):
        games.append((rules, n, scripted, len(cyc)))
        for seed in (1, 2):
            r = np.random.default_rng(seed + 10 * len(games))

            def rnd(t, mask, r=r):
                cand = np.flatnonzero(mask[:-1])
                if len(cand) == 0 or r.random() < (0.02 if t < 60 else 0.45):
                    return -1
                return int(cand[r.integers(len(cand))])
            games.append((rules, n, rnd, 160))
    for gi, (rules, size, fn, plies) in enumerate(games):
        boards, players, legal, moves, term, res = play(rules, size, fn, plies)
        rec[f"g{gi}_rules"] = rules
        rec[f"g{gi}_n"] = size
        rec[f"g{gi}_boards"] = np.array(boards, np.int8)
        rec[f"g{gi}_players"] = np.array(players, np.int8)
        rec[f"g{gi}_legal"] = np.packbits(np.array(legal), axis=1)
        rec[f"g{gi}_moves"] = np.array(moves, np.int16)
        rec[f"g{gi}_terminal"] = np.array(term)
        rec[f"g{gi}_result"] = np.array(res, np.int8)
        print(f"game {gi} {rules}: {len(moves)} plies, terminal {term[-1]}, result {res[-1]}")
    rec["games"] = len(games)
    path = os.path.join(HERE, "go_rulesets.npz")
    np.savez_compressed(path, **rec)
    print(path, os.path.getsize(path))


if __name__ == "__main__":
    main()
