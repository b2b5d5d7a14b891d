"""Host-side Go position: root construction and move application between searches.

The rules are those the device engine searches with - the reference's GoState with Chinese rules
(src/games/go/go_state.cpp:227-420, go_rules.cpp:34-110, isTerminal :502-506): no play on an
occupied point or on the ko point; opponent groups without liberties are captured; suicide is
illegal; capturing exactly one stone makes its point the ko point; pass is always legal, clears
the ko point, and two consecutive passes end the game. With positional superko (on by default,
as GoState's default constructor has it) a move is also refused when the position it makes -
board after captures plus the new ko point - equals one recorded after an earlier non-pass move
of the game (GoState::isLegalMove, go_state.cpp:359-418). Positions are keyed by 64-bit Zobrist
hashes (``position_key``), the keys the device engine uses. Actions are y * n + x, pass = n * n
(the NN action space; GoState itself encodes pass as -1).

This is host bookkeeping for a handful of moves per search (root positions, the move a search
chose); the search itself never calls it.
"""
from __future__ import annotations

import numpy as np

HISTORY = 8
_M64 = (1 << 64) - 1
_KEY_TABLES = {}


def _mix64(x: int) -> int:
    """SplitMix64 finaliser (Steele, Lea & Flood 2014)."""
    x &= _M64
    x ^= x >> 30
    x = (x * 0xBF58476D1CE4E5B9) & _M64
    x ^= x >> 27
    x = (x * 0x94D049BB133111EB) & _M64
    x ^= x >> 31
    return x


def _key_tables(n: int):
    """uint64 stone keys [n*n, 3] (colour 1, 2) and ko keys [n*n]."""
    t = _KEY_TABLES.get(n)
    if t is None:
        stones = np.zeros((n * n, 3), np.uint64)
        for c in range(n * n):
            for col in (1, 2):
                stones[c, col] = _mix64(0x6A09E667F3BCC909 ^ (c * 4 + col))
        ko = np.array([_mix64(0xBB67AE8584CAA73B ^ c) for c in range(n * n)], np.uint64)
        t = _KEY_TABLES[n] = (stones, ko)
    return t


def side_key(player: int) -> int:
    """Side-to-move key of the repetition rule (Japanese / Korean): mix64(0x3C6EF372FE94F82B ^ p)."""
    return _mix64(0x3C6EF372FE94F82B ^ int(player))


def position_key(board: np.ndarray, ko: int = -1) -> int:
    """64-bit key of (stones, ko point): XOR of mix64(0x6A09E667F3BCC909 ^ (cell * 4 + colour))
    over the stones, and mix64(0xBB67AE8584CAA73B ^ ko) when there is a ko point."""
    b = np.asarray(board).reshape(-1)
    stones, kok = _key_tables(int(round(np.sqrt(b.size))))
    idx = np.flatnonzero(b)
    k = np.bitwise_xor.reduce(stones[idx, b[idx].astype(np.int64)]) if len(idx) else np.uint64(0)
    if ko >= 0:
        k = np.uint64(k) ^ kok[ko]
    return int(k)


class GoPosition:
    def __init__(self, board_size: int = 19, komi: float = None, superko: bool = True,
                 rules: str = "chinese"):
        """``rules``: "chinese" (positional superko unless ``superko=False``, area scoring, komi
        7.5), "japanese" or "korean" (no superko; a third repetition of (board, ko point, side to
        move) ends the game - no result / draw; territory + prisoners scoring, komi 6.5),
        as GoState(board_size, RuleSet) sets them (go_state.cpp:15-66, 342-356, 516-544)."""
        if rules not in ("chinese", "japanese", "korean"):
            raise ValueError(f"unknown Go rules {rules!r}")
        self.n = int(board_size)
        self.rules = rules
        self.komi = float(komi) if komi is not None else (7.5 if rules == "chinese" else 6.5)
        self.superko = bool(superko) and rules == "chinese"
        self.cycle = rules != "chinese"
        self.repeated = False     # a third repetition happened (Japanese / Korean)
        self.prisoners = [0, 0, 0]  # stones captured by black [1] and by white [2]
        # superko: keys after each non-pass move (GoState::position_history_); repetition rule:
        # keys with the side to move after every move (position_frequency_)
        self.keys = []
        self.board = np.zeros((self.n, self.n), np.int8)
        self.to_move = 1
        self.ko = -1
        self.passes = 0
        self.history = [self.board.copy()]  # most recent last

    @property
    def pass_action(self) -> int:
        return self.n * self.n

    def copy(self) -> "GoPosition":
        g = GoPosition.__new__(GoPosition)
        g.n, g.rules, g.komi, g.superko, g.cycle = self.n, self.rules, self.komi, self.superko, self.cycle
        g.repeated, g.prisoners = self.repeated, list(self.prisoners)
        g.keys = list(self.keys)
        g.board = self.board.copy()
        g.to_move, g.ko, g.passes = self.to_move, self.ko, self.passes
        g.history = [h.copy() for h in self.history[-HISTORY:]]
        return g

    def is_terminal(self) -> bool:
        return self.passes >= 2 or self.repeated

    def _group(self, b, y, x):
        """Stones of the group at (y, x) and whether it has a liberty."""
        color = b[y, x]
        stack, seen, lib = [(y, x)], {(y, x)}, False
        while stack:
            cy, cx = stack.pop()
            for ny, nx in ((cy - 1, cx), (cy + 1, cx), (cy, cx - 1), (cy, cx + 1)):
                if 0 <= ny < self.n and 0 <= nx < self.n and (ny, nx) not in seen:
                    if b[ny, nx] == 0:
                        lib = True
                    elif b[ny, nx] == color:
                        seen.add((ny, nx))
                        stack.append((ny, nx))
        return seen, lib

    def _try(self, action: int):
        """(new board, new ko) or None if illegal; does not change the position."""
        if action == self.pass_action:
            return self.board.copy(), -1
        if not 0 <= action < self.pass_action or action == self.ko:
            return None
        y, x = divmod(action, self.n)
        if self.board[y, x] != 0:
            return None
        b = self.board.copy()
        b[y, x] = self.to_move
        opp = 3 - self.to_move
        groups, captured, last = 0, 0, -1
        for ny, nx in ((y - 1, x), (y + 1, x), (y, x - 1), (y, x + 1)):
            if 0 <= ny < self.n and 0 <= nx < self.n and b[ny, nx] == opp:
                stones, lib = self._group(b, ny, nx)
                if not lib:
                    groups += 1
                    captured += len(stones)
                    for sy, sx in stones:
                        b[sy, sx] = 0
                    last = next(iter(stones))
        if captured == 0 and not self._group(b, y, x)[1]:
            return None  # suicide
        ko = last[0] * self.n + last[1] if (groups == 1 and captured == 1) else -1
        if self.superko and self.keys and position_key(b, ko) in self.keys:
            return None  # positional superko
        return b, ko

    def is_legal(self, action: int) -> bool:
        return self._try(int(action)) is not None

    def _group_liberties(self):
        """Per cell: the liberty count of its group (0 on empty cells)."""
        n, b = self.n, self.board
        libs = np.zeros((n, n), np.int32)
        seen = np.zeros((n, n), bool)
        for y in range(n):
            for x in range(n):
                if b[y, x] == 0 or seen[y, x]:
                    continue
                stones, empties, stack = [], set(), [(y, x)]
                seen[y, x] = True
                while stack:
                    cy, cx = stack.pop()
                    stones.append((cy, cx))
                    for ny, nx in ((cy - 1, cx), (cy + 1, cx), (cy, cx - 1), (cy, cx + 1)):
                        if 0 <= ny < n and 0 <= nx < n:
                            if b[ny, nx] == 0:
                                empties.add((ny, nx))
                            elif b[ny, nx] == b[y, x] and not seen[ny, nx]:
                                seen[ny, nx] = True
                                stack.append((ny, nx))
                for cy, cx in stones:
                    libs[cy, cx] = len(empties)
        return libs

    def legal_mask(self) -> np.ndarray:
        """bool [n*n + 1], pass last. A cell with an empty neighbour that captures nothing and is
        not the ko point is a legal placement whose new position key is one XOR away (no ko
        point arises without a capture), so only the other cells need the full trial move."""
        n = self.n
        m = np.zeros(self.pass_action + 1, bool)
        libs = self._group_liberties()
        b = self.board
        opp = 3 - self.to_move
        stones, _ = _key_tables(n)
        base = position_key(b, -1) if self.superko and self.keys else 0
        keys = set(self.keys) if self.superko else ()
        for a in np.flatnonzero(b.reshape(-1) == 0):
            a = int(a)
            y, x = divmod(a, n)
            empty_nb = capture = False
            for ny, nx in ((y - 1, x), (y + 1, x), (y, x - 1), (y, x + 1)):
                if 0 <= ny < n and 0 <= nx < n:
                    if b[ny, nx] == 0:
                        empty_nb = True
                    elif b[ny, nx] == opp and libs[ny, nx] == 1:
                        capture = True
            if empty_nb and not capture and a != self.ko:
                m[a] = not (keys and (base ^ int(stones[a, self.to_move])) in keys)
            else:
                m[a] = self._try(a) is not None
        m[self.pass_action] = True
        return m

    def play(self, action: int) -> None:
        res = self._try(int(action))
        if res is None:
            raise ValueError(f"illegal Go move {action} for player {self.to_move}")
        before = int((self.board == 3 - self.to_move).sum())
        self.board, self.ko = res
        self.prisoners[self.to_move] += before - int((self.board == 3 - self.to_move).sum())
        if action != self.pass_action and not self.cycle:
            self.keys.append(position_key(self.board, self.ko))
        self.passes = self.passes + 1 if action == self.pass_action else 0
        self.to_move = 3 - self.to_move
        if self.cycle and not self.repeated:
            k = position_key(self.board, self.ko) ^ side_key(self.to_move)
            self.keys.append(k)
            self.repeated = self.keys.count(k) >= 3
        self.history.append(self.board.copy())
        del self.history[:-HISTORY]

    def history_planes(self) -> np.ndarray:
        """int8 [8, n, n]: [0] = this position, [k] = k plies earlier (zeros before the game)."""
        h = np.zeros((HISTORY, self.n, self.n), np.int8)
        for k, b in enumerate(reversed(self.history[-HISTORY:])):
            h[k] = b
        return h

    def score(self):
        """(black, white) scores (GoRules::calculateScores / getTerritoryOwnership,
        go_rules.cpp:211-260, 343-380): each empty region bordered by one colour only counts for
        that colour; Chinese rules add the stones on the board, Japanese / Korean the prisoners;
        komi goes to white. No stones are marked dead."""
        b = self.board
        if self.rules == "chinese":
            black = float((b == 1).sum())
            white = float((b == 2).sum()) + self.komi
        else:
            black = float(self.prisoners[1])
            white = float(self.prisoners[2]) + self.komi
        seen = np.zeros_like(b, dtype=bool)
        for y in range(self.n):
            for x in range(self.n):
                if b[y, x] != 0 or seen[y, x]:
                    continue
                stack, region, border = [(y, x)], 0, set()
                seen[y, x] = True
                while stack:
                    cy, cx = stack.pop()
                    region += 1
                    for ny, nx in ((cy - 1, cx), (cy + 1, cx), (cy, cx - 1), (cy, cx + 1)):
                        if 0 <= ny < self.n and 0 <= nx < self.n:
                            if b[ny, nx] == 0 and not seen[ny, nx]:
                                seen[ny, nx] = True
                                stack.append((ny, nx))
                            elif b[ny, nx] != 0:
                                border.add(int(b[ny, nx]))
                if border == {1}:
                    black += region
                elif border == {2}:
                    white += region
        return black, white

    def result(self) -> int:
        """The reference's GameResult: 0 ongoing, 1 black wins, 2 white wins, 3 draw, 4 no result
        (a Japanese repetition)."""
        if not self.is_terminal():
            return 0
        if self.repeated:
            return 4 if self.rules == "japanese" else 3
        black, white = self.score()
        return 1 if black > white else 2 if white > black else 3

    def root_keys(self) -> np.ndarray:
        """uint64 [k]: the game's position keys so far - the engine's root history for superko
        (Chinese) or for the repetition rule (Japanese / Korean)."""
        return np.array(self.keys, np.uint64)

    def meta(self) -> np.ndarray:
        """int32 [3]: side to move, ko point, consecutive passes (the engine's root record)."""
        return np.array([self.to_move, self.ko, self.passes], np.int32)


def random_position(seed: int, moves: int = 60, board_size: int = 19) -> GoPosition:
    """``moves`` uniformly random legal non-pass moves from the empty board, colours alternating
    from black, captures resolved by the rules (benchmark config 3's "60 stones placed at random
    under the legality rules"); numpy.random.default_rng(seed)."""
    rng = np.random.default_rng(seed)
    g = GoPosition(board_size)
    for _ in range(moves):
        cand = np.flatnonzero(g.legal_mask()[:-1])
        if len(cand) == 0:
            break
        g.play(int(cand[rng.integers(len(cand))]))
    return g


def random_roots(seed: int, count: int, moves: int = 60, board_size: int = 19):
    """``count`` seeded Go roots (root i uses seed ``seed * 1_000_003 + i``):
    (history int8 [count, 8, n, n], meta int32 [count, 3])."""
    ps = [random_position(seed * 1_000_003 + i, moves, board_size) for i in range(count)]
    return np.stack([p.history_planes() for p in ps]), np.stack([p.meta() for p in ps])
