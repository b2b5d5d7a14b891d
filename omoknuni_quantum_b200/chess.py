"""Host-side chess position: root construction and move application between searches.

The rules are those the device engine searches with - the reference's ChessState
(src/games/chess/chess_state.cpp, chess_rules.cpp; standard chess) as it behaves, including:
its pawn-attack test looks on the mirrored side (chess_rules.cpp:135-150), so a king may step
next to an enemy pawn and be captured, and a side without a king is never in check; a double
pawn push always sets the en-passant square; the repetition key is the piece placement alone
(the position hash is only updated for piece changes, chess_state.cpp:255-267); terminal order
is no legal move, insufficient material (chess_rules.cpp:236-394), halfmove clock >= 100, third
occurrence (chess_state.cpp:623-676).

Squares are rank * 8 + file with rank 0 = the eighth rank; white pawns move towards rank 0.
Moves use the reference encoding (promotion << 12) | (from << 6) | to (promotion 1 queen, 2 rook,
3 bishop, 4 knight). The engine's action space is the AlphaZero 8x8x73 = 4672 encoding in the
mover's frame (``move_to_action`` / ``action_to_move``).

Host bookkeeping for a handful of moves per search; the search itself never calls it.
"""
from __future__ import annotations

import numpy as np

PAWN, KNIGHT, BISHOP, ROOK, QUEEN, KING = 1, 2, 3, 4, 5, 6
WHITE, BLACK = 1, 2
START_FEN = "rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1"
PRIOR = 100  # earlier positions kept for the repetition count and the history planes

# position record shared with the engine (80 bytes, the layout of the engine's root records)
POS_DTYPE = np.dtype([("sq", np.int8, 64), ("side", np.int8), ("castle", np.int8), ("ep", np.int8),
                      ("reps", np.int8), ("halfmove", np.int16), ("fullmove", np.int16),
                      ("c960", np.int8), ("rook_file", np.int8, 4), ("pad", np.int8, 3)])
_KRN = ((0, 1), (0, 2), (0, 3), (0, 4), (1, 2), (1, 3), (1, 4), (2, 3), (2, 4), (3, 4))

_KNIGHT = ((-2, -1), (-2, 1), (-1, -2), (-1, 2), (1, -2), (1, 2), (2, -1), (2, 1))
_KING = ((-1, -1), (-1, 0), (-1, 1), (0, -1), (0, 1), (1, -1), (1, 0), (1, 1))
_DIAG = ((-1, -1), (-1, 1), (1, -1), (1, 1))
_ORTHO = ((-1, 0), (1, 0), (0, -1), (0, 1))
_QUEEN_DIRS = ((-1, 0), (-1, 1), (0, 1), (1, 1), (1, 0), (1, -1), (0, -1), (-1, -1))


def _color(p: int) -> int:
    return 0 if p == 0 else (BLACK if p & 8 else WHITE)


def _piece(t: int, c: int) -> int:
    return t | (8 if c == BLACK else 0)


def chess960_fen(number: int) -> str:
    """Start FEN of Chess960 position ``number`` (0..959) in the reference's numbering
    (Chess960::getPermutation, src/games/chess/chess960.cpp:454-530: n % 4 picks the bishop on
    files a/c/e/g, n / 4 % 4 the one on b/d/f/h, n / 16 % 6 the queen among the free files,
    n / 96 the knight pair in lexicographic order, then rook, king, rook on what is left; 518 is special-cased to
    the classical setup), the
    castling field naming the rook files as the reference prints it."""
    n = int(number)
    if not 0 <= n < 960:
        raise ValueError("Chess960 position numbers are 0..959")
    if n == 518:   # hard-coded to the classical setup (chess960.cpp:449-453); 521 decodes to it too
        n = 521
    row = [""] * 8
    row[2 * (n % 4)] = "b"        # files a, c, e, g
    n //= 4
    row[2 * (n % 4) + 1] = "b"    # files b, d, f, h
    n //= 4
    free = [f for f in range(8) if not row[f]]
    row[free[n % 6]] = "q"
    n //= 6
    free = [f for f in range(8) if not row[f]]
    for i in _KRN[n]:
        row[free[i]] = "n"
    free = [f for f in range(8) if not row[f]]
    row[free[0]], row[free[1]], row[free[2]] = "r", "k", "r"
    back = "".join(row)
    cast = "ABCDEFGH"[free[2]] + "ABCDEFGH"[free[0]] + "abcdefgh"[free[2]] + "abcdefgh"[free[0]]
    return f"{back}/pppppppp/8/8/8/8/PPPPPPPP/{back.upper()} w {cast} - 0 1"


class ChessPosition:
    def __init__(self, fen: str = START_FEN, chess960: bool = False):
        self.sq = [0] * 64
        self.side, self.castle, self.ep, self.halfmove, self.fullmove = WHITE, 0, -1, 0, 1
        self.c960 = bool(chess960)
        self.rook_file = [7, 0, 7, 0]  # original rook files: white k, white q, black k, black q
        self._parse(fen)
        self.prior: list = []   # earlier positions (records), most recent first
        self.reps = 1

    # -- FEN -----------------------------------------------------------------------------------
    def _parse(self, fen: str) -> None:
        f = fen.split()
        s = 0
        for ch in f[0]:
            if ch == "/":
                continue
            if ch.isdigit():
                s += int(ch)
                continue
            self.sq[s] = _piece("pnbrqk".index(ch.lower()) + 1, BLACK if ch.islower() else WHITE)
            s += 1
        if s != 64:
            raise ValueError(f"bad FEN {fen!r}")
        self.side = BLACK if f[1] == "b" else WHITE
        self.castle = sum(b for c, b in (("K", 1), ("Q", 2), ("k", 4), ("q", 8)) if c in f[2])
        for ch in f[2]:  # rook files (ChessState::setFromFEN, chess_state.cpp:460-487)
            if ch.upper() in "ABCDEFGH" and ch not in "-":
                white = ch.isupper()
                file = "ABCDEFGH".index(ch.upper())
                k = self._king(WHITE if white else BLACK)
                kside = k >= 0 and file > (k & 7)
                self.castle |= (1 if kside else 2) if white else (4 if kside else 8)
                self.rook_file[(0 if white else 2) + (0 if kside else 1)] = file
        self.ep = -1 if f[3] == "-" else (8 - int(f[3][1])) * 8 + "abcdefgh".index(f[3][0])
        self.halfmove = int(f[4]) if len(f) > 4 else 0
        self.fullmove = int(f[5]) if len(f) > 5 else 1

    def fen(self) -> str:
        rows = []
        for r in range(8):
            row, empty = "", 0
            for f in range(8):
                p = self.sq[r * 8 + f]
                if p == 0:
                    empty += 1
                    continue
                if empty:
                    row += str(empty)
                    empty = 0
                ch = "pnbrqk"[(p & 7) - 1]
                row += ch if p & 8 else ch.upper()
            rows.append(row + (str(empty) if empty else ""))
        if self.c960:  # the reference prints rook files in Chess960 mode
            cs = "".join(("ABCDEFGH" if b < 4 else "abcdefgh")[self.rook_file[i]]
                         for i, b in enumerate((1, 2, 4, 8)) if self.castle & b) or "-"
        else:
            cs = "".join(c for c, b in (("K", 1), ("Q", 2), ("k", 4), ("q", 8)) if self.castle & b) or "-"
        ep = "-" if self.ep < 0 else "abcdefgh"[self.ep % 8] + str(8 - self.ep // 8)
        return f"{'/'.join(rows)} {'w' if self.side == WHITE else 'b'} {cs} {ep} {self.halfmove} {self.fullmove}"

    # -- rules ---------------------------------------------------------------------------------
    def _attacked(self, s: int, by: int) -> bool:
        sq, r, f = self.sq, s >> 3, s & 7
        pr = r + (-1 if by == WHITE else 1)   # the reference's pawn direction (mirrored)
        for df in (-1, 1):
            if 0 <= pr < 8 and 0 <= f + df < 8 and sq[pr * 8 + f + df] == _piece(PAWN, by):
                return True
        for dr, df in _KNIGHT:
            if 0 <= r + dr < 8 and 0 <= f + df < 8 and sq[(r + dr) * 8 + f + df] == _piece(KNIGHT, by):
                return True
        for dr, df in _KING:
            if 0 <= r + dr < 8 and 0 <= f + df < 8 and sq[(r + dr) * 8 + f + df] == _piece(KING, by):
                return True
        for dirs, slider in ((_DIAG, BISHOP), (_ORTHO, ROOK)):
            for dr, df in dirs:
                rr, ff = r + dr, f + df
                while 0 <= rr < 8 and 0 <= ff < 8:
                    q = sq[rr * 8 + ff]
                    if q:
                        if _color(q) == by and (q & 7) in (slider, QUEEN):
                            return True
                        break
                    rr, ff = rr + dr, ff + df
        return False

    def _king(self, color: int) -> int:
        k = _piece(KING, color)
        for s in range(64):
            if self.sq[s] == k:
                return s
        return -1

    def in_check(self, color: int | None = None) -> bool:
        c = self.side if color is None else color
        k = self._king(c)
        return k >= 0 and self._attacked(k, 3 - c)

    def _pseudo(self):
        sq, me, out = self.sq, self.side, []
        for s in range(64):
            p = sq[s]
            if _color(p) != me:
                continue
            r, f, t = s >> 3, s & 7, p & 7
            if t == PAWN:
                d = -1 if me == WHITE else 1
                nr = r + d
                if 0 <= nr < 8:
                    if sq[nr * 8 + f] == 0:
                        if nr in (0, 7):
                            out += [(pc << 12) | (s << 6) | (nr * 8 + f) for pc in (1, 2, 3, 4)]
                        else:
                            out.append((s << 6) | (nr * 8 + f))
                        if (me == WHITE and r == 6) or (me == BLACK and r == 1):
                            n2 = (nr + d) * 8 + f
                            if sq[n2] == 0:
                                out.append((s << 6) | n2)
                    for df in (-1, 1):
                        nf = f + df
                        if not 0 <= nf < 8:
                            continue
                        to = nr * 8 + nf
                        if sq[to] and _color(sq[to]) != me:
                            if nr in (0, 7):
                                out += [(pc << 12) | (s << 6) | to for pc in (1, 2, 3, 4)]
                            else:
                                out.append((s << 6) | to)
                        if self.ep == to:
                            out.append((s << 6) | to)
            elif t in (KNIGHT, KING):
                for dr, df in (_KNIGHT if t == KNIGHT else _KING):
                    rr, ff = r + dr, f + df
                    if 0 <= rr < 8 and 0 <= ff < 8 and (sq[rr * 8 + ff] == 0 or _color(sq[rr * 8 + ff]) != me):
                        out.append((s << 6) | (rr * 8 + ff))
            else:
                dirs = (_DIAG if t == BISHOP else _ORTHO if t == ROOK else _DIAG + _ORTHO)
                for dr, df in dirs:
                    rr, ff = r + dr, f + df
                    while 0 <= rr < 8 and 0 <= ff < 8:
                        q = sq[rr * 8 + ff]
                        if q == 0:
                            out.append((s << 6) | (rr * 8 + ff))
                        else:
                            if _color(q) != me:
                                out.append((s << 6) | (rr * 8 + ff))
                            break
                        rr, ff = rr + dr, ff + df
        if not self.in_check(me):
            ks = self.castle & (1 if me == WHITE else 4)
            qs = self.castle & (2 if me == WHITE else 8)
            k = self._king(me)
            if (ks or qs) and k >= 0:
                home = 7 if me == WHITE else 0
                for kingside, right in ((True, ks), (False, qs)):
                    if not right:
                        continue
                    tfile = ((k & 7) if self.c960 else 4) + (2 if kingside else -2)
                    if not 0 <= tfile <= 7:
                        continue  # the reference's target leaves the board here
                    target = home * 8 + tfile
                    fr, ff, tf = k >> 3, k & 7, target & 7
                    rook_file = self.rook_file[(0 if me == WHITE else 2) + (0 if kingside else 1)]
                    rook_sq = fr * 8 + rook_file
                    if sq[rook_sq] != _piece(ROOK, me):
                        continue
                    lo, hi = min(ff, rook_file), max(ff, rook_file)
                    ok = all(sq[fr * 8 + x] == 0 for x in range(lo + 1, hi))
                    step = 1 if tf > ff else -1
                    x = ff
                    while ok and x != tf + step:
                        s2 = fr * 8 + x
                        if s2 != k:
                            if self._attacked(s2, 3 - me) or (s2 != rook_sq and sq[s2] != 0):
                                ok = False
                        x += step
                    if ok:
                        out.append((k << 6) | target)
        return out

    def _apply(self, m: int) -> None:
        """ChessState::makeMove (chess_state.cpp:1232-1346), without history bookkeeping."""
        sq = self.sq
        frm, to, promo = (m >> 6) & 63, m & 63, (m >> 12) & 7
        piece, captured = sq[frm], sq[to]
        me = _color(piece)
        self.halfmove = 0 if (piece & 7) == PAWN or captured else self.halfmove + 1
        old_ep, self.ep = self.ep, -1
        if (piece & 7) == PAWN:
            fr, tr = frm >> 3, to >> 3
            if abs(fr - tr) == 2:
                self.ep = ((fr + tr) // 2) * 8 + (frm & 7)
            if to == old_ep:
                sq[fr * 8 + (to & 7)] = 0
            if promo:
                piece = _piece({1: QUEEN, 2: ROOK, 3: BISHOP, 4: KNIGHT}[promo], me)
        if (piece & 7) == KING and abs((frm & 7) - (to & 7)) == 2:
            r = frm >> 3
            kingside = (to & 7) > (frm & 7)
            rfile = self.rook_file[(0 if me == WHITE else 2) + (0 if kingside else 1)]
            tfile = ((to & 7) - 1 if kingside else (to & 7) + 1) if self.c960 else (5 if kingside else 3)
            rf, rt = r * 8 + rfile, r * 8 + tfile
            rook = sq[rf]
            sq[rf] = 0
            sq[rt] = rook
        if (piece & 7) == KING:
            self.castle &= ~(3 if me == WHITE else 12)
        if (piece & 7) == ROOK and (frm >> 3) == (7 if me == WHITE else 0):
            base = 0 if me == WHITE else 2
            if (frm & 7) == self.rook_file[base]:
                self.castle &= ~(1 if me == WHITE else 4)
            elif (frm & 7) == self.rook_file[base + 1]:
                self.castle &= ~(2 if me == WHITE else 8)
        if captured and (captured & 7) == ROOK:
            c = _color(captured)
            base = 0 if c == WHITE else 2
            if (to >> 3) == (7 if c == WHITE else 0):
                if (to & 7) == self.rook_file[base]:
                    self.castle &= ~(1 if c == WHITE else 4)
                elif (to & 7) == self.rook_file[base + 1]:
                    self.castle &= ~(2 if c == WHITE else 8)
        sq[frm], sq[to] = 0, piece
        self.side = 3 - self.side
        if self.side == WHITE:
            self.fullmove += 1

    def _copy_board(self) -> "ChessPosition":
        c = ChessPosition.__new__(ChessPosition)
        c.sq = list(self.sq)
        c.side, c.castle, c.ep, c.halfmove, c.fullmove = self.side, self.castle, self.ep, self.halfmove, self.fullmove
        c.c960, c.rook_file = self.c960, list(self.rook_file)
        c.prior, c.reps = self.prior, self.reps
        return c

    def _legal(self, m: int) -> bool:
        """A pseudo-legal move that does not leave the mover's king attacked."""
        c = self._copy_board()
        c._apply(m)
        return not c.in_check(self.side)

    def legal_moves(self) -> list:
        """Legal moves (reference encoding), sorted."""
        return sorted(m for m in self._pseudo() if self._legal(m))

    def has_legal_move(self) -> bool:
        return any(self._legal(m) for m in self._pseudo())

    def _insufficient(self) -> bool:
        cnt = {(c, t): 0 for c in (WHITE, BLACK) for t in range(1, 7)}
        light = {WHITE: False, BLACK: False}
        dark = {WHITE: False, BLACK: False}
        pieces = 0
        for s, p in enumerate(self.sq):
            if not p:
                continue
            pieces += 1
            c, t = _color(p), p & 7
            cnt[(c, t)] += 1
            if t == BISHOP:
                (light if ((s >> 3) + (s & 7)) % 2 == 0 else dark)[c] = True
        if pieces == 2:
            return True
        if any(cnt[(c, t)] for c in (WHITE, BLACK) for t in (PAWN, ROOK, QUEEN)):
            return False
        wn, bn, wb, bb = cnt[(WHITE, KNIGHT)], cnt[(BLACK, KNIGHT)], cnt[(WHITE, BISHOP)], cnt[(BLACK, BISHOP)]
        return ((wn, bn) in ((1, 0), (0, 1)) and wb == bb == 0
                or (wb, bb) in ((1, 0), (0, 1)) and wn == bn == 0
                or wn == bn == 0 and wb == bb == 1 and (light[WHITE] and light[BLACK] or dark[WHITE] and dark[BLACK])
                or (wn, bn, wb, bb) in ((2, 0, 0, 0), (0, 2, 0, 0), (1, 1, 0, 0), (1, 0, 0, 1), (0, 1, 1, 0)))

    def result(self) -> int:
        """The reference's GameResult: 0 ongoing, 1 white wins, 2 black wins, 3 draw."""
        if not self.has_legal_move():
            return (2 if self.side == WHITE else 1) if self.in_check() else 3
        if self._insufficient() or self.halfmove >= 100 or self.reps >= 3:
            return 3
        return 0

    def is_terminal(self) -> bool:
        return self.result() != 0

    def record(self) -> np.ndarray:
        r = np.zeros((), POS_DTYPE)
        r["sq"] = self.sq
        r["side"], r["castle"], r["ep"], r["reps"] = self.side, self.castle, self.ep, min(self.reps, 127)
        r["halfmove"], r["fullmove"] = self.halfmove, self.fullmove
        r["c960"] = int(self.c960)
        r["rook_file"] = self.rook_file
        return r

    def play(self, move: int) -> None:
        """Play a legal move (reference encoding); keeps the earlier positions for repetitions."""
        if move not in self._pseudo() or not self._legal(move):
            raise ValueError(f"illegal chess move {move}")
        rec = self.record()
        self._apply(int(move))
        self.prior = ([rec] + self.prior)[:PRIOR]
        key = bytes(np.asarray(self.sq, np.int8))
        self.reps = 1 + sum(bytes(p["sq"]) == key for p in self.prior)

    def copy(self) -> "ChessPosition":
        c = self._copy_board()
        c.prior = list(self.prior)
        return c

    # -- engine records ------------------------------------------------------------------------
    @classmethod
    def from_records(cls, records: np.ndarray, nprior: int) -> "ChessPosition":
        """The position of engine root records (POS_DTYPE [1 + PRIOR], as ``root_records``
        writes them) with ``nprior`` earlier positions; the inverse of ``root_records``."""
        r = records[0]
        c = cls.__new__(cls)
        c.sq = [int(x) for x in r["sq"]]
        c.side, c.castle, c.ep = int(r["side"]), int(r["castle"]), int(r["ep"])
        c.halfmove, c.fullmove = int(r["halfmove"]), int(r["fullmove"])
        c.c960, c.rook_file = bool(r["c960"]), [int(x) for x in r["rook_file"]]
        c.reps = int(r["reps"])
        c.prior = [np.array(records[1 + i]) for i in range(min(int(nprior), PRIOR))]
        return c

    def root_records(self) -> np.ndarray:
        """POS_DTYPE [1 + PRIOR]: the position, then earlier positions (most recent first); the
        engine's root input together with ``len(self.prior)``."""
        out = np.zeros(1 + PRIOR, POS_DTYPE)
        out[0] = self.record()
        for i, p in enumerate(self.prior[:PRIOR]):
            out[1 + i] = p
        return out

    def move_to_action(self, move: int) -> int:
        frm, to, promo = (move >> 6) & 63, move & 63, (move >> 12) & 7
        flip = self.side == BLACK
        fr, ff = (7 - (frm >> 3) if flip else frm >> 3), frm & 7
        tr, tf = (7 - (to >> 3) if flip else to >> 3), to & 7
        dr, df = tr - fr, tf - ff
        if promo >= 2:
            plane = 64 + 3 * {4: 0, 3: 1, 2: 2}[promo] + (df + 1)
        elif (abs(dr), abs(df)) in ((2, 1), (1, 2)):
            plane = 56 + _KNIGHT.index((dr, df))
        else:
            dist = max(abs(dr), abs(df))
            plane = _QUEEN_DIRS.index((int(np.sign(dr)), int(np.sign(df)))) * 7 + dist - 1
        return (fr * 8 + ff) * 73 + plane

    def action_to_move(self, a: int) -> int:
        flip = self.side == BLACK
        s, plane = divmod(int(a), 73)
        fr, ff = s >> 3, s & 7
        promo = 0
        if plane < 56:
            dr, df = _QUEEN_DIRS[plane // 7]
            dist = plane % 7 + 1
            tr, tf = fr + dr * dist, ff + df * dist
        elif plane < 64:
            dr, df = _KNIGHT[plane - 56]
            tr, tf = fr + dr, ff + df
        else:
            kind, step = divmod(plane - 64, 3)
            tr, tf, promo = fr - 1, ff + step - 1, (4, 3, 2)[kind]
        frm = (7 - fr if flip else fr) * 8 + ff
        to = (7 - tr if flip else tr) * 8 + tf
        if not promo and (self.sq[frm] & 7) == PAWN and tr == 0:
            promo = 1
        return (promo << 12) | (frm << 6) | to


def random_position(seed: int, min_plies: int = 10, max_plies: int = 40) -> ChessPosition:
    """Seeded uniformly random legal playout of min..max plies from the start position (benchmark
    config 4's roots); stops early at a terminal position."""
    rng = np.random.default_rng(seed)
    plies = int(rng.integers(min_plies, max_plies + 1))
    p = ChessPosition()
    for _ in range(plies):
        if p.is_terminal():
            break
        ms = p.legal_moves()
        p.play(ms[int(rng.integers(len(ms)))])
    return p


def random_roots(seed: int, count: int, min_plies: int = 10, max_plies: int = 40):
    """``count`` seeded roots (root i uses seed ``seed * 1_000_003 + i``):
    (records POS_DTYPE [count, 1 + PRIOR], prior counts int32 [count])."""
    ps = [random_position(seed * 1_000_003 + i, min_plies, max_plies) for i in range(count)]
    return (np.stack([p.root_records() for p in ps]),
            np.array([min(len(p.prior), PRIOR) for p in ps], np.int32))
