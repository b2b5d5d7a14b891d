// Chess rules on the device.
//
// Rules as the reference's ChessState plays them (src/games/chess/chess_state.cpp,
// chess_rules.cpp; standard chess), including its non-FIDE behaviours: the pawn-attack test looks
// on the mirrored side (chess_rules.cpp:135-150), so kings can step next to enemy pawns and be
// captured and a side without a king is never in check; a double push always sets the en-passant
// square; the repetition key is the piece placement alone (the reference's hash is only updated
// for piece changes, chess_state.cpp:255-267); terminal order is no legal move, insufficient
// material (chess_rules.cpp:236-394), halfmove clock >= 100, third occurrence
// (chess_state.cpp:623-676).
//
// Squares are rank * 8 + file with rank 0 = the eighth rank; white pawns move towards rank 0.
// Moves use the reference encoding (promotion << 12) | (from << 6) | to; the engine's actions are
// the AlphaZero 8x8x73 = 4672 encoding in the mover's frame (ranks mirrored for black).
//
// Legal moves of a position are found by one warp: each lane generates the pseudo-legal moves of
// two squares and tests each on a private copy of the position (play, then "own king attacked?"),
// setting the move's action bit in a shared 4672-bit mask. Repetitions compare 64-bit placement
// hashes (Zobrist keys drawn from SplitMix64), as the reference compares its 64-bit Zobrist
// hashes.
#pragma once
#include "omq_internal.cuh"

namespace omq {

constexpr int kChessActions = 4672;
constexpr int kChessPlanes = 119;
constexpr int kChessPrior = 100;          // earlier game positions kept per root
constexpr int kChessMaskWords = 148;      // ceil(4672 / 32) = 146, padded
constexpr int kChessMaxChildren = 256;    // legal moves per position (218 at most)

struct __align__(8) ChessRec {
  int8_t sq[64];   // 0 empty; type 1..6 (P N B R Q K), +8 for black
  int8_t side;     // 1 white, 2 black
  int8_t castle;   // 1 white kingside, 2 white queenside, 4 black kingside, 8 black queenside
  int8_t ep;       // en-passant square or -1
  int8_t reps;     // occurrences so far, itself included
  int16_t halfmove;
  int16_t fullmove;
  int8_t c960;          // Chess960 castling (king file +- 2, rook beside the king's target)
  int8_t rook_file[4];  // original rook files: white kingside, white queenside, black k, black q
  int8_t pad[3];
};
static_assert(sizeof(ChessRec) == 80, "chess record layout");

namespace chess {
constexpr int P = 1, N = 2, B = 3, R = 4, Q = 5, K = 6;
constexpr int WHITE = 1, BLACK = 2;
__device__ __forceinline__ int color_of(int p) { return p == 0 ? 0 : ((p & 8) ? BLACK : WHITE); }
__device__ __forceinline__ int piece(int t, int c) { return t | (c == BLACK ? 8 : 0); }
__device__ __forceinline__ bool on(int r, int f) { return (unsigned)r < 8u && (unsigned)f < 8u; }
__constant__ int8_t kKnightD[8][2] = {{-2, -1}, {-2, 1}, {-1, -2}, {-1, 2}, {1, -2}, {1, 2}, {2, -1}, {2, 1}};
__constant__ int8_t kKingD[8][2] = {{-1, -1}, {-1, 0}, {-1, 1}, {0, -1}, {0, 1}, {1, -1}, {1, 0}, {1, 1}};
// queen-like directions N, NE, E, SE, S, SW, W, NW in the mover's frame (N = towards rank 0)
__constant__ int8_t kQueenD[8][2] = {{-1, 0}, {-1, 1}, {0, 1}, {1, 1}, {1, 0}, {1, -1}, {0, -1}, {-1, -1}};
}  // namespace chess

// ChessRules::isSquareAttacked with the reference's pawn direction, on the board that `at(sq)`
// reads (the position itself, or a position after a move, see ChessAfter).
template <class At>
__device__ inline bool ch_attacked_on(const At& at, int s, int by) {
  using namespace chess;
  const int r = s >> 3, f = s & 7;
  const int pr = r + (by == WHITE ? -1 : 1);
  const int8_t pawn = (int8_t)piece(P, by), knight = (int8_t)piece(N, by), king = (int8_t)piece(K, by);
  if (on(pr, f - 1) && at(pr * 8 + f - 1) == pawn) return true;
  if (on(pr, f + 1) && at(pr * 8 + f + 1) == pawn) return true;
  for (int k = 0; k < 8; ++k) {
    const int rr = r + kKnightD[k][0], ff = f + kKnightD[k][1];
    if (on(rr, ff) && at(rr * 8 + ff) == knight) return true;
  }
  for (int k = 0; k < 8; ++k) {
    const int rr = r + kKingD[k][0], ff = f + kKingD[k][1];
    if (on(rr, ff) && at(rr * 8 + ff) == king) return true;
  }
  for (int k = 0; k < 8; ++k) {
    const int dr = kKingD[k][0], df = kKingD[k][1];
    const bool diag = dr != 0 && df != 0;
    int rr = r + dr, ff = f + df;
    for (int st = 0; st < 7 && on(rr, ff); ++st, rr += dr, ff += df) {
      const int q = at(rr * 8 + ff);
      if (!q) continue;
      const int t = q & 7;
      if (color_of(q) == by && (t == Q || t == (diag ? B : R))) return true;
      break;
    }
  }
  return false;
}

struct ChessAt {
  const ChessRec& p;
  __device__ int operator()(int s) const { return p.sq[s]; }
};

__device__ inline bool ch_attacked(const ChessRec& p, int s, int by) {
  return ch_attacked_on(ChessAt{p}, s, by);
}

// The board after move m of p without copying it: the squares ch_play changes - origin emptied,
// the moving (or promoted) piece on the target, a pawn taken en passant removed, the castling
// rook moved beside the king - read through, everything else from p.
struct ChessAfter {
  const ChessRec& p;
  int from, to, pc, ep_cap, rook_from, rook_to;
  __device__ ChessAfter(const ChessRec& pos, int m) : p(pos) {
    using namespace chess;
    from = (m >> 6) & 63;
    to = m & 63;
    pc = p.sq[from];
    ep_cap = -1;
    rook_from = rook_to = -1;
    if ((pc & 7) == P && to == p.ep) ep_cap = (from >> 3) * 8 + (to & 7);
    if ((pc & 7) == K && ((from & 7) - (to & 7) == 2 || (to & 7) - (from & 7) == 2)) {
      const int r = from >> 3, me = color_of(pc);
      const bool ks = (to & 7) > (from & 7);
      rook_to = r * 8 + (p.c960 ? (ks ? (to & 7) - 1 : (to & 7) + 1) : (ks ? 5 : 3));
      rook_from = r * 8 + p.rook_file[(me == WHITE ? 0 : 2) + (ks ? 0 : 1)];
    }
  }
  __device__ int operator()(int s) const {
    // the target holds the mover's piece (a promotion changes only its type, and the mover's
    // own pieces can only block attacks on its king)
    if (s == to) return pc;
    if (s == rook_to) return p.sq[rook_from];
    if (s == from || s == rook_from || s == ep_cap) return 0;
    return p.sq[s];
  }
};

__device__ inline int ch_king(const ChessRec& p, int color) {
  const int8_t k = (int8_t)chess::piece(chess::K, color);
  for (int s = 0; s < 64; ++s)
    if (p.sq[s] == k) return s;
  return -1;
}

__device__ inline bool ch_in_check(const ChessRec& p, int color) {
  const int k = ch_king(p, color);
  return k >= 0 && ch_attacked(p, k, 3 - color);
}

// ChessState::makeMove (chess_state.cpp:1232-1346) for a move of the reference encoding; the
// repetition count is left to the caller.
__device__ inline void ch_play(ChessRec& p, int m) {
  using namespace chess;
  const int from = (m >> 6) & 63, to = m & 63, promo = (m >> 12) & 7;
  int pc = p.sq[from];
  const int captured = p.sq[to];
  const int me = color_of(pc);
  p.halfmove = ((pc & 7) == P || captured != 0) ? 0 : (int16_t)(p.halfmove + 1);
  const int old_ep = p.ep;
  p.ep = -1;
  if ((pc & 7) == P) {
    const int fr = from >> 3, tr = to >> 3;
    if (fr - tr == 2 || tr - fr == 2) p.ep = (int8_t)(((fr + tr) >> 1) * 8 + (from & 7));
    if (to == old_ep) p.sq[fr * 8 + (to & 7)] = 0;
    if (promo) pc = piece(promo == 1 ? Q : promo == 2 ? R : promo == 3 ? B : N, me);
  }
  if ((pc & 7) == K && ((from & 7) - (to & 7) == 2 || (to & 7) - (from & 7) == 2)) {
    const int r = from >> 3;
    const bool ks = (to & 7) > (from & 7);
    // chess_state.cpp:1296-1312: the rook ends beside the king's target in Chess960
    const int rook_to = p.c960 ? (ks ? (to & 7) - 1 : (to & 7) + 1) : (ks ? 5 : 3);
    const int rf = r * 8 + p.rook_file[(me == WHITE ? 0 : 2) + (ks ? 0 : 1)], rt = r * 8 + rook_to;
    const int8_t rook = p.sq[rf];
    p.sq[rf] = 0;
    p.sq[rt] = rook;
  }
  if ((pc & 7) == K) p.castle &= (int8_t)(me == WHITE ? ~3 : ~12);
  if ((pc & 7) == R && (from >> 3) == (me == WHITE ? 7 : 0)) {
    const int base = me == WHITE ? 0 : 2;
    if ((from & 7) == p.rook_file[base]) p.castle &= (int8_t)~(me == WHITE ? 1 : 4);
    else if ((from & 7) == p.rook_file[base + 1]) p.castle &= (int8_t)~(me == WHITE ? 2 : 8);
  }
  if (captured != 0 && (captured & 7) == R) {
    const int c = color_of(captured);
    if ((to >> 3) == (c == WHITE ? 7 : 0)) {
      const int base = c == WHITE ? 0 : 2;
      if ((to & 7) == p.rook_file[base]) p.castle &= (int8_t)~(c == WHITE ? 1 : 4);
      else if ((to & 7) == p.rook_file[base + 1]) p.castle &= (int8_t)~(c == WHITE ? 2 : 8);
    }
  }
  p.sq[from] = 0;
  p.sq[to] = (int8_t)pc;
  p.side = (int8_t)(3 - p.side);
  if (p.side == WHITE) p.fullmove = (int16_t)(p.fullmove + 1);
}

// ChessRules::hasInsufficientMaterial (chess_rules.cpp:236-394).
__device__ inline bool ch_insufficient(const ChessRec& p) {
  using namespace chess;
  int pieces = 0, wn = 0, bn = 0, wb = 0, bb = 0, other = 0;
  bool wl = false, wd = false, bl = false, bd = false;
  for (int s = 0; s < 64; ++s) {
    const int q = p.sq[s];
    if (!q) continue;
    ++pieces;
    const int t = q & 7;
    const bool white = color_of(q) == WHITE;
    const bool light = (((s >> 3) + (s & 7)) & 1) == 0;
    if (t == N) { if (white) ++wn; else ++bn; }
    else if (t == B) {
      if (white) { ++wb; wl |= light; wd |= !light; } else { ++bb; bl |= light; bd |= !light; }
    } else if (t != K) {
      ++other;
    }
  }
  if (pieces == 2) return true;
  if (other) return false;
  if (((wn == 1 && bn == 0) || (wn == 0 && bn == 1)) && wb == 0 && bb == 0) return true;
  if (((wb == 1 && bb == 0) || (wb == 0 && bb == 1)) && wn == 0 && bn == 0) return true;
  if (wn == 0 && bn == 0 && wb == 1 && bb == 1 && ((wl && bl) || (wd && bd))) return true;
  if (wn == 2 && bn == 0 && wb == 0 && bb == 0) return true;
  if (wn == 0 && bn == 2 && wb == 0 && bb == 0) return true;
  if (wn == 1 && bn == 1 && wb == 0 && bb == 0) return true;
  if ((wn == 1 && bb == 1 && bn == 0 && wb == 0) || (bn == 1 && wb == 1 && wn == 0 && bb == 0)) return true;
  return false;
}

// Move (reference encoding) -> engine action 0..4671 in the mover's frame.
__device__ inline int ch_action(const ChessRec& p, int m) {
  using namespace chess;
  const int from = (m >> 6) & 63, to = m & 63, promo = (m >> 12) & 7;
  const bool flip = p.side == BLACK;
  const int fr = flip ? 7 - (from >> 3) : from >> 3, ff = from & 7;
  const int tr = flip ? 7 - (to >> 3) : to >> 3, tf = to & 7;
  const int dr = tr - fr, df = tf - ff;
  const int adr = dr < 0 ? -dr : dr, adf = df < 0 ? -df : df;
  int plane;
  if (promo >= 2) {
    plane = 64 + 3 * (promo == 4 ? 0 : promo == 3 ? 1 : 2) + (df + 1);
  } else if ((adr == 2 && adf == 1) || (adr == 1 && adf == 2)) {
    plane = 56;
    for (int k = 0; k < 8; ++k)
      if (kKnightD[k][0] == dr && kKnightD[k][1] == df) plane = 56 + k;
  } else {
    const int dist = adr > adf ? adr : adf;
    const int ur = (dr > 0) - (dr < 0), uf = (df > 0) - (df < 0);
    plane = 0;
    for (int k = 0; k < 8; ++k)
      if (kQueenD[k][0] == ur && kQueenD[k][1] == uf) plane = k * 7 + dist - 1;
  }
  return (fr * 8 + ff) * 73 + plane;
}

// Engine action -> move (reference encoding) of position p.
__device__ inline int ch_move(const ChessRec& p, int a) {
  using namespace chess;
  const bool flip = p.side == BLACK;
  const int s = a / 73, plane = a - s * 73;
  const int fr = s >> 3, ff = s & 7;
  int tr, tf, promo = 0;
  if (plane < 56) {
    const int k = plane / 7, dist = plane - k * 7 + 1;
    tr = fr + kQueenD[k][0] * dist;
    tf = ff + kQueenD[k][1] * dist;
  } else if (plane < 64) {
    tr = fr + kKnightD[plane - 56][0];
    tf = ff + kKnightD[plane - 56][1];
  } else {
    const int kind = (plane - 64) / 3, step = (plane - 64) % 3 - 1;
    tr = fr - 1;
    tf = ff + step;
    promo = kind == 0 ? 4 : kind == 1 ? 3 : 2;
  }
  const int from = (flip ? 7 - fr : fr) * 8 + ff, to = (flip ? 7 - tr : tr) * 8 + tf;
  if (!promo && (p.sq[from] & 7) == P && tr == 0) promo = 1;
  return (promo << 12) | (from << 6) | (to & 63);
}

// Whether move m of p leaves the mover's king unattacked (ch_play, then ChessRules::isInCheck):
// `king` is the mover's king square before the move (-1: no king, never in check).
__device__ inline bool ch_legal_after(const ChessRec& p, int m, int king) {
  const ChessAfter after(p, m);
  const int k = (after.pc & 7) == chess::K ? after.to : king;
  return k < 0 || !ch_attacked_on(after, k, 3 - p.side);
}

// Per-warp list of pseudo-legal moves (shared memory).
constexpr int kChessMaxPseudo = 384;      // pseudo-legal moves per position (218 legal at most)
struct ChessMoveList {
  int32_t m[kChessMaxPseudo];
  int n;
  __device__ void push(int mv) {
    const int i = atomicAdd(&n, 1);
    if (i < kChessMaxPseudo) m[i] = mv;
  }
};

// Pseudo-legal moves of the piece on square s (chess_rules.cpp:476-617), each tested.
__device__ inline void ch_square_moves(const ChessRec& p, int s, ChessMoveList& mask) {
  using namespace chess;
  const int pc = p.sq[s], me = p.side;
  if (color_of(pc) != me) return;
  const int r = s >> 3, f = s & 7, t = pc & 7;
  if (t == P) {
    const int dir = me == WHITE ? -1 : 1, nr = r + dir;
    if (nr < 0 || nr > 7) return;
    if (p.sq[nr * 8 + f] == 0) {
      if (nr == 0 || nr == 7) {
        for (int k = 1; k <= 4; ++k) mask.push((k << 12) | (s << 6) | (nr * 8 + f));
      } else {
        mask.push((s << 6) | (nr * 8 + f));
      }
      if ((me == WHITE && r == 6) || (me == BLACK && r == 1)) {
        const int n2 = (nr + dir) * 8 + f;
        if (p.sq[n2] == 0) mask.push((s << 6) | n2);
      }
    }
    for (int df = -1; df <= 1; df += 2) {
      const int nf = f + df;
      if (nf < 0 || nf > 7) continue;
      const int to = nr * 8 + nf;
      if (p.sq[to] != 0 && color_of(p.sq[to]) != me) {
        if (nr == 0 || nr == 7) {
          for (int k = 1; k <= 4; ++k) mask.push((k << 12) | (s << 6) | to);
        } else {
          mask.push((s << 6) | to);
        }
      }
      if (p.ep == to) mask.push((s << 6) | to);
    }
    return;
  }
  if (t == N || t == K) {
    for (int k = 0; k < 8; ++k) {
      const int rr = r + (t == N ? kKnightD[k][0] : kKingD[k][0]);
      const int ff = f + (t == N ? kKnightD[k][1] : kKingD[k][1]);
      if (!on(rr, ff)) continue;
      const int q = p.sq[rr * 8 + ff];
      if (q == 0 || color_of(q) != me) mask.push((s << 6) | (rr * 8 + ff));
    }
    return;
  }
  for (int k = 0; k < 8; ++k) {
    const int dr = kKingD[k][0], df = kKingD[k][1];
    const bool diag = dr != 0 && df != 0;
    if ((t == B && !diag) || (t == R && diag)) continue;
    int rr = r + dr, ff = f + df;
    for (int st = 0; st < 7 && on(rr, ff); ++st, rr += dr, ff += df) {
      const int q = p.sq[rr * 8 + ff];
      if (q == 0) { mask.push((s << 6) | (rr * 8 + ff)); continue; }
      if (color_of(q) != me) mask.push((s << 6) | (rr * 8 + ff));
      break;
    }
  }
}

// Castling moves (ChessRules::addCastlingMoves / isValidCastle, chess_rules.cpp:619-733).
__device__ inline void ch_castling(const ChessRec& p, ChessMoveList& mask) {
  using namespace chess;
  const int me = p.side;
  if (ch_in_check(p, me)) return;
  const bool ks = p.castle & (me == WHITE ? 1 : 4), qs = p.castle & (me == WHITE ? 2 : 8);
  const int k = ch_king(p, me);
  if ((!ks && !qs) || k < 0) return;
  const int home = me == WHITE ? 7 : 0;
  for (int side = 0; side < 2; ++side) {
    if (side == 0 ? !ks : !qs) continue;
    const bool kingside = side == 0;
    // getCastlingSquares: king file +- 2 (e-file based in standard chess); a Chess960 king on the
    // b- or g-file would get an off-board target in the reference and castles nowhere here
    const int tfile = (p.c960 ? (k & 7) : 4) + (kingside ? 2 : -2);
    if (tfile < 0 || tfile > 7) continue;
    const int target = home * 8 + tfile;
    const int fr = k >> 3, ff = k & 7, tf = tfile;
    const int rook_file = p.rook_file[(me == WHITE ? 0 : 2) + (kingside ? 0 : 1)];
    const int rook_sq = fr * 8 + rook_file;
    if (p.sq[rook_sq] != piece(R, me)) continue;
    bool ok = true;
    const int lo = ff < rook_file ? ff : rook_file, hi = ff < rook_file ? rook_file : ff;
    for (int x = lo + 1; x < hi && ok; ++x) ok = p.sq[fr * 8 + x] == 0;
    const int step = tf > ff ? 1 : -1;
    for (int x = ff, it = 0; ok && x != tf + step && it < 8; x += step, ++it) {
      const int s = fr * 8 + x;
      if (s == k) continue;
      if (ch_attacked(p, s, 3 - me)) ok = false;
      else if (s != rook_sq && p.sq[s] != 0) ok = false;
    }
    if (ok) mask.push((k << 6) | target);
  }
}

// Legal-action mask of p (warp-collective; mask[kChessMaskWords] and the move list in shared
// memory). Pseudo-legal moves are generated per square (chess_rules.cpp:476-733) into the list,
// then each lane tests its share of the list against the board after the move. Returns the
// number of legal moves.
__device__ inline int warp_ch_legal(const ChessRec& p, uint32_t* mask, ChessMoveList& list) {
  const int lane = threadIdx.x & 31;
  for (int w = lane; w < kChessMaskWords; w += 32) mask[w] = 0;
  if (lane == 0) list.n = 0;
  __syncwarp();
  ch_square_moves(p, lane, list);
  ch_square_moves(p, lane + 32, list);
  if (lane == 0) ch_castling(p, list);
  int king = -1;
  const int8_t kp = (int8_t)chess::piece(chess::K, p.side);
  for (int s = lane; s < 64; s += 32)
    if (p.sq[s] == kp) king = king < 0 ? s : king;
  // first king in square order (ChessState's king search)
  for (int o = 16; o > 0; o >>= 1) {
    const int x = __shfl_xor_sync(0xFFFFFFFFu, king, o);
    if (x >= 0 && (king < 0 || x < king)) king = x;
  }
  __syncwarp();
  const int n = min(list.n, kChessMaxPseudo);
  for (int i = lane; i < n; i += 32) {
    const int m = list.m[i];
    if (ch_legal_after(p, m, king)) {
      const int a = ch_action(p, m);
      atomicOr(&mask[a >> 5], 1u << (a & 31));
    }
  }
  __syncwarp();
  int c = 0;
  for (int w = lane; w < kChessMaskWords; w += 32) c += __popc(mask[w]);
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
  return c;
}

// 64-bit placement hash (Zobrist keys from SplitMix64), warp-collective.
__device__ inline uint64_t warp_ch_hash(const ChessRec& p) {
  const int lane = threadIdx.x & 31;
  uint64_t h = 0;
  for (int s = lane; s < 64; s += 32)
    if (p.sq[s]) h ^= mix64(0x6A09E667F3BCC909ull + (uint64_t)(s * 16 + p.sq[s]));
  for (int o = 16; o > 0; o >>= 1) h ^= __shfl_xor_sync(0xFFFFFFFFu, h, o);
  return h;
}

// Per-warp replay state of a chess node.
struct ChessReplay {
  ChessRec pos;                 // the node's position (reps filled in)
  ChessRec ring[8];             // positions at depth j % 8 for j >= depth - 7 (history planes)
  uint64_t hash[128];           // placement hashes along the path, [0] = root
  int16_t acts[128];
  int depth;
};

__device__ __forceinline__ const ChessRec* ch_root(const EngineView& v, int r) {
  return reinterpret_cast<const ChessRec*>(v.root_board) + (size_t)r * (1 + kChessPrior);
}

// Occurrences of hash h among the first n path hashes and the root's prior positions.
__device__ inline int warp_ch_count(const EngineView& v, int r, const uint64_t* path, int n,
                                    uint64_t h) {
  const int lane = threadIdx.x & 31;
  const int nprior = v.hdr[r].root_prior;
  const uint64_t* ph = v.chess_prior_hash + (size_t)r * kChessPrior;
  int c = 0;
  for (int i = lane; i < n; i += 32) c += path[i] == h;
  for (int i = lane; i < nprior; i += 32) c += ph[i] == h;
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
  return c;
}

// Rebuild `node` of tree r by replaying its path from the root. Warp-collective; returns the
// depth or -1 on a corrupted parent chain. With `ring`, the last 8 positions are kept.
__device__ inline int warp_ch_replay(const EngineView& v, int r, int node, ChessReplay& w, bool ring) {
  const int lane = threadIdx.x & 31;
  int d = 0;
  if (lane == 0) d = path_actions(v.topo + (size_t)r * v.T, node, 127, w.acts);
  d = __shfl_sync(0xFFFFFFFFu, d, 0);
  if (d < 0) return -1;
  if (lane == 0) w.pos = *ch_root(v, r);
  __syncwarp();
  uint64_t h = warp_ch_hash(w.pos);
  if (lane == 0) w.hash[0] = h;
  if (ring && d < 8 && lane == 0) w.ring[0] = w.pos;
  __syncwarp();
  for (int j = 0; j < d; ++j) {
    if (lane == 0) ch_play(w.pos, ch_move(w.pos, w.acts[j]));
    __syncwarp();
    h = warp_ch_hash(w.pos);
    const int reps = 1 + warp_ch_count(v, r, w.hash, j + 1, h);
    if (lane == 0) {
      w.pos.reps = (int8_t)(reps < 127 ? reps : 127);
      w.hash[j + 1] = h;
      if (ring && j + 1 >= d - 7) w.ring[(j + 1) & 7] = w.pos;
    }
    __syncwarp();
  }
  w.depth = d;
  return d;
}

// Position k plies before the replayed one (k = 0..7): the ring, else the root's prior list
// (null when the game is shorter).
__device__ __forceinline__ const ChessRec* ch_hist(const EngineView& v, int r, const ChessReplay& w,
                                                   int k) {
  const int j = w.depth - k;
  if (j >= 0) return &w.ring[j & 7];
  const int i = -j;  // 1-based index into the prior list
  return i <= v.hdr[r].root_prior ? ch_root(v, r) + i : nullptr;
}

// Feature plane value at square s (in the mover's frame) of plane c (chess_rules.h layout).
__device__ inline float ch_plane(const EngineView& v, int r, const ChessReplay& w, int c, int s) {
  using namespace chess;
  const ChessRec& cur = w.pos;
  const int me = cur.side;
  if (c < 112) {
    const ChessRec* h = ch_hist(v, r, w, c / 14);
    if (!h) return 0.0f;
    const int j = c % 14;
    if (j == 12) return h->reps >= 2 ? 1.0f : 0.0f;
    if (j == 13) return h->reps >= 3 ? 1.0f : 0.0f;
    const int bs = me == BLACK ? (7 - (s >> 3)) * 8 + (s & 7) : s;  // frame square -> board square
    const int q = h->sq[bs];
    if (!q) return 0.0f;
    return (((color_of(q) == me) ? 0 : 6) + (q & 7) - 1) == j ? 1.0f : 0.0f;
  }
  switch (c) {
    case 112: return me == WHITE ? 1.0f : 0.0f;
    case 113: return __fdiv_rn((float)cur.fullmove, 100.0f);
    case 114: return (cur.castle & (me == WHITE ? 1 : 4)) ? 1.0f : 0.0f;
    case 115: return (cur.castle & (me == WHITE ? 2 : 8)) ? 1.0f : 0.0f;
    case 116: return (cur.castle & (me == WHITE ? 4 : 1)) ? 1.0f : 0.0f;
    case 117: return (cur.castle & (me == WHITE ? 8 : 2)) ? 1.0f : 0.0f;
    default: return __fdiv_rn((float)cur.halfmove, 100.0f);
  }
}

// Terminal test of the replayed position given its legal-move count (ChessState::isTerminal order).
__device__ inline bool ch_terminal(const ChessRec& p, int legal) {
  return legal == 0 || ch_insufficient(p) || p.halfmove >= 100 || p.reps >= 3;
}

}  // namespace omq
