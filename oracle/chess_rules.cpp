// Parity oracle (TEST INFRASTRUCTURE ONLY). Chess rules restated from the reference engine; the
// behaviours kept from it are listed in chess_rules.h.
#include "chess_rules.h"

#include <cstdlib>
#include <cstring>

namespace {

constexpr int kPawn = 1, kKnight = 2, kBishop = 3, kRook = 4, kQueen = 5, kKing = 6;
constexpr int kWhite = 1, kBlack = 2;

inline int rank_of(int s) { return s >> 3; }
inline int file_of(int s) { return s & 7; }
inline int type_of(int8_t p) { return p & 7; }
inline int color_of(int8_t p) { return p == 0 ? 0 : ((p & 8) ? kBlack : kWhite); }
inline int8_t make_piece(int type, int color) { return (int8_t)(type | (color == kBlack ? 8 : 0)); }
inline bool on_board(int r, int f) { return r >= 0 && r < 8 && f >= 0 && f < 8; }

const int kKnightD[8][2] = {{-2, -1}, {-2, 1}, {-1, -2}, {-1, 2}, {1, -2}, {1, 2}, {2, -1}, {2, 1}};
const int kKingD[8][2] = {{-1, -1}, {-1, 0}, {-1, 1}, {0, -1}, {0, 1}, {1, -1}, {1, 0}, {1, 1}};
const int kDiag[4][2] = {{-1, -1}, {-1, 1}, {1, -1}, {1, 1}};
const int kOrtho[4][2] = {{-1, 0}, {1, 0}, {0, -1}, {0, 1}};

// ChessRules::isSquareAttacked, pawn direction as the reference evaluates it.
bool attacked(const oracle_chess_pos& p, int s, int by) {
  const int r = rank_of(s), f = file_of(s);
  const int pr = r + (by == kWhite ? -1 : 1);
  for (int df = -1; df <= 1; df += 2)
    if (on_board(pr, f + df) && p.sq[pr * 8 + f + df] == make_piece(kPawn, by)) return true;
  for (auto& d : kKnightD)
    if (on_board(r + d[0], f + d[1]) && p.sq[(r + d[0]) * 8 + f + d[1]] == make_piece(kKnight, by))
      return true;
  for (auto& d : kKingD)
    if (on_board(r + d[0], f + d[1]) && p.sq[(r + d[0]) * 8 + f + d[1]] == make_piece(kKing, by))
      return true;
  for (int pass = 0; pass < 2; ++pass) {
    const int(*dirs)[2] = pass == 0 ? kDiag : kOrtho;
    const int slider = pass == 0 ? kBishop : kRook;
    for (int k = 0; k < 4; ++k)
      for (int st = 1;; ++st) {
        const int rr = r + dirs[k][0] * st, ff = f + dirs[k][1] * st;
        if (!on_board(rr, ff)) break;
        const int8_t q = p.sq[rr * 8 + ff];
        if (q) {
          if (color_of(q) == by && (type_of(q) == slider || type_of(q) == kQueen)) return true;
          break;
        }
      }
  }
  return false;
}

int king_square(const oracle_chess_pos& p, int color) {
  for (int s = 0; s < 64; ++s)
    if (p.sq[s] == make_piece(kKing, color)) return s;
  return -1;
}

bool in_check(const oracle_chess_pos& p, int color) {
  const int k = king_square(p, color);
  return k >= 0 && attacked(p, k, 3 - color);
}

inline int32_t mv(int from, int to, int promo = 0) { return (promo << 12) | (from << 6) | to; }

int pseudo_moves(const oracle_chess_pos& p, int32_t* out) {
  const int me = p.side;
  int n = 0;
  auto add_promos = [&](int from, int to) {
    for (int pc = 1; pc <= 4; ++pc) out[n++] = mv(from, to, pc);
  };
  for (int s = 0; s < 64; ++s) {
    const int8_t pc = p.sq[s];
    if (color_of(pc) != me) continue;
    const int r = rank_of(s), f = file_of(s), t = type_of(pc);
    if (t == kPawn) {
      const int dir = me == kWhite ? -1 : 1, nr = r + dir;
      if (nr >= 0 && nr < 8) {
        if (p.sq[nr * 8 + f] == 0) {
          if (nr == 0 || nr == 7) add_promos(s, nr * 8 + f);
          else out[n++] = mv(s, nr * 8 + f);
          if ((me == kWhite && r == 6) || (me == kBlack && r == 1)) {
            const int n2 = (nr + dir) * 8 + f;
            if (p.sq[n2] == 0) out[n++] = mv(s, n2);
          }
        }
        for (int df = -1; df <= 1; df += 2) {
          const int nf = f + df;
          if (nf < 0 || nf >= 8) continue;
          const int to = nr * 8 + nf;
          if (p.sq[to] != 0 && color_of(p.sq[to]) != me) {
            if (nr == 0 || nr == 7) add_promos(s, to);
            else out[n++] = mv(s, to);
          }
          if (p.ep == to) out[n++] = mv(s, to);
        }
      }
    } else if (t == kKnight || t == kKing) {
      const int(*d)[2] = t == kKnight ? kKnightD : kKingD;
      for (int k = 0; k < 8; ++k) {
        const int rr = r + d[k][0], ff = f + d[k][1];
        if (!on_board(rr, ff)) continue;
        const int8_t q = p.sq[rr * 8 + ff];
        if (q == 0 || color_of(q) != me) out[n++] = mv(s, rr * 8 + ff);
      }
    } else {
      for (int pass = 0; pass < 2; ++pass) {
        if (pass == 0 && t == kRook) continue;
        if (pass == 1 && t == kBishop) continue;
        const int(*dirs)[2] = pass == 0 ? kDiag : kOrtho;
        for (int k = 0; k < 4; ++k)
          for (int st = 1;; ++st) {
            const int rr = r + dirs[k][0] * st, ff = f + dirs[k][1] * st;
            if (!on_board(rr, ff)) break;
            const int8_t q = p.sq[rr * 8 + ff];
            if (q == 0) { out[n++] = mv(s, rr * 8 + ff); continue; }
            if (color_of(q) != me) out[n++] = mv(s, rr * 8 + ff);
            break;
          }
      }
    }
  }
  // castling (ChessRules::addCastlingMoves / isValidCastle, chess_rules.cpp:619-733)
  if (!in_check(p, me)) {
    const bool ks = p.castle & (me == kWhite ? 1 : 4), qs = p.castle & (me == kWhite ? 2 : 8);
    const int k = king_square(p, me);
    if ((ks || qs) && k >= 0) {
      const int home = me == kWhite ? 7 : 0;
      for (int side = 0; side < 2; ++side) {
        if (side == 0 ? !ks : !qs) continue;
        const bool kingside = side == 0;
        const int kf = p.c960 ? file_of(k) : 4;  // getCastlingSquares
        const int tfile = kf + (kingside ? 2 : -2);
        if (tfile < 0 || tfile > 7) continue;     // off-board target in the reference
        const int target = home * 8 + tfile;
        const int fr = rank_of(k), ff = file_of(k), tf = tfile;
        const int rook_file = p.rook_file[(me == kWhite ? 0 : 2) + (kingside ? 0 : 1)];
        const int rook_sq = fr * 8 + rook_file;
        if (p.sq[rook_sq] != make_piece(kRook, me)) continue;
        bool ok = true;
        const int lo = ff < rook_file ? ff : rook_file, hi = ff < rook_file ? rook_file : ff;
        for (int x = lo + 1; x < hi && ok; ++x) ok = p.sq[fr * 8 + x] == 0;
        const int step = tf > ff ? 1 : -1;
        for (int x = ff; ok && x != tf + step; x += step) {
          const int s = fr * 8 + x;
          if (s == k) continue;
          if (attacked(p, s, 3 - me)) ok = false;
          else if (s != rook_sq && p.sq[s] != 0) ok = false;
        }
        if (ok) out[n++] = mv(k, target);
      }
    }
  }
  return n;
}

bool insufficient(const oracle_chess_pos& p) {
  int pieces = 0, cnt[3][7] = {{0}};
  bool light[3] = {false, false, false}, dark[3] = {false, false, false};
  for (int s = 0; s < 64; ++s) {
    const int8_t q = p.sq[s];
    if (!q) continue;
    ++pieces;
    const int c = color_of(q), t = type_of(q);
    ++cnt[c][t];
    if (t == kBishop) ((rank_of(s) + file_of(s)) % 2 == 0 ? light : dark)[c] = true;
  }
  const int W = kWhite, B = kBlack;
  const bool no_pawns = cnt[W][kPawn] == 0 && cnt[B][kPawn] == 0;
  const bool no_heavy = cnt[W][kRook] == 0 && cnt[B][kRook] == 0 && cnt[W][kQueen] == 0 &&
                        cnt[B][kQueen] == 0;
  const int wn = cnt[W][kKnight], bn = cnt[B][kKnight], wb = cnt[W][kBishop], bb = cnt[B][kBishop];
  if (pieces == 2) return true;
  if (!no_pawns || !no_heavy) return false;
  if (((wn == 1 && bn == 0) || (wn == 0 && bn == 1)) && wb == 0 && bb == 0) return true;
  if (((wb == 1 && bb == 0) || (wb == 0 && bb == 1)) && wn == 0 && bn == 0) return true;
  if (wn == 0 && bn == 0 && wb == 1 && bb == 1 && ((light[W] && light[B]) || (dark[W] && dark[B])))
    return true;
  if (wn == 2 && bn == 0 && wb == 0 && bb == 0) return true;
  if (wn == 0 && bn == 2 && wb == 0 && bb == 0) return true;
  if (wn == 1 && bn == 1 && wb == 0 && bb == 0) return true;
  if ((wn == 1 && bb == 1 && bn == 0 && wb == 0) || (bn == 1 && wb == 1 && wn == 0 && bb == 0))
    return true;
  return false;
}

const int kQueenD[8][2] = {{-1, 0}, {-1, 1}, {0, 1}, {1, 1}, {1, 0}, {1, -1}, {0, -1}, {-1, -1}};

}  // namespace

extern "C" {

static int parse_fen(const char* fen, oracle_chess_pos* out, int c960) {
  oracle_chess_pos p;
  std::memset(&p, 0, sizeof(p));
  p.ep = -1;
  p.c960 = (int8_t)c960;
  p.rook_file[0] = 7; p.rook_file[1] = 0; p.rook_file[2] = 7; p.rook_file[3] = 0;
  const char* c = fen;
  int s = 0;
  for (; *c && *c != ' '; ++c) {
    if (*c == '/') continue;
    if (*c >= '1' && *c <= '8') { s += *c - '0'; continue; }
    const char* kinds = "pnbrqk";
    const char lower = (char)(*c | 0x20);
    const char* k = std::strchr(kinds, lower);
    if (!k || s >= 64) return 1;
    p.sq[s++] = make_piece((int)(k - kinds) + 1, (*c == lower) ? kBlack : kWhite);
  }
  if (s != 64 || *c != ' ') return 1;
  ++c;
  p.side = *c == 'b' ? kBlack : kWhite;
  c += 2;
  for (; *c && *c != ' '; ++c) {
    if (*c == 'K') p.castle |= 1;
    else if (*c == 'Q') p.castle |= 2;
    else if (*c == 'k') p.castle |= 4;
    else if (*c == 'q') p.castle |= 8;
    else if ((*c >= 'A' && *c <= 'H') || (*c >= 'a' && *c <= 'h')) {
      // a rook file (ChessState::setFromFEN, chess_state.cpp:460-487): king side if right of the king
      const bool white = *c <= 'H';
      const int f = white ? *c - 'A' : *c - 'a';
      const int ksq = king_square(p, white ? kWhite : kBlack);
      const bool kside = ksq >= 0 && f > file_of(ksq);
      p.castle |= (int8_t)(white ? (kside ? 1 : 2) : (kside ? 4 : 8));
      p.rook_file[(white ? 0 : 2) + (kside ? 0 : 1)] = (int8_t)f;
    }
  }
  if (*c) ++c;
  if (*c && *c != '-') {
    p.ep = (int8_t)((8 - (c[1] - '0')) * 8 + (c[0] - 'a'));
    c += 2;
  } else if (*c) {
    ++c;
  }
  int hm = 0, fm = 1;
  if (*c) hm = (int)std::strtol(c, const_cast<char**>(&c), 10);
  if (*c) fm = (int)std::strtol(c, const_cast<char**>(&c), 10);
  p.halfmove = (int16_t)hm;
  p.fullmove = (int16_t)fm;
  p.reps = 1;
  *out = p;
  return 0;
}

int oracle_chess_from_fen(const char* fen, oracle_chess_pos* out) { return parse_fen(fen, out, 0); }
int oracle_chess_from_fen960(const char* fen, oracle_chess_pos* out) { return parse_fen(fen, out, 1); }

void oracle_chess_play(oracle_chess_pos* pp, int32_t m) {
  oracle_chess_pos& p = *pp;
  const int from = (m >> 6) & 63, to = m & 63, promo = (m >> 12) & 7;
  int8_t piece = p.sq[from];
  const int8_t captured = p.sq[to];
  const int me = color_of(piece);
  if (type_of(piece) == kPawn || captured != 0) p.halfmove = 0;
  else p.halfmove = (int16_t)(p.halfmove + 1);
  const int old_ep = p.ep;
  p.ep = -1;
  if (type_of(piece) == kPawn) {
    const int fr = rank_of(from), tr = rank_of(to);
    if (std::abs(fr - tr) == 2) p.ep = (int8_t)(((fr + tr) / 2) * 8 + file_of(from));
    if (to == old_ep) p.sq[fr * 8 + file_of(to)] = 0;
    if (promo) {
      const int t = promo == 1 ? kQueen : promo == 2 ? kRook : promo == 3 ? kBishop : kKnight;
      piece = make_piece(t, me);
    }
  }
  if (type_of(piece) == kKing && std::abs(file_of(from) - file_of(to)) == 2) {
    const int r = rank_of(from);
    const bool kingside = file_of(to) > file_of(from);
    const int rook_file = p.rook_file[(me == kWhite ? 0 : 2) + (kingside ? 0 : 1)];
    const int rook_to = p.c960 ? (kingside ? file_of(to) - 1 : file_of(to) + 1) : (kingside ? 5 : 3);
    const int rf = r * 8 + rook_file, rt = r * 8 + rook_to;
    const int8_t rook = p.sq[rf];
    p.sq[rf] = 0;
    p.sq[rt] = rook;
  }
  // ChessRules::getUpdatedCastlingRights (chess_rules.cpp:400-474)
  if (type_of(piece) == kKing) p.castle &= (int8_t)(me == kWhite ? ~3 : ~12);
  if (type_of(piece) == kRook) {
    const int home = me == kWhite ? 7 : 0, base = me == kWhite ? 0 : 2;
    if (rank_of(from) == home) {
      if (file_of(from) == p.rook_file[base]) p.castle &= (int8_t)~(me == kWhite ? 1 : 4);
      else if (file_of(from) == p.rook_file[base + 1]) p.castle &= (int8_t)~(me == kWhite ? 2 : 8);
    }
  }
  if (captured != 0 && type_of(captured) == kRook) {
    const int c = color_of(captured), home = c == kWhite ? 7 : 0, base = c == kWhite ? 0 : 2;
    if (rank_of(to) == home) {
      if (file_of(to) == p.rook_file[base]) p.castle &= (int8_t)~(c == kWhite ? 1 : 4);
      else if (file_of(to) == p.rook_file[base + 1]) p.castle &= (int8_t)~(c == kWhite ? 2 : 8);
    }
  }
  p.sq[from] = 0;
  p.sq[to] = piece;
  p.side = (int8_t)(3 - p.side);
  if (p.side == kWhite) p.fullmove = (int16_t)(p.fullmove + 1);
  p.reps = 1;
}

int oracle_chess_legal(const oracle_chess_pos* p, int32_t* moves) {
  int32_t pseudo[320];
  const int n = pseudo_moves(*p, pseudo);
  int k = 0;
  for (int i = 0; i < n; ++i) {
    oracle_chess_pos q = *p;
    oracle_chess_play(&q, pseudo[i]);
    if (!in_check(q, p->side)) moves[k++] = pseudo[i];
  }
  return k;
}

int oracle_chess_terminal(const oracle_chess_pos* p, int reps, int* result) {
  int32_t m[320];
  int r = 0;
  if (oracle_chess_legal(p, m) == 0)
    r = in_check(*p, p->side) ? (p->side == kWhite ? 2 : 1) : 3;
  else if (insufficient(*p) || p->halfmove >= 100 || reps >= 3)
    r = 3;
  if (result) *result = r;
  return r != 0;
}

int oracle_chess_same(const oracle_chess_pos* a, const oracle_chess_pos* b) {
  return std::memcmp(a->sq, b->sq, 64) == 0;
}

int oracle_chess_action(const oracle_chess_pos* p, int32_t m) {
  const int from = (m >> 6) & 63, to = m & 63, promo = (m >> 12) & 7;
  const bool flip = p->side == kBlack;
  const int fr = flip ? 7 - rank_of(from) : rank_of(from), ff = file_of(from);
  const int tr = flip ? 7 - rank_of(to) : rank_of(to), tf = file_of(to);
  const int dr = tr - fr, df = tf - ff;
  int plane = -1;
  if (promo >= 2) {
    const int kind = promo == 4 ? 0 : promo == 3 ? 1 : 2;  // knight, bishop, rook
    plane = 64 + 3 * kind + (df + 1);
  } else if ((std::abs(dr) == 2 && std::abs(df) == 1) || (std::abs(dr) == 1 && std::abs(df) == 2)) {
    for (int k = 0; k < 8; ++k)
      if (kKnightD[k][0] == dr && kKnightD[k][1] == df) plane = 56 + k;
  } else {
    const int dist = std::abs(dr) > std::abs(df) ? std::abs(dr) : std::abs(df);
    const int ur = dr == 0 ? 0 : dr / std::abs(dr), uf = df == 0 ? 0 : df / std::abs(df);
    for (int k = 0; k < 8; ++k)
      if (kQueenD[k][0] == ur && kQueenD[k][1] == uf) plane = k * 7 + (dist - 1);
  }
  return (fr * 8 + ff) * 73 + plane;
}

int32_t oracle_chess_move(const oracle_chess_pos* p, int a) {
  const bool flip = p->side == kBlack;
  const int sq = a / 73, plane = a % 73;
  const int fr = sq >> 3, ff = sq & 7;
  int tr, tf, promo = 0;
  if (plane < 56) {
    const int k = plane / 7, dist = plane % 7 + 1;
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
  if (!promo && type_of(p->sq[from]) == kPawn && (tr == 0)) promo = 1;  // queen promotion
  return mv(from, to, promo);
}

void oracle_chess_features(const oracle_chess_pos* const* hist, float* out) {
  std::memset(out, 0, sizeof(float) * 119 * 64);
  const oracle_chess_pos& cur = *hist[0];
  const int me = cur.side;
  const bool flip = me == kBlack;
  for (int k = 0; k < 8; ++k) {
    const oracle_chess_pos* h = hist[k];
    if (!h) continue;
    float* o = out + (size_t)14 * k * 64;
    for (int s = 0; s < 64; ++s) {
      const int8_t q = h->sq[s];
      if (!q) continue;
      const int fs = flip ? (7 - rank_of(s)) * 8 + file_of(s) : s;
      const int plane = (color_of(q) == me ? 0 : 6) + type_of(q) - 1;
      o[plane * 64 + fs] = 1.0f;
    }
    for (int s = 0; s < 64; ++s) {
      o[12 * 64 + s] = h->reps >= 2 ? 1.0f : 0.0f;
      o[13 * 64 + s] = h->reps >= 3 ? 1.0f : 0.0f;
    }
  }
  const int own_k = me == kWhite ? 1 : 4, own_q = me == kWhite ? 2 : 8;
  const int opp_k = me == kWhite ? 4 : 1, opp_q = me == kWhite ? 8 : 2;
  const float c[7] = {me == kWhite ? 1.0f : 0.0f, (float)cur.fullmove / 100.0f,
                      (cur.castle & own_k) ? 1.0f : 0.0f, (cur.castle & own_q) ? 1.0f : 0.0f,
                      (cur.castle & opp_k) ? 1.0f : 0.0f, (cur.castle & opp_q) ? 1.0f : 0.0f,
                      (float)cur.halfmove / 100.0f};
  for (int j = 0; j < 7; ++j)
    for (int s = 0; s < 64; ++s) out[(112 + j) * 64 + s] = c[j];
}

}  // extern "C"
