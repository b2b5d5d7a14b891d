// Go rules on the device, one warp per position in shared memory.
//
// Rules as the reference's C++ engine plays them with Chinese rules and superko off
// (src/games/go/go_state.cpp:227-420, go_rules.cpp:34-110): a stone may not be placed on an
// occupied point or on the ko point; opponent groups left without liberties are captured; a move
// that captures nothing and leaves its own group without liberties is suicide and illegal; a move
// capturing exactly one stone (one group of one stone) makes that point the ko point; pass is
// always legal, clears the ko point, and two consecutive passes end the game.
//
// Groups are labelled by a lock-free union-find over the warp (links always go from the larger
// root index to the smaller, so the forest stays acyclic under concurrent CAS), then every empty
// point adds one liberty to each distinct adjacent group. With exact liberty counts, a move at an
// empty point p is legal iff p is not the ko point and p has an empty neighbour, or an own
// neighbour group with two or more liberties (p is one of them), or an opponent neighbour group
// whose only liberty is p.
#pragma once
#include "omq_internal.cuh"

namespace omq {

constexpr int kGoPlanes = 17;
constexpr int kGoHistory = 8;
constexpr int kGoMaskWords = 12;  // ceil(362 / 32): legal bits, pass at bit `cells`

struct GoScratch {
  int par[kMaxCells + 1];   // union-find parent; after analysis the group root of each stone
  int libs[kMaxCells + 1];  // distinct liberties, indexed by group root
  unsigned long long gkey[kMaxCells + 1];  // superko: XOR of the group's stone keys, by root
};

// Superko position keys (64-bit Zobrist): stone keys mix64(0x6A09E667F3BCC909 ^ (cell*4 + colour))
// and ko-point keys mix64(0xBB67AE8584CAA73B ^ cell).
__device__ __forceinline__ uint64_t go_stone_key(int c, int colour) {
  return mix64(0x6A09E667F3BCC909ull ^ (uint64_t)(c * 4 + colour));
}
__device__ __forceinline__ uint64_t go_ko_key(int c) { return mix64(0xBB67AE8584CAA73Bull ^ (uint64_t)c); }
// Side-to-move key of the repetition rule's keys (Japanese / Korean).
__device__ __forceinline__ uint64_t go_side_key(int p) { return mix64(0x3C6EF372FE94F82Bull ^ (uint64_t)p); }

// Key of the stones of board b (without a ko point). Warp-collective.
__device__ inline uint64_t warp_go_board_key(const int8_t* b, int C) {
  const int lane = threadIdx.x & 31;
  uint64_t k = 0;
  for (int c = lane; c < C; c += 32)
    if (b[c]) k ^= go_stone_key(c, b[c]);
  for (int o = 16; o > 0; o >>= 1) k ^= __shfl_xor_sync(0xFFFFFFFFu, k, o);
  return k;
}

__device__ __forceinline__ int go_find(volatile int* par, int x) {
  for (int it = 0; it < kMaxCells && par[x] != x; ++it) x = par[x];
  return x;
}

__device__ __forceinline__ void go_unite(int* par, int a, int b) {
  volatile int* vp = par;
  for (int it = 0; it < 4 * kMaxCells; ++it) {
    a = go_find(vp, a);
    b = go_find(vp, b);
    if (a == b) return;
    if (a < b) { const int t = a; a = b; b = t; }
    if (atomicCAS(&par[a], a, b) == a) return;
  }
}

// Neighbours of cell c on an S x S board (-1 off the board): up, down, left, right.
__device__ __forceinline__ void go_neighbours(int c, int S, int nb[4]) {
  const int y = c / S, x = c - y * S;
  nb[0] = y > 0 ? c - S : -1;
  nb[1] = y < S - 1 ? c + S : -1;
  nb[2] = x > 0 ? c - 1 : -1;
  nb[3] = x < S - 1 ? c + 1 : -1;
}

// Label the groups of board b and count their liberties. Warp-collective; on return par[c] is
// the root of the group holding c (for stones) and libs[root] its liberty count.
__device__ inline void warp_go_analyze(const int8_t* b, int S, GoScratch& g, bool keys = false) {
  const int lane = threadIdx.x & 31, C = S * S;
  for (int c = lane; c < C; c += 32) { g.par[c] = c; g.libs[c] = 0; if (keys) g.gkey[c] = 0ull; }
  __syncwarp();
  for (int c = lane; c < C; c += 32) {
    const int8_t s = b[c];
    if (!s) continue;
    const int x = c % S;
    if (x < S - 1 && b[c + 1] == s) go_unite(g.par, c, c + 1);
    if (c + S < C && b[c + S] == s) go_unite(g.par, c, c + S);
  }
  __syncwarp();
  for (int c = lane; c < C; c += 32)
    if (b[c]) g.par[c] = go_find(g.par, c);
  __syncwarp();
  if (keys)
    for (int c = lane; c < C; c += 32)
      if (b[c]) atomicXor(&g.gkey[g.par[c]], (unsigned long long)go_stone_key(c, b[c]));
  for (int c = lane; c < C; c += 32) {
    if (b[c]) continue;
    int nb[4];
    go_neighbours(c, S, nb);
    int seen[4];
    int ns = 0;
    for (int k = 0; k < 4; ++k) {
      if (nb[k] < 0 || !b[nb[k]]) continue;
      const int r = g.par[nb[k]];
      bool dup = false;
      for (int j = 0; j < ns; ++j) dup |= seen[j] == r;
      if (!dup) { seen[ns++] = r; atomicAdd(&g.libs[r], 1); }
    }
  }
  __syncwarp();
}

// Legal move bits of `player` after warp_go_analyze(b): mask[w] bit i = action 32 w + i, pass
// (action C) always set. Returns the number of legal actions. Warp-collective.
__device__ inline int warp_go_legal(const int8_t* b, int S, int player, int ko, const GoScratch& g,
                             uint32_t* mask) {
  const int lane = threadIdx.x & 31, C = S * S;
  int total = 0;
  for (int w = 0; w * 32 <= C; ++w) {
    const int c = w * 32 + lane;
    bool legal = false;
    if (c < C) {
      if (b[c] == 0 && c != ko) {
        int nb[4];
        go_neighbours(c, S, nb);
        for (int k = 0; k < 4 && !legal; ++k) {
          const int q = nb[k];
          if (q < 0) continue;
          if (b[q] == 0) legal = true;
          else if (b[q] == player) legal = g.libs[g.par[q]] >= 2;
          else legal = g.libs[g.par[q]] == 1;
        }
      }
    } else if (c == C) {
      legal = true;  // pass
    }
    const uint32_t m = __ballot_sync(0xFFFFFFFFu, legal);
    if (lane == 0) mask[w] = m;
    total += __popc(m);
  }
  __syncwarp();
  return total;
}

// Play action a (C = pass) for `player` on board b, which must be legal. ko and passes are the
// position's state and are updated. Warp-collective; all lanes see the same ko/passes on return.
__device__ inline void warp_go_play(int8_t* b, int S, int player, int a, GoScratch& g, int& ko,
                             int& passes) {
  const int lane = threadIdx.x & 31, C = S * S;
  if (a >= C) { ko = -1; ++passes; return; }
  warp_go_analyze(b, S, g);
  const int opp = 3 - player;
  int nb[4];
  go_neighbours(a, S, nb);
  int cap[4];
  int ncap = 0;
  for (int k = 0; k < 4; ++k) {  // every lane computes the same (small) set
    const int q = nb[k];
    if (q < 0 || b[q] != opp) continue;
    const int r = g.par[q];
    if (g.libs[r] != 1) continue;
    bool dup = false;
    for (int j = 0; j < ncap; ++j) dup |= cap[j] == r;
    if (!dup) cap[ncap++] = r;
  }
  __syncwarp();
  int removed = 0;
  if (ncap > 0) {
    for (int c = lane; c < C; c += 32) {
      if (b[c] != opp) continue;
      const int r = g.par[c];
      bool hit = false;
      for (int j = 0; j < ncap; ++j) hit |= cap[j] == r;
      if (hit) { b[c] = 0; ++removed; }
    }
    for (int o = 16; o > 0; o >>= 1) removed += __shfl_xor_sync(0xFFFFFFFFu, removed, o);
  }
  __syncwarp();
  if (lane == 0) b[a] = (int8_t)player;
  __syncwarp();
  // a group of one stone is its own root, so the captured point is cap[0]
  ko = (ncap == 1 && removed == 1) ? cap[0] : -1;
  passes = 0;
}

// Position of a Go tree node rebuilt from the root by replaying the moves on its path.
struct GoPos {
  int16_t acts[128];
  int8_t board[kMaxCells + 3];
  GoScratch g;
  uint64_t pkeys[128];  // superko: keys of the path's positions reached by non-pass moves
  int ko, passes, player, depth, npk;
};

// Root history of tree r: kGoHistory boards, [0] = the root position.
__device__ __forceinline__ const int8_t* go_root_hist(const EngineView& v, int r, int k) {
  return v.root_board + ((size_t)r * kGoHistory + k) * v.C;
}

// Rebuild `node` of tree r into pos (board after its move, side to move, ko, passes). When ring
// is not null, ring[j % 8] receives the board at every depth j >= depth - 7 (the history planes).
// Returns the depth, or -1 on a corrupted parent chain. Warp-collective.
__device__ inline int warp_go_replay(const EngineView& v, int r, int node, GoPos& pos, int8_t* ring,
                                     bool keys = false) {
  const int lane = threadIdx.x & 31;
  int d = 0;
  if (lane == 0) d = path_actions(v.topo + (size_t)r * v.T, node, 127, pos.acts);
  d = __shfl_sync(0xFFFFFFFFu, d, 0);
  if (d < 0) return -1;
  const TreeHeader& H = v.hdr[r];
  const int8_t* root = go_root_hist(v, r, 0);
  for (int c = lane; c < v.C; c += 32) pos.board[c] = root[c];
  __syncwarp();
  if (ring && d < kGoHistory)
    for (int c = lane; c < v.C; c += 32) ring[c] = root[c];
  int ko = H.root_ko, passes = H.root_passes, player = H.root_player;
  int npk = 0;
  for (int j = 0; j < d; ++j) {
    warp_go_play(pos.board, v.S, player, pos.acts[j], pos.g, ko, passes);
    player = 3 - player;
    // superko: positions after non-pass moves; repetition rule: after every move, side included
    if (keys && (v.go_cycle || pos.acts[j] < v.C)) {
      uint64_t k = warp_go_board_key(pos.board, v.C) ^ (ko >= 0 ? go_ko_key(ko) : 0ull);
      if (v.go_cycle) k ^= go_side_key(player);
      if ((threadIdx.x & 31) == 0) pos.pkeys[npk] = k;
      ++npk;
    }
    if (ring && j + 1 >= d - (kGoHistory - 1)) {
      int8_t* dst = ring + (size_t)((j + 1) % kGoHistory) * v.C;
      for (int c = lane; c < v.C; c += 32) dst[c] = pos.board[c];
    }
  }
  __syncwarp();
  pos.ko = ko;
  pos.passes = passes;
  pos.player = player;
  pos.depth = d;
  pos.npk = npk;
  return d;
}

// Key of the position that candidate c (C = pass) makes: board after captures, new ko point.
// Needs warp_go_analyze(..., keys = true). Per lane.
__device__ inline uint64_t go_child_key(const GoPos& pos, int S, uint64_t bkey, int c) {
  const int C = S * S;
  if (c >= C) return bkey;  // pass: same stones, no ko point
  const int8_t* b = pos.board;
  const GoScratch& g = pos.g;
  const int me = pos.player, opp = 3 - me;
  int nb[4];
  go_neighbours(c, S, nb);
  int cap[4];
  int ncap = 0;
  uint64_t k = bkey ^ go_stone_key(c, me);
  for (int q = 0; q < 4; ++q) {
    const int s = nb[q];
    if (s < 0 || b[s] != opp) continue;
    const int root = g.par[s];
    if (g.libs[root] != 1) continue;
    bool dup = false;
    for (int j = 0; j < ncap; ++j) dup |= cap[j] == root;
    if (!dup) { cap[ncap++] = root; k ^= g.gkey[root]; }
  }
  if (ncap == 1) {
    int snb[4];
    go_neighbours(cap[0], S, snb);
    bool single = true;
    for (int q = 0; q < 4; ++q) single &= snb[q] < 0 || b[snb[q]] != opp;
    if (single) k ^= go_ko_key(cap[0]);
  }
  return k;
}

// Japanese / Korean repetition rule: tmask bit of a legal child is set when its position
// (board, ko point, side to move) already occurred twice - in the root's game (sorted keys with
// repeats) plus on the path - so that reaching it ends the game. Warp-collective.
__device__ inline void warp_go_cycle(const EngineView& v, int r, const GoPos& pos, const uint32_t* mask,
                                     uint32_t* tmask) {
  const int lane = threadIdx.x & 31, C = v.C;
  const uint64_t bkey = warp_go_board_key(pos.board, C);
  const int nroot = v.hdr[r].root_nkeys;
  const uint64_t* rk = v.go_keys + (size_t)r * OMQ_GO_MAX_KEYS;
  const uint64_t side = go_side_key(3 - pos.player);
  for (int w = 0; w * 32 <= C; ++w) {
    const int c = w * 32 + lane;
    bool term = false;
    if ((mask[w] >> lane) & 1u) {
      const uint64_t k = go_child_key(pos, v.S, bkey, c) ^ side;
      int count = 0;
      for (int i = 0; i < pos.npk; ++i) count += pos.pkeys[i] == k;
      int lo = 0, hi = nroot;  // first root key >= k
      for (int it = 0; it < 16 && lo < hi; ++it) {
        const int mid = (lo + hi) >> 1;
        if (rk[mid] < k) lo = mid + 1; else hi = mid;
      }
      for (int i = lo; i < nroot && rk[i] == k && count < 2; ++i) ++count;
      term = count >= 2;
    }
    const uint32_t tm = __ballot_sync(0xFFFFFFFFu, term);
    if (lane == 0) tmask[w] = tm;
  }
  __syncwarp();
}

// Positional superko (GoState::isLegalMove with enforce_superko, go_state.cpp:359-418): clears
// the legal bits of moves whose resulting position (board after captures + new ko point) has the
// key of a position of the root's game (sorted keys + 4096-bit filter) or of the path (pos.pkeys).
// Needs warp_go_analyze(..., keys = true) on pos.board. Returns the new legal count.
// Warp-collective.
__device__ inline int warp_go_superko(const EngineView& v, int r, const GoPos& pos, uint32_t* mask) {
  const int lane = threadIdx.x & 31, S = v.S, C = v.C;
  const int8_t* b = pos.board;
  const GoScratch& g = pos.g;
  const int me = pos.player, opp = 3 - me;
  const uint64_t bkey = warp_go_board_key(b, C);
  const int nroot = v.hdr[r].root_nkeys;
  const uint64_t* rk = v.go_keys + (size_t)r * OMQ_GO_MAX_KEYS;
  const uint32_t* bloom = v.go_bloom + (size_t)r * 128;
  int total = 0;
  for (int w = 0; w * 32 <= C; ++w) {
    const uint32_t m = mask[w];
    const int c = w * 32 + lane;
    bool legal = (m >> lane) & 1u;
    if (legal && c < C) {
      int nb[4];
      go_neighbours(c, S, nb);
      int cap[4];
      int ncap = 0;
      uint64_t k = bkey ^ go_stone_key(c, me);
      for (int q = 0; q < 4; ++q) {
        const int s = nb[q];
        if (s < 0 || b[s] != opp) continue;
        const int root = g.par[s];
        if (g.libs[root] != 1) continue;
        bool dup = false;
        for (int j = 0; j < ncap; ++j) dup |= cap[j] == root;
        if (!dup) { cap[ncap++] = root; k ^= g.gkey[root]; }
      }
      if (ncap == 1) {  // a captured group of one stone (no same-coloured neighbour) is the ko point
        int snb[4];
        go_neighbours(cap[0], S, snb);
        bool single = true;
        for (int q = 0; q < 4; ++q) single &= snb[q] < 0 || b[snb[q]] != opp;
        if (single) k ^= go_ko_key(cap[0]);
      }
      bool seen = false;
      for (int i = 0; i < pos.npk && !seen; ++i) seen = pos.pkeys[i] == k;
      if (!seen && ((bloom[(k & 4095) >> 5] >> (k & 31)) & 1u)) {
        int lo = 0, hi = nroot;  // binary search in the sorted root keys
        for (int it = 0; it < 16 && lo < hi; ++it) {
          const int mid = (lo + hi) >> 1;
          if (rk[mid] < k) lo = mid + 1; else hi = mid;
        }
        seen = lo < nroot && rk[lo] == k;
      }
      legal = !seen;
    }
    const uint32_t nm = __ballot_sync(0xFFFFFFFFu, legal);
    __syncwarp();
    if (lane == 0) mask[w] = nm;
    total += __popc(nm);
  }
  __syncwarp();
  return total;
}

// Board k plies before the replayed position (k = 0..7): the ring for k <= depth, else the root
// history.
__device__ __forceinline__ const int8_t* go_hist_board(const EngineView& v, int r, const GoPos& pos,
                                                       const int8_t* ring, int k) {
  const int j = pos.depth - k;
  return j >= 0 ? ring + (size_t)(j % kGoHistory) * v.C : go_root_hist(v, r, -j);
}

}  // namespace omq
