// Tree kernels of the wave search: root reset, selection, expansion + child pick, backup.
//
// One CTA per tree; all trees of an engine advance in lockstep, their leaves meeting in the
// engine's on-device leaf queues (the role of the reference's BatchEvaluationCoordinator,
// python/mcts/utils/batch_evaluation_coordinator.py:48-500).
//
// Selection is not simulated one path at a time. The reference's rank distribution
// (python/mcts/core/wave_search.py:1300-1319) hands the simulations at a parent - always a
// contiguous index range [lo, lo+k) - to its UCB-sorted children in rank order, so a wave is a
// frontier of (node, lo, k, depth) records per depth level. Every visited node appears in
// exactly one record per wave, which makes backup free of atomics and lets it add the values
// of [lo, lo+k) in ascending simulation order - the reference's sequential order
// (python/mcts/gpu/mcts_gpu_accelerator.py:378-393) - so W is bit-exact for any evaluator.
#include <atomic>

#include "chess_device.cuh"
#include "go_device.cuh"
#include "omq_internal.cuh"

namespace omq {

// Block size of the per-tree kernels, chosen at launch: 32 warps per tree when the trees fit in
// about two waves of the SMs (latency: one tree's parents and leaves spread over 32 warps), 8
// warps otherwise (several trees share an SM). Kernels use blockDim, bounded by kThreads.
constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;

// ---------------------------------------------------------------------------------------------
// Gomoku rules on a shared-memory board
// ---------------------------------------------------------------------------------------------
// Warp-collective: for each row y < S, fm[y] gets bit x set when placing `p` on the empty cell
// (y, x) of board b makes five or more in a row through it; fm[32 ..] holds the same cells as a
// flat bit set indexed by cell. For a non-terminal parent this equals
// the reference's full-board scan (python/mcts/utils/fast_terminal_check.py:233-332): any new
// five must contain the new stone. Lane y holds row y's stone mask; a cell completes a five in direction (dr, dc) when one
// of the five windows of 5 cells containing it has its other 4 cells occupied by `p`. Row j of
// a window comes from lane y + j*dr by shuffle, its column offset is a shift by j*dc.
// The board comes as bit rows: lane y holds `row` (the mover's stones of row y, bit x) and `occ`
// (all stones of row y); lanes >= S hold zeros.
__device__ void warp_five_masks(uint32_t row, uint32_t occ, int S, uint32_t* fm) {
  const int lane = threadIdx.x & 31;
  const uint32_t full = (1u << S) - 1u;
  uint32_t five = 0;
#pragma unroll
  for (int d = 0; d < 4; ++d) {
    const int dr = d == 0 ? 0 : 1, dc = d == 1 ? 0 : (d == 3 ? -1 : 1);
    uint32_t t[9];                                  // t[j + 4]: bit x = stone at (y + j*dr, x + j*dc)
#pragma unroll
    for (int j = -4; j <= 4; ++j) {
      const int src = lane + j * dr;
      uint32_t m = __shfl_sync(0xFFFFFFFFu, row, src & 31);
      if (src < 0 || src >= S) m = 0;
      const int sh = j * dc;
      t[j + 4] = sh >= 0 ? (m >> sh) : ((m << -sh) & full);
    }
    // a window covering offsets -k .. 4-k: stones at the k cells before and the 4-k cells after
    const uint32_t l1 = t[3], l2 = l1 & t[2], l3 = l2 & t[1], l4 = l3 & t[0];
    const uint32_t r1 = t[5], r2 = r1 & t[6], r3 = r2 & t[7], r4 = r3 & t[8];
    five |= l4 | (l3 & r1) | (l2 & r2) | (l1 & r3) | r4;
  }
  // flat form: bit (y * S + x) % 32 of word (y * S + x) / 32, so a child's action indexes it
  // without a division by S
  for (int w = lane; w < (kMaxCells + 31) / 32; w += 32) fm[32 + w] = 0u;
  __syncwarp();
  if (lane < S) {
    const uint32_t m = five & ~occ & full;
    const int bit = lane * S, w = bit >> 5, o = bit & 31;
    if (m) {
      atomicOr(&fm[32 + w], m << o);
      if (o + S > 32) atomicOr(&fm[32 + w + 1], m >> (32 - o));
    }
  }
  __syncwarp();
}

// Five in a row starting at cell i in any of the 4 forward directions.
__device__ bool five_from(const int8_t* b, int S, int i) {
  const int p = b[i];
  if (p == 0) return false;
  const int r0 = i / S, c0 = i % S;
  const int dr[4] = {0, 1, 1, 1}, dc[4] = {1, 0, 1, -1};
  for (int d = 0; d < 4; ++d) {
    int s = 1;
    for (; s < 5; ++s) {
      int r = r0 + dr[d] * s, c = c0 + dc[d] * s;
      if (r < 0 || r >= S || c < 0 || c >= S || b[r * S + c] != p) break;
    }
    if (s == 5) return true;
  }
  return false;
}

// ---------------------------------------------------------------------------------------------
// block helpers
// ---------------------------------------------------------------------------------------------
// Exclusive scan of vals[0..n) in place (n <= kThreads * 4), returns the total.
__device__ int block_exclusive_scan(int* vals, int n, int* warp_tot) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = 4;
  int loc[per];
  int sum = 0;
  for (int j = 0; j < per; ++j) {
    int i = tid * per + j;
    loc[j] = i < n ? vals[i] : 0;
    sum += loc[j];
  }
  int inc = sum;
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += t;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { int t = warp_tot[w]; warp_tot[w] = acc; acc += t; }
    warp_tot[blockDim.x >> 5] = acc;
  }
  __syncthreads();
  int run = warp_tot[warp] + inc - sum;
  for (int j = 0; j < per; ++j) {
    int i = tid * per + j;
    if (i < n) vals[i] = run;
    run += loc[j];
  }
  __syncthreads();
  return warp_tot[blockDim.x >> 5];
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long x) {
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long y = __shfl_xor_sync(0xFFFFFFFFu, x, o);
    x = y > x ? y : x;
  }
  return x;
}

// Descending bitonic sort of keys[0..p2) by one warp (p2 a power of two).
__device__ void warp_sort_desc(unsigned long long* keys, int p2) {
  const int lane = threadIdx.x & 31;
  for (int size = 2; size <= p2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = lane; i < (p2 >> 1); i += 32) {
        const int j = 2 * i - (i & (stride - 1));
        const int l = j + stride;
        const bool desc = (j & size) == 0;
        unsigned long long a = keys[j], b = keys[l];
        if ((a < b) == desc) { keys[j] = b; keys[l] = a; }
      }
      __syncwarp();
    }
  }
}

// ---------------------------------------------------------------------------------------------
// begin: reset trees, install roots, queue the roots for the forced root expansion
// ---------------------------------------------------------------------------------------------
// Header + node 0 of tree r for a new search (one thread). After omq_reroot the tree may be kept:
// mode 2 keeps nodes [0, num_nodes) and, with the root already expanded, skips the forced root
// expansion (the root stays queued, its evaluation unused); mode 1 starts a fresh tree whose root
// begins with the chosen child's visit count and value sum.
__device__ void install_root(const EngineView& v, int r, TreeHeader h, int root_flags) {
  const TreeHeader old = v.hdr[r];
  const size_t base = (size_t)r * v.T;
  h.kept = 0;
  if (old.kept == 2 && h.status == OMQ_OK) {
    h.num_nodes = old.num_nodes;
    h.nleaves = 0;
    h.exp_cnt = 0;
  } else {
    h.num_nodes = 1;
    const bool carry = old.kept == 1 && h.status == OMQ_OK;
    v.stats[base] = NodeStats{carry ? old.carry_n : 0, carry ? old.carry_w : 0.0f, 1.0f, 0};
    v.topo[base] = NodeTopo{-1, pack_act_depth(-1, 0), 0, pack_cnt_flags(0, root_flags)};
    v.leaves[(size_t)r * v.WCAP] = Visit{0, 0, 0, 0};
    v.leaf_final[(size_t)r * v.WCAP] = make_int2(0, r);
  }
  v.hdr[r] = h;
  v.q_entries[0][r] = make_int2(r, 0);
  if (r == 0) { v.q_count[0] = v.R; v.q_count[1] = 0; }
}

__global__ void __launch_bounds__(kThreads) k_begin(EngineView v, const int8_t* boards, int search_id) {
  const int r = blockIdx.x, tid = threadIdx.x;
  __shared__ int8_t sb[kMaxCells];
  __shared__ int s_stones, s_five;
  if (tid == 0) { s_stones = 0; s_five = 0; }
  __syncthreads();
  int cnt = 0;
  for (int i = tid; i < v.C; i += blockDim.x) {
    int8_t x = boards[(size_t)r * v.C + i];
    sb[i] = x;
    v.root_board[(size_t)r * v.C + i] = x;
    cnt += x != 0;
  }
  atomicAdd(&s_stones, cnt);
  __syncthreads();
  int five = 0;
  for (int i = tid; i < v.C; i += blockDim.x) five |= five_from(sb, v.S, i) ? 1 : 0;
  if (five) atomicOr(&s_five, 1);
  __syncthreads();
  if (tid == 0) {
    TreeHeader h{};
    h.status = OMQ_OK;
    h.root_player = (s_stones % 2 == 0) ? 1 : 2;
    h.root_mc = s_stones;
    h.root_five = s_five;
    h.nleaves = 1;
    h.exp_off = r;
    h.exp_cnt = 1;
    h.wave_idx = 0;
    h.search_idx = search_id;
    install_root(v, r, h, 0);
  }
}

// Go roots: history boards [R][8][C] and {side to move, ko, passes} per tree. A root reached by
// two passes is terminal and gets no children.
__global__ void k_begin_go(EngineView v, const int8_t* hist, const int32_t* meta, const uint64_t* keys,
                           const int32_t* nkeys, int search_id) {
  const int r = blockIdx.x, tid = threadIdx.x;
  const size_t n = (size_t)kGoHistory * v.C;
  for (size_t i = tid; i < n; i += blockDim.x) v.root_board[(size_t)r * n + i] = hist[(size_t)r * n + i];
  // superko keys of the root's game: sorted (bitonic, padded with all-ones) plus a 4096-bit filter
  __shared__ unsigned long long sk[OMQ_GO_MAX_KEYS];
  __shared__ uint32_t sbloom[128];
  const int nk = (keys && nkeys) ? min(max(nkeys[r], 0), OMQ_GO_MAX_KEYS) : 0;
  for (int i = tid; i < OMQ_GO_MAX_KEYS; i += blockDim.x)
    sk[i] = i < nk ? keys[(size_t)r * OMQ_GO_MAX_KEYS + i] : ~0ull;
  for (int i = tid; i < 128; i += blockDim.x) sbloom[i] = 0u;
  __syncthreads();
  for (int i = tid; i < nk; i += blockDim.x) atomicOr(&sbloom[(sk[i] & 4095) >> 5], 1u << (sk[i] & 31));
  for (int size = 2; size <= OMQ_GO_MAX_KEYS; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = tid; i < OMQ_GO_MAX_KEYS / 2; i += blockDim.x) {
        const int j = 2 * i - (i & (stride - 1)), l = j + stride;
        const bool up = (j & size) == 0;
        const unsigned long long a = sk[j], b = sk[l];
        if ((a > b) == up) { sk[j] = b; sk[l] = a; }
      }
    }
  __syncthreads();
  for (int i = tid; i < OMQ_GO_MAX_KEYS; i += blockDim.x) v.go_keys[(size_t)r * OMQ_GO_MAX_KEYS + i] = sk[i];
  for (int i = tid; i < 128; i += blockDim.x) v.go_bloom[(size_t)r * 128 + i] = sbloom[i];
  if (tid == 0) {
    TreeHeader h{};
    h.num_nodes = 1;
    h.status = OMQ_OK;
    const int player = meta[3 * r], ko = meta[3 * r + 1], passes = meta[3 * r + 2];
    if ((player != 1 && player != 2) || ko < -1 || ko >= v.C || passes < 0) h.status = OMQ_BAD_ARG;
    h.root_player = player;
    h.root_ko = ko;
    h.root_passes = passes;
    h.root_nkeys = nk;
    h.nleaves = 1;
    h.exp_off = r;
    h.exp_cnt = 1;
    h.search_idx = search_id;
    install_root(v, r, h, passes >= 2 ? kFlagTerminal : 0);
  }
}

// Chess roots: position records [R][101] (root + earlier positions) and the number of earlier
// positions; their placement hashes are kept for the repetition count.
__global__ void k_begin_chess(EngineView v, const ChessRec* rec, const int32_t* nprior, int search_id) {
  const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t per = 1 + kChessPrior;
  ChessRec* dst = reinterpret_cast<ChessRec*>(v.root_board) + (size_t)r * per;
  const int np = min(max(nprior[r], 0), kChessPrior);
  for (size_t i = tid; i < per; i += blockDim.x) dst[i] = rec[(size_t)r * per + i];
  for (int i = warp; i < np; i += (int)(blockDim.x >> 5)) {
    const uint64_t h = warp_ch_hash(rec[(size_t)r * per + 1 + i]);
    if (lane == 0) v.chess_prior_hash[(size_t)r * kChessPrior + i] = h;
  }
  if (tid == 0) {
    TreeHeader h{};
    h.num_nodes = 1;
    h.status = OMQ_OK;
    const int side = rec[(size_t)r * per].side;
    if ((side != 1 && side != 2) || nprior[r] < 0 || nprior[r] > kChessPrior) h.status = OMQ_BAD_ARG;
    h.root_player = side;
    h.root_prior = np;
    h.nleaves = 1;
    h.exp_off = r;
    h.exp_cnt = 1;
    h.search_idx = search_id;
    install_root(v, r, h, 0);
  }
}

// ---------------------------------------------------------------------------------------------
// reroot: after a move, keep the chosen child's subtree (or its statistics) for the next search
// ---------------------------------------------------------------------------------------------
// One CTA per tree, trees [r0, r0 + gridDim.x). actions[r] is the move played (-1: fresh tree).
// Mode 1 records the child's visit count and value sum for the next root (the reference's
// use_gpu_tree_reuse path, mcts.py:1929-2005, observably keeps only those). Mode 2 keeps the
// whole subtree, renumbered in breadth-first order with children in action order (the layout
// CSRTree.shift_root describes, csr_tree.py:1020-1229): level by level, a block-wide scan of
// the child counts gives each node's new child_start, and nodes are written to a scratch copy
// (the old id parked in child_start until the node's level is processed), then copied back.
// A chosen child without children falls back to mode 1.
__global__ void __launch_bounds__(1024) k_reroot(EngineView v, const int32_t* actions, int mode,
                                                 NodeStats* sst, NodeTopo* stp, int r0) {
  const int r = r0 + blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ int s_child, s_wsum[32], s_total;
  TreeHeader* H = &v.hdr[r];
  const size_t base = (size_t)r * v.T;
  if (tid == 0) s_child = -1;
  __syncthreads();
  const int a = actions[r];
  const NodeTopo rt = v.topo[base];
  if (H->status != OMQ_OK || H->num_nodes < 1 || a < 0) {
    if (tid == 0) H->kept = 0;
    return;
  }
  for (int j = tid; j < topo_count(rt); j += blockDim.x)
    if (topo_action(v.topo[base + rt.child_start + j]) == a) s_child = rt.child_start + j;
  __syncthreads();
  const int c = s_child;
  if (c < 0) {                         // the move is not in the tree: fresh tree
    if (tid == 0) H->kept = 0;
    return;
  }
  const NodeTopo ct = v.topo[base + c];
  if (mode == 1 || topo_count(ct) == 0) {
    if (tid == 0) {
      const NodeStats cs = v.stats[base + c];
      H->kept = 1;
      H->carry_n = cs.N;
      H->carry_w = cs.W;
    }
    return;
  }
  NodeStats* S = sst + (size_t)blockIdx.x * v.T;
  NodeTopo* P = stp + (size_t)blockIdx.x * v.T;
  if (tid == 0) {
    S[0] = v.stats[base + c];
    P[0] = NodeTopo{-1, pack_act_depth(-1, 0), c, ct.cnt_flags};
  }
  __syncthreads();
  int lo = 0, hi = 1;
  for (int level = 0; lo < hi && level <= v.max_depth + 1; ++level) {
    int carry = 0;
    for (int start = lo; start < hi; start += blockDim.x) {
      const int i = start + tid;
      int cnt = 0, ocs = 0;
      if (i < hi) {
        const NodeTopo ot = v.topo[base + P[i].child_start];
        cnt = topo_count(ot);
        ocs = ot.child_start;
      }
      // block-wide exclusive scan of cnt
      int x = cnt;
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (lane == 31) s_wsum[warp] = x;
      __syncthreads();
      if (warp == 0) {
        int w = lane < (int)(blockDim.x >> 5) ? s_wsum[lane] : 0;
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, w, o);
          if (lane >= o) w += y;
        }
        s_wsum[lane] = w;                 // inclusive warp totals
        if (lane == 31) s_total = w;
      }
      __syncthreads();
      const int excl = x - cnt + (warp ? s_wsum[warp - 1] : 0);
      if (i < hi) {
        const int ns = hi + carry + excl;
        const int d = topo_depth(P[i]);
        for (int j = 0; j < cnt; ++j) {
          const NodeTopo ot = v.topo[base + ocs + j];
          S[ns + j] = v.stats[base + ocs + j];
          P[ns + j] = NodeTopo{i, pack_act_depth(topo_action(ot), d + 1), ocs + j, ot.cnt_flags};
        }
        P[i].child_start = cnt ? ns : 0;
      }
      carry += s_total;
      __syncthreads();
    }
    lo = hi;
    hi += carry;
  }
  for (int i = tid; i < hi; i += blockDim.x) {
    v.stats[base + i] = S[i];
    v.topo[base + i] = P[i];
  }
  if (tid == 0) {
    H->num_nodes = hi;
    H->kept = 2;
  }
}

void launch_reroot(const EngineView& v, const int32_t* actions, int mode, NodeStats* scratch_stats,
                   NodeTopo* scratch_topo, int chunk, cudaStream_t s) {
  for (int r0 = 0; r0 < v.R; r0 += chunk) {
    k_reroot<<<min(chunk, v.R - r0), 1024, 0, s>>>(v, actions, mode, scratch_stats, scratch_topo, r0);
    count_launches(1);
  }
}

// ---------------------------------------------------------------------------------------------
// root Dirichlet noise
// ---------------------------------------------------------------------------------------------
// Uniform in (0, 1) from a 64-bit counter hash (24 significant bits).
__device__ __forceinline__ float unit_uniform(uint64_t key) {
  return ((float)(mix64(key) >> 40) + 0.5f) * (1.0f / 16777216.0f);
}

// Gamma(alpha, 1) by Marsaglia & Tsang (2000, "A simple method for generating gamma variables"),
// with the alpha < 1 boost Gamma(alpha) = Gamma(alpha + 1) * U^(1/alpha). Normal deviates by
// Box-Muller. The rejection loop is bounded (16 rounds; acceptance is > 95% per round), after
// which the mode of Gamma(alpha + 1) stands in.
__device__ float gamma_sample(uint64_t key, float alpha) {
  const float a = alpha < 1.0f ? alpha + 1.0f : alpha;
  const float d = a - 1.0f / 3.0f;
  const float c = rsqrtf(9.0f * d);
  float g = d;
  for (int it = 0; it < 16; ++it) {
    const uint64_t k = key + 0x9E3779B97F4A7C15ull * (uint64_t)(4 * it + 1);
    const float u1 = unit_uniform(k), u2 = unit_uniform(k + 1);
    const float x = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    float t = 1.0f + c * x;
    if (t <= 0.0f) continue;
    t = t * t * t;
    const float u = unit_uniform(k + 2);
    if (logf(u) < 0.5f * x * x + d - d * t + d * logf(t)) { g = d * t; break; }
  }
  if (alpha < 1.0f) g *= powf(unit_uniform(key ^ 0xA0761D6478BD642Full), 1.0f / alpha);
  return g;
}

// ---------------------------------------------------------------------------------------------
// selection
// ---------------------------------------------------------------------------------------------
struct SelectShared {
  int cnt[2];
  int nleaf;
  int nlog;
  int overflow;
  int warp_tot[kWarps + 1];
};

__device__ __forceinline__ void emit_child(const EngineView& v, int r, Visit* next, int* next_cnt,
                                           Visit* log, int* nlog, int* overflow, int child, int lo,
                                           int k, int depth) {
  const size_t base = (size_t)r * v.T;
  if (v.enable_vl) v.stats[base + child].VL += k;  // only this warp touches this child this wave
  const int fi = atomicAdd(next_cnt, 1);
  const Visit x{child, lo, k, depth};
  next[fi] = x;
  const int li = atomicAdd(nlog, 1);
  if (li < v.LOGCAP) log[li] = x; else *overflow = 1;
}

__device__ void select_finish(const EngineView& v, int r, int wave, Visit* s_leaves, int* s_scan, int* warp_tot,
                              int nleaf, int nlog, int overflow);

__global__ void __launch_bounds__(kThreads, 1) k_select(EngineView v, int wave) {
  extern __shared__ unsigned char smem_raw[];
  SelectShared& sh = *reinterpret_cast<SelectShared*>(smem_raw);
  int p2 = 1;
  while (p2 < v.max_children) p2 <<= 1;
  unsigned long long* keys_all =
      reinterpret_cast<unsigned long long*>(smem_raw + ((sizeof(SelectShared) + 15) & ~15));
  Visit* s_leaves = reinterpret_cast<Visit*>(keys_all + (size_t)(blockDim.x >> 5) * p2);
  int* s_scan = reinterpret_cast<int*>(s_leaves + v.WCAP);

  const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // Slices: with few trees, gridDim.y CTAs share a tree. Every slice ranks the root's children
  // the same way; slice y emits the children of rank i with i % gridDim.y == y and then descends
  // their subtrees alone (its own frontier; subtrees are disjoint, so no slice waits on another).
  // The visit log and the leaves go to per-tree global counters, and k_select_commit sorts the
  // leaves and queues the expandable ones afterwards.
  const int slices = (int)gridDim.y, slice = (int)blockIdx.y;
  TreeHeader* H = &v.hdr[r];
  if (H->status != OMQ_OK) return;
  const size_t base = (size_t)r * v.T;
  Visit* F[2] = {v.frontier + ((size_t)r * slices + slice) * 2 * v.WCAP,
                 v.frontier + ((size_t)r * slices + slice) * 2 * v.WCAP + v.WCAP};
  Visit* log = v.vlog + (size_t)r * v.LOGCAP;
  unsigned long long* keys = keys_all + (size_t)warp * p2;
  int32_t* gctr = v.sel_ctr + 4 * (size_t)r;  // sliced: {log entries, leaves, overflow, 0}
  int* nlogp = slices > 1 ? gctr : &sh.nlog;
  int* ovfp = slices > 1 ? gctr + 2 : &sh.overflow;
  // whether this slice emits the root child of rank `rank` (children of other nodes: always)
  auto owns = [&](int node, int rank) { return node != 0 || rank % slices == slice; };

  if (tid == 0) {
    const Visit root{0, 0, wave, 0};
    F[0][0] = root;
    if (slices == 1) {
      log[0] = root;
    } else if (slice == 0) {
      const int li = atomicAdd(gctr, 1);
      if (li < v.LOGCAP) log[li] = root; else gctr[2] = 1;
    }
    sh.cnt[0] = 1; sh.cnt[1] = 0;
    sh.nleaf = 0; sh.nlog = 1; sh.overflow = 0;
  }
  __syncthreads();
  int cur = 0, depth0 = 1;
  {
    // Depth 1 is the root alone. When its simulations take the sorted-children path (more than 8
    // of them, or more than it has children) and no root noise is mixed in, the whole block
    // scores, sorts and distributes them instead of one warp; the keys are unique, so the order
    // - and every result - is the one the warp path gives.
    const NodeTopo rt = v.topo[base];
    const int n = topo_count(rt);
    if (n > 0 && !(v.noise_eps > 0.0f) && !(wave <= n && wave <= 8)) {
      const int cs = rt.child_start;
      const float sq = parent_sqrt(v.stats[base].N);
      unsigned long long* bk = keys_all;                  // p2 >= n entries
      for (int j = tid; j < p2; j += blockDim.x)
        bk[j] = j < n ? rank_key(ucb_score_sq(v.stats[base + cs + j], sq, v.c_puct, v.vl_value,
                                              v.enable_vl), j)
                      : 0ull;
      __syncthreads();
      for (int size = 2; size <= p2; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          for (int i = tid; i < (p2 >> 1); i += blockDim.x) {
            const int j = 2 * i - (i & (stride - 1)), l = j + stride;
            const bool desc = (j & size) == 0;
            const unsigned long long x = bk[j], y = bk[l];
            if ((x < y) == desc) { bk[j] = y; bk[l] = x; }
          }
          __syncthreads();
        }
      if (wave <= n) {
        for (int rr = tid; rr < wave; rr += blockDim.x)
          if (owns(0, rr))
            emit_child(v, r, F[1], &sh.cnt[1], log, nlogp, ovfp, cs + key_slot(bk[rr]), rr, 1, 1);
      } else {
        const int basek = wave / n, extra = wave % n;
        for (int rr = tid; rr < n; rr += blockDim.x) {
          const int c = basek + (rr < extra ? 1 : 0);
          const int off = rr * basek + (rr < extra ? rr : extra);
          if (owns(0, rr))
            emit_child(v, r, F[1], &sh.cnt[1], log, nlogp, ovfp, cs + key_slot(bk[rr]), off, c, 1);
        }
      }
      __syncthreads();
      if (tid == 0) sh.cnt[0] = 0;
      cur = 1;
      depth0 = 2;
      __syncthreads();
    }
  }
  for (int depth = depth0; depth < v.max_depth; ++depth) {
    const int n_cur = sh.cnt[cur];
    if (n_cur == 0) break;
    const int nwarps = (int)(blockDim.x >> 5);
    // this warp's parents are i = warp + nwarps * t; lane t prefetches parent t of each group of
    // 32 (frontier entry, topology, visit count), so the dependent loads of 32 parents overlap
    for (int g0 = warp; g0 < n_cur; g0 += 32 * nwarps) {
      const int mine = g0 + nwarps * lane;
      Visit pe{0, 0, 0, 0};
      NodeTopo ptp{0, 0, 0, 0};
      int32_t pn = 0;
      if (mine < n_cur) {
        pe = F[cur][mine];
        ptp = v.topo[base + pe.node];
        if (topo_count(ptp) > 0) pn = v.stats[base + pe.node].N;
      }
      const int ng = min(32, (n_cur - g0 + nwarps - 1) / nwarps);
      // children lane and lane + 32 of the next parent, loaded while this one is scored
      NodeStats pre0{0, 0.0f, 0.0f, 0}, pre1{0, 0.0f, 0.0f, 0};
      auto prefetch = [&](int tt) {
        const int pcs = __shfl_sync(0xFFFFFFFFu, ptp.child_start, tt);
        const int pnn = topo_count(NodeTopo{0, 0, 0, __shfl_sync(0xFFFFFFFFu, ptp.cnt_flags, tt)});
        if (lane < pnn) pre0 = v.stats[base + pcs + lane];
        if (lane + 32 < pnn) pre1 = v.stats[base + pcs + lane + 32];
      };
      prefetch(0);
    for (int t = 0; t < ng; ++t) {
      const NodeStats cur0 = pre0, cur1 = pre1;
      if (t + 1 < ng) prefetch(t + 1);
      const Visit e{__shfl_sync(0xFFFFFFFFu, pe.node, t), __shfl_sync(0xFFFFFFFFu, pe.lo, t),
                    __shfl_sync(0xFFFFFFFFu, pe.k, t), __shfl_sync(0xFFFFFFFFu, pe.depth, t)};
      const int n = topo_count(NodeTopo{0, 0, 0, __shfl_sync(0xFFFFFFFFu, ptp.cnt_flags, t)});
      if (n == 0) {  // no children: the simulation stops here (wave_search.py:762-768)
        if (lane == 0 && (e.node != 0 || slice == 0)) {
          int li = atomicAdd(&sh.nleaf, 1);
          if (li < v.WCAP) s_leaves[li] = e; else sh.overflow = 1;
        }
        continue;
      }
      const int cs = __shfl_sync(0xFFFFFFFFu, ptp.child_start, t);
      const int32_t np = __shfl_sync(0xFFFFFFFFu, pn, t);
      unsigned long long lanebest = 0;
      bool regbest = false;
      if (e.node == 0 && v.noise_eps > 0.0f) {
        // One Dirichlet(alpha) vector per wave at the root (wave_search.py:1160-1170): gamma draws
        // normalised in the engine's fixed summation order (lane-strided partials, butterfly).
        float g[12];
        float part = 0.0f;
        const uint64_t wkey = v.noise_seed ^ mix64(((uint64_t)(uint32_t)H->search_idx << 32) |
                                                   (uint32_t)H->wave_idx) ^ mix64((uint64_t)r + 0x51ED27ull);
#pragma unroll
        for (int t = 0; t < 12; ++t) {
          const int j = lane + 32 * t;
          g[t] = j < n ? gamma_sample(mix64(wkey + (uint64_t)j * 0xD1B54A32D192ED03ull), v.noise_alpha) : 0.0f;
          part = __fadd_rn(part, g[t]);
        }
        for (int o = 16; o > 0; o >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xFFFFFFFFu, part, o));
        float* out = v.root_noise + (size_t)r * v.A;
        if (slice == 0)
          for (int a = lane; a < v.A; a += 32) out[a] = 0.0f;
        __syncwarp();
#pragma unroll
        for (int t = 0; t < 12; ++t) {
          const int j = lane + 32 * t;
          if (j >= n) continue;
          const float noise = __fdiv_rn(g[t], part);
          NodeStats st = v.stats[base + cs + j];
          st.P = __fadd_rn(__fmul_rn(v.noise_keep, st.P), __fmul_rn(v.noise_eps, noise));
          keys[j] = rank_key(ucb_score(st, np, v.c_puct, v.vl_value, v.enable_vl), j);
          if (slice == 0) out[topo_action(v.topo[base + cs + j])] = noise;
        }
      } else {
        // children statistics: the first two per lane came with the prefetch, the rest four
        // independent 16-byte loads in flight per lane
        // (one simulation at this parent: only the arg-max is needed, kept in registers)
        const NodeStats* cst = v.stats + base + cs;
        const float sq = parent_sqrt(np);
        auto put = [&](int j, unsigned long long key) {
          if (e.k == 1) lanebest = key > lanebest ? key : lanebest;
          else keys[j] = key;
        };
        if (lane < n) put(lane, rank_key(ucb_score_sq(cur0, sq, v.c_puct, v.vl_value, v.enable_vl), lane));
        if (lane + 32 < n)
          put(lane + 32, rank_key(ucb_score_sq(cur1, sq, v.c_puct, v.vl_value, v.enable_vl), lane + 32));
        int j = lane + 64;
        for (; j + 96 < n; j += 128) {
          const NodeStats s0 = cst[j], s1 = cst[j + 32], s2 = cst[j + 64], s3 = cst[j + 96];
          put(j, rank_key(ucb_score_sq(s0, sq, v.c_puct, v.vl_value, v.enable_vl), j));
          put(j + 32, rank_key(ucb_score_sq(s1, sq, v.c_puct, v.vl_value, v.enable_vl), j + 32));
          put(j + 64, rank_key(ucb_score_sq(s2, sq, v.c_puct, v.vl_value, v.enable_vl), j + 64));
          put(j + 96, rank_key(ucb_score_sq(s3, sq, v.c_puct, v.vl_value, v.enable_vl), j + 96));
        }
        for (; j < n; j += 32) {
          const NodeStats st = cst[j];
          put(j, rank_key(ucb_score_sq(st, sq, v.c_puct, v.vl_value, v.enable_vl), j));
        }
        regbest = e.k == 1;
      }
      __syncwarp();
      if (regbest) {
        const unsigned long long best = warp_max_u64(lanebest);
        if (lane == 0 && owns(e.node, 0))
          emit_child(v, r, F[cur ^ 1], &sh.cnt[cur ^ 1], log, nlogp, ovfp, cs + key_slot(best), e.lo, 1,
                     e.depth + 1);
        __syncwarp();
      } else if (e.k <= n && e.k <= 8) {
        // k best children, one simulation each, by repeated arg-max
        for (int rr = 0; rr < e.k; ++rr) {
          unsigned long long best = 0;
          for (int j = lane; j < n; j += 32) best = keys[j] > best ? keys[j] : best;
          best = warp_max_u64(best);
          const int slot = key_slot(best);
          if (lane == 0) {
            keys[slot] = 0;
            if (owns(e.node, rr))
              emit_child(v, r, F[cur ^ 1], &sh.cnt[cur ^ 1], log, nlogp, ovfp, cs + slot, e.lo + rr, 1,
                         e.depth + 1);
          }
          __syncwarp();
        }
      } else {
        for (int j = n + lane; j < p2; j += 32) keys[j] = 0;
        __syncwarp();
        warp_sort_desc(keys, p2);
        if (e.k <= n) {
          for (int rr = lane; rr < e.k; rr += 32)
            if (owns(e.node, rr))
              emit_child(v, r, F[cur ^ 1], &sh.cnt[cur ^ 1], log, nlogp, ovfp, cs + key_slot(keys[rr]),
                         e.lo + rr, 1, e.depth + 1);
        } else {
          const int basek = e.k / n, extra = e.k % n;
          for (int rr = lane; rr < n; rr += 32) {
            const int c = basek + (rr < extra ? 1 : 0);
            const int off = rr * basek + (rr < extra ? rr : extra);
            if (owns(e.node, rr))
              emit_child(v, r, F[cur ^ 1], &sh.cnt[cur ^ 1], log, nlogp, ovfp, cs + key_slot(keys[rr]),
                         e.lo + off, c, e.depth + 1);
          }
        }
      }
      __syncwarp();
    }
    }
    __syncthreads();
    if (tid == 0) sh.cnt[cur] = 0;
    cur ^= 1;
    __syncthreads();
  }
  // depth limit reached: the remaining simulations stop at nodes that still have children
  for (int i = tid; i < sh.cnt[cur]; i += blockDim.x) {
    if (F[cur][i].node == 0 && slice != 0) continue;  // the root: slice 0's
    int li = atomicAdd(&sh.nleaf, 1);
    if (li < v.WCAP) s_leaves[li] = F[cur][i]; else sh.overflow = 1;
  }
  __syncthreads();
  if (slices > 1) {
    // this slice's leaves into the tree's (unsorted) leaf list; k_select_commit finishes
    __shared__ int s_off;
    const int nl = min(sh.nleaf, v.WCAP);
    if (tid == 0) {
      s_off = atomicAdd(gctr + 1, nl);
      if (sh.overflow) gctr[2] = 1;
    }
    __syncthreads();
    Visit* gl = v.leaves + (size_t)r * v.WCAP;
    for (int i = tid; i < nl; i += blockDim.x) {
      if (s_off + i < v.WCAP) gl[s_off + i] = s_leaves[i];
      else gctr[2] = 1;
    }
    return;
  }
  select_finish(v, r, wave, s_leaves, s_scan, sh.warp_tot, min(sh.nleaf, v.WCAP), sh.nlog, sh.overflow);
}

// Selection's end for tree r: sort its leaves (s_leaves, in shared memory) ascending by node id into
// v.leaves, flag the expandable ones, reserve their expansion-queue entries, and set the header's
// wave fields. Block-collective.
__device__ void select_finish(const EngineView& v, int r, int wave, Visit* s_leaves, int* s_scan, int* warp_tot,
                              int nleaf, int nlog, int overflow) {
  const int tid = threadIdx.x;
  TreeHeader* H = &v.hdr[r];
  const size_t base = (size_t)r * v.T;
  // sort leaves ascending by node id (each node is a leaf at most once per wave)
  Visit* gleaves = v.leaves + (size_t)r * v.WCAP;
  for (int i = tid; i < nleaf; i += blockDim.x) {
    const int key = s_leaves[i].node;
    int rank = 0;
    for (int j = 0; j < nleaf; ++j) rank += s_leaves[j].node < key;
    gleaves[rank] = s_leaves[i];
  }
  __syncthreads();
  // expandable leaves: no children, not terminal (wave_search.py:829-855)
  for (int i = tid; i < nleaf; i += blockDim.x) {
    const NodeTopo tp = v.topo[base + gleaves[i].node];
    s_scan[i] = (topo_count(tp) == 0 && !(topo_flags(tp) & kFlagTerminal)) ? 1 : 0;
  }
  __syncthreads();
  // keep the flags (scan overwrites them): stash in leaf_final.y as 0/1 first
  int2* lf = v.leaf_final + (size_t)r * v.WCAP;
  for (int i = tid; i < nleaf; i += blockDim.x) lf[i] = make_int2(-1, s_scan[i]);
  __syncthreads();
  const int nexp = block_exclusive_scan(s_scan, nleaf, warp_tot);
  __shared__ int s_qbase;
  if (tid == 0) s_qbase = nexp > 0 ? atomicAdd(&v.q_count[0], nexp) : 0;
  __syncthreads();
  const int qbase = s_qbase;
  for (int i = tid; i < nleaf; i += blockDim.x) {
    if (lf[i].y) {
      const int q = qbase + s_scan[i];
      v.q_entries[0][q] = make_int2(r, gleaves[i].node);
      lf[i] = make_int2(-1, q);
    } else {
      lf[i] = make_int2(-1, -1);
    }
  }
  if (tid == 0) {
    H->nleaves = nleaf;
    H->nlog = min(nlog, v.LOGCAP);
    H->exp_off = qbase;
    H->exp_cnt = nexp;
    H->wave = wave;
    H->wave_idx += 1;
    if (overflow) H->status = OMQ_QUEUE_OVERFLOW;
  }
}

// The end of a sliced k_select: the tree's leaves (from every slice) into shared memory, then
// select_finish. Dynamic shared memory: WCAP leaves and WCAP ints.
__global__ void __launch_bounds__(kThreads) k_select_commit(EngineView v, int wave) {
  extern __shared__ unsigned char commit_smem[];
  Visit* s_leaves = reinterpret_cast<Visit*>(commit_smem);
  int* s_scan = reinterpret_cast<int*>(s_leaves + v.WCAP);
  __shared__ int warp_tot[kWarps + 1];
  const int r = blockIdx.x, tid = threadIdx.x;
  if (v.hdr[r].status != OMQ_OK) return;
  const int32_t* gctr = v.sel_ctr + 4 * (size_t)r;
  const int nleaf = min(gctr[1], v.WCAP);
  const Visit* gl = v.leaves + (size_t)r * v.WCAP;
  for (int i = tid; i < nleaf; i += blockDim.x) s_leaves[i] = gl[i];
  __syncthreads();
  select_finish(v, r, wave, s_leaves, s_scan, warp_tot, nleaf, gctr[0], gctr[2]);
}

// ---------------------------------------------------------------------------------------------
// expansion + child pick
// ---------------------------------------------------------------------------------------------
constexpr int kMaxDepthCap = 128;

struct ChessWarpSmem {
  ChessReplay rep;
  uint32_t mask[kChessMaskWords];
  ChessMoveList list;
};

struct ExpandWarpSmem {
  uint32_t five[32 + (kMaxCells + 31) / 32];  // Gomoku: cells where the mover completes five
                                              // (warp_five_masks): rows, then flat by cell
  int16_t acts[kMaxDepthCap];
  int16_t legal[kMaxCells + 1];
  float pv[kMaxCells + 1];
};

// Sum of the legal-move policy pv[0..n) in exactly the order in which torch's CPU sum kernel adds
// a contiguous fp32 vector, which is what the reference's `priors.sum()` runs on its CPU path
// (wave_search.py:894-895). That kernel (ATen's cascade sum for an inner reduction) views the
// vector as 8-lane vectors: 4 interleaved vector accumulators take rows of 32 elements (lane L of
// this warp holds accumulator L, i.e. elements L, L+32, L+64, ...); after every 16 rows the
// accumulators are added into a second level and restarted (a third level after 256 rows, and so
// on); the full vectors left after the last row go to the first vector accumulator; the four
// vector accumulators are then added 0+1, +2, +3; finally a scalar starting at 0 adds the elements
// after the last full vector, then the 8 lanes in order. Fewer than 8 elements: 4 scalar
// accumulators instead of vectors, the same way. The order is pinned against torch.sum for every
// length up to 5,000 (oracle/torch_sum.cpp holds the host twin) and is the same under the AVX2,
// AVX-512 and default CPU kernels. Valid for n < 2^21 (16-row cascade blocks).
__device__ float warp_torch_sum(const float* pv, int n) {
  const int lane = threadIdx.x & 31;
  float r = 0.0f;
  if (n < 8) {
    if (lane == 0) {
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const int rows = n >> 2;  // 0 or 1 row of 4 scalars
      for (int k = 0; k < 4 * rows; ++k) acc[k] = __fadd_rn(acc[k], pv[k]);
      for (int k = 4 * rows; k < n; ++k) acc[0] = __fadd_rn(acc[0], pv[k]);
      r = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), acc[2]), acc[3]);
    }
    return __shfl_sync(0xFFFFFFFFu, r, 0);
  }
  const int vecs = n >> 3, rows = vecs >> 2;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  int i = 0;
  for (; i + 16 <= rows;) {
    for (int j = 0; j < 16; ++j, ++i) acc[0] = __fadd_rn(acc[0], pv[32 * i + lane]);
#pragma unroll
    for (int l = 1; l < 4; ++l) {
      acc[l] = __fadd_rn(acc[l], acc[l - 1]);
      acc[l - 1] = 0.0f;
      if (i & (15 << (4 * l))) break;
    }
  }
  for (; i < rows; ++i) acc[0] = __fadd_rn(acc[0], pv[32 * i + lane]);
  float a = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), acc[2]), acc[3]);
  // full vectors after the last row: into vector accumulator 0 (lanes 0..7)
  if (lane < 8)
    for (int t = 4 * rows; t < vecs; ++t) a = __fadd_rn(a, pv[8 * t + lane]);
  // vector accumulators 0 + 1 + 2 + 3, lane by lane
  const float a1 = __shfl_sync(0xFFFFFFFFu, a, (lane + 8) & 31);
  const float a2 = __shfl_sync(0xFFFFFFFFu, a, (lane + 16) & 31);
  const float a3 = __shfl_sync(0xFFFFFFFFu, a, (lane + 24) & 31);
  const float v = __fadd_rn(__fadd_rn(__fadd_rn(a, a1), a2), a3);
  float fin = 0.0f;
  for (int k = 8 * vecs; k < n; ++k) fin = __fadd_rn(fin, pv[k]);
#pragma unroll
  for (int l = 0; l < 8; ++l) fin = __fadd_rn(fin, __shfl_sync(0xFFFFFFFFu, v, l));
  return fin;
}

__global__ void __launch_bounds__(kThreads, 1) k_expand(EngineView v, int root_mode) {
  extern __shared__ unsigned char expand_smem[];
  ExpandWarpSmem* ws = reinterpret_cast<ExpandWarpSmem*>(expand_smem);  // [warps]
  __shared__ int s_cnt[1024];
  __shared__ int warp_tot[kWarps + 1];
  __shared__ int s_fbase;
  const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // Slices: with few trees (Gomoku), gridDim.y CTAs share one tree, CTA y taking the leaves
  // i with i % gridDim.y == y; H->num_nodes is then left unchanged here (every slice reads it)
  // and k_expand_commit applies the node count and the final-node queue afterwards.
  const int slices = (int)gridDim.y, slice = (int)blockIdx.y;
  TreeHeader* H = &v.hdr[r];
  if (H->status != OMQ_OK) return;
  const size_t base = (size_t)r * v.T;
  const int nleaf = H->nleaves;
  const int num_nodes = H->num_nodes;
  Visit* leaves = v.leaves + (size_t)r * v.WCAP;
  int2* lf = v.leaf_final + (size_t)r * v.WCAP;
  const float* pol = v.q_policy[0];

  const bool go = v.game == OMQ_GAME_GO;
  const bool chs = v.game == OMQ_GAME_CHESS;
  // Gomoku: the root position as bit rows per player and as a flat occupancy bit set (bit c % 32
  // of word c / 32); a leaf's position is these plus the few stones of its path
  __shared__ uint32_t s_rows[2][32];
  __shared__ uint32_t s_occ[(kMaxCells + 31) / 32];
  if (!go && !chs) {
    const int8_t* rb = v.root_board + (size_t)r * v.C;
    if (tid < 32) {
      uint32_t p1 = 0, p2 = 0;
      if (tid < v.S)
        for (int x = 0; x < v.S; ++x) {
          const int q = rb[tid * v.S + x];
          p1 |= (q == 1 ? 1u : 0u) << x;
          p2 |= (q == 2 ? 1u : 0u) << x;
        }
      s_rows[0][tid] = p1;
      s_rows[1][tid] = p2;
    } else if (tid < 32 + (kMaxCells + 31) / 32) {
      const int w = tid - 32;
      uint32_t o = 0;
      for (int b = 0; b < 32; ++b) {
        const int c = 32 * w + b;
        if (c < v.C && rb[c] != 0) o |= 1u << b;
      }
      s_occ[w] = o;
    }
  }
  GoPos* gpos = reinterpret_cast<GoPos*>(expand_smem + (blockDim.x >> 5) * sizeof(ExpandWarpSmem));
  ChessWarpSmem* cws = reinterpret_cast<ChessWarpSmem*>(expand_smem + (blockDim.x >> 5) * sizeof(ExpandWarpSmem));
  if (chs) {
    // chess: replay the leaf, find its legal moves; a terminal leaf (ChessState::isTerminal)
    // is flagged here and gets no children
    ChessWarpSmem& cw = cws[warp];
    for (int i = warp; i < nleaf; i += (int)(blockDim.x >> 5)) {
      int n = 0;
      const int node = leaves[i].node;
      if (lf[i].y >= 0 && !(topo_flags(v.topo[base + node]) & kFlagTerminal)) {
        const int d = warp_ch_replay(v, r, node, cw.rep, false);
        if (d < 0) { if (lane == 0) H->status = OMQ_BAD_ARG; }
        else {
          n = warp_ch_legal(cw.rep.pos, cw.mask, cw.list);
          if (lane == 0 && ch_terminal(cw.rep.pos, n)) {
            NodeTopo lt = v.topo[base + node];
            lt.cnt_flags = pack_cnt_flags(topo_count(lt), topo_flags(lt) | kFlagTerminal);
            v.topo[base + node] = lt;
          }
          if (ch_terminal(cw.rep.pos, n)) n = 0;
          uint32_t* m = v.go_mask + ((size_t)r * v.WCAP + i) * kChessMaskWords;
          for (int w = lane; w < kChessMaskWords; w += 32) m[w] = n ? cw.mask[w] : 0u;
        }
      }
      if (lane == 0) s_cnt[i] = n;
      __syncwarp();
    }
  } else if (go) {
    // Go: children are the legal moves of the leaf position (replayed from the root); the
    // legal bits and the leaf's pass count go to a per-leaf scratch for the second pass
    GoPos& gp = gpos[warp];
    for (int i = warp; i < nleaf; i += (int)(blockDim.x >> 5)) {
      int n = 0;
      if (lf[i].y >= 0 && !(topo_flags(v.topo[base + leaves[i].node]) & kFlagTerminal)) {
        const bool keyed = v.go_superko || v.go_cycle;
        const int d = warp_go_replay(v, r, leaves[i].node, gp, nullptr, keyed);
        if (d < 0) { if (lane == 0) H->status = OMQ_BAD_ARG; n = 0; }
        else {
          uint32_t* m = v.go_mask + ((size_t)r * v.WCAP + i) * 32;
          warp_go_analyze(gp.board, v.S, gp.g, keyed);
          n = warp_go_legal(gp.board, v.S, gp.player, gp.ko, gp.g, m);
          if (v.go_superko) n = warp_go_superko(v, r, gp, m);
          if (v.go_cycle) warp_go_cycle(v, r, gp, m, m + 16);
          if (lane == 0) m[12] = (uint32_t)gp.passes;
        }
      }
      if (lane == 0) s_cnt[i] = n;
      __syncwarp();
    }
  } else {
    // children per expandable leaf: the empty cells of its board, i.e. C - move_count
    for (int i = tid; i < nleaf; i += blockDim.x)
      s_cnt[i] = lf[i].y >= 0 ? max(v.C - (H->root_mc + leaves[i].depth), 0) : 0;
  }
  __syncthreads();
  const int total = block_exclusive_scan(s_cnt, nleaf, warp_tot);
  if (num_nodes + total > v.T) {  // "Tree full" (csr_tree.py:405-406)
    if (tid == 0) H->status = OMQ_TREE_FULL;
    return;
  }
  if (slices > 1 && slice == 0 && tid == 0) H->exp_total = total;
  ExpandWarpSmem& W = ws[warp];
  // Gomoku: every thread walks one expandable leaf's parent chain into the path scratch (slot
  // kMaxDepthCap - 1 holds the depth), so the chains' dependent loads overlap across leaves
  int16_t* gpath = v.leaf_paths + (size_t)r * v.WCAP * kMaxDepthCap;
  if (!go && !chs) {
    for (int i = slice + slices * tid; i < nleaf; i += slices * blockDim.x)
      if (lf[i].y >= 0) {
        int16_t* P = gpath + (size_t)i * kMaxDepthCap;
        P[kMaxDepthCap - 1] = (int16_t)path_actions(v.topo + base, leaves[i].node, kMaxDepthCap - 2, P);
      }
    __syncthreads();
  }
  for (int i = slice + slices * warp; i < nleaf; i += slices * (int)(blockDim.x >> 5)) {
    const Visit e = leaves[i];
    const int q = lf[i].y;
    int final_node = e.node, ext = 0;
    if (q >= 0 && (go || chs)) {
      const uint32_t* m = v.go_mask + ((size_t)r * v.WCAP + i) * (chs ? kChessMaskWords : 32);
      const int leaf_passes = go ? (int)m[12] : 0;
      int n = 0;
      if (!(topo_flags(v.topo[base + e.node]) & kFlagTerminal)) {
        for (int w = 0; w < (chs ? kChessMaskWords : kGoMaskWords) && w * 32 < v.A; ++w) {
          const int c = w * 32 + lane;
          const bool legal = c < v.A && ((m[w] >> lane) & 1u);
          const unsigned bm = __ballot_sync(0xFFFFFFFFu, legal);
          if (legal) {
            const int j = n + __popc(bm & ((1u << lane) - 1));
            W.legal[j] = (int16_t)c;
            W.pv[j] = pol[(size_t)q * v.A + c];
          }
          n += __popc(bm);
        }
      }
      __syncwarp();
      const float denom = __fadd_rn(warp_torch_sum(W.pv, n), 1e-8f);
      const int start = num_nodes + s_cnt[i];
      const int d = e.depth;
      unsigned long long best = 0;
      const float sq_leaf = parent_sqrt(v.stats[base + e.node].N);
      for (int j = lane; j < n; j += 32) {
        const int a = W.legal[j];
        const float P = __fdiv_rn(W.pv[j], denom);
        // second consecutive pass, or (Japanese / Korean) a third repetition
        const bool term = go && ((a == v.C && leaf_passes >= 1) ||
                                 (v.go_cycle && ((m[16 + (a >> 5)] >> (a & 31)) & 1u)));
        const int c = start + j;
        const NodeStats st{0, 0.0f, P, 0};
        v.stats[base + c] = st;
        v.topo[base + c] = NodeTopo{e.node, pack_act_depth(a, d + 1), 0,
                                    pack_cnt_flags(0, term ? kFlagTerminal : 0)};
        const unsigned long long key =
            rank_key(ucb_score_sq(st, sq_leaf, v.c_puct, v.vl_value, v.enable_vl), j);
        best = key > best ? key : best;
      }
      best = warp_max_u64(best);
      if (lane == 0) {
        NodeTopo lt = v.topo[base + e.node];
        lt.child_start = start;
        lt.cnt_flags = pack_cnt_flags(n, topo_flags(lt));
        v.topo[base + e.node] = lt;
      }
      if (!root_mode && n > 0) {
        final_node = start + key_slot(best);
        ext = (e.depth + 1 < v.max_depth) ? 1 : 0;
        if (lane == 0 && v.enable_vl) v.stats[base + final_node].VL += 1;
      }
    } else if (q >= 0) {
      // reconstruct the leaf's board: root board + the stones along its path (walked above)
      constexpr int kChunks = (kMaxCells + 31) / 32;
      float pq[kChunks];
      const float* prow = pol + (size_t)q * v.A;
#pragma unroll
      for (int t = 0; t < kChunks; ++t) {         // the leaf's policy row: independent loads
        const int c = lane + 32 * t;
        pq[t] = c < v.C ? prow[c] : 0.0f;
      }
      const int16_t* P = gpath + (size_t)i * kMaxDepthCap;
      const int d = P[kMaxDepthCap - 1];
      if (d < 0) { if (lane == 0) H->status = OMQ_BAD_ARG; continue; }
      // the leaf's position as bit rows (lane y) and flat occupancy words (lane w): the root's plus
      // the path's stones, black and white alternating from the root's side to move
      // (y = a / S by a multiply-shift: floor(a * (2^16 / S + 1) / 2^16) is exact for a < 361 and
      // S <= 19, the error term a / 2^16 staying below 1 / S)
      uint32_t p1 = s_rows[0][lane], p2 = s_rows[1][lane];
      uint32_t occw = lane < (kMaxCells + 31) / 32 ? s_occ[lane] : 0u;
      const uint32_t rdiv = 65536u / (uint32_t)v.S + 1u;
      for (int j = 0; j < d; ++j) {
        const int a = P[j];
        const int y = (int)(((uint32_t)a * rdiv) >> 16), x = a - y * v.S;
        const bool black = ((j % 2 == 0) ? H->root_player : 3 - H->root_player) == 1;
        if (lane == y) { if (black) p1 |= 1u << x; else p2 |= 1u << x; }
        if (lane == (a >> 5)) occw |= 1u << (a & 31);
      }
      const int player = (d % 2 == 0) ? H->root_player : 3 - H->root_player;
      const int mc = H->root_mc + d;
      warp_five_masks(player == 1 ? p1 : p2, p1 | p2, v.S, W.five);
      const bool root_five = H->root_five != 0;
      // legal actions in ascending order and their policy values: cell c = lane + 32 t is word t
      // of the occupancy, bit lane
      int n = 0;
#pragma unroll
      for (int t = 0; t < kChunks; ++t) {
        const int c = lane + 32 * t;
        const int rem = v.C - 32 * t;
        const uint32_t valid = rem >= 32 ? 0xFFFFFFFFu : (rem > 0 ? (1u << rem) - 1u : 0u);
        const unsigned m = ~__shfl_sync(0xFFFFFFFFu, occw, t) & valid;
        const bool legal = (m >> lane) & 1u;
        if (legal) {
          const int j = n + __popc(m & ((1u << lane) - 1));
          W.legal[j] = (int16_t)c;
          W.pv[j] = pq[t];
        }
        n += __popc(m);
      }
      __syncwarp();
      const float denom = __fadd_rn(warp_torch_sum(W.pv, n), 1e-8f);
      const int start = num_nodes + s_cnt[i];
      unsigned long long best = 0;
      const float sq_leaf = parent_sqrt(v.stats[base + e.node].N);
      for (int j = lane; j < n; j += 32) {
        const int a = W.legal[j];
        const float P = __fdiv_rn(W.pv[j], denom);
        const bool term = root_five || ((W.five[32 + (a >> 5)] >> (a & 31)) & 1u) || (mc + 1 >= v.C);
        const int c = start + j;
        const NodeStats st{0, 0.0f, P, 0};
        v.stats[base + c] = st;
        v.topo[base + c] = NodeTopo{e.node, pack_act_depth(a, d + 1), 0,
                                    pack_cnt_flags(0, term ? kFlagTerminal : 0)};
        const unsigned long long key =
            rank_key(ucb_score_sq(st, sq_leaf, v.c_puct, v.vl_value, v.enable_vl), j);
        best = key > best ? key : best;
      }
      best = warp_max_u64(best);
      if (lane == 0) {
        NodeTopo lt = v.topo[base + e.node];
        lt.child_start = start;
        lt.cnt_flags = pack_cnt_flags(n, topo_flags(lt));
        v.topo[base + e.node] = lt;
      }
      if (!root_mode && n > 0) {
        // child pick on the fresh children (wave_search.py:1053-1077): first maximum
        final_node = start + key_slot(best);
        ext = (e.depth + 1 < v.max_depth) ? 1 : 0;
        if (lane == 0 && v.enable_vl) v.stats[base + final_node].VL += 1;
      }
    } else if (!root_mode) {
      const NodeTopo tp = v.topo[base + e.node];
      const int n = topo_count(tp);
      if (n > 0) {  // depth-limited leaf that already has children
        const int32_t np = v.stats[base + e.node].N;
        unsigned long long best = 0;
        for (int j = lane; j < n; j += 32) {
          const NodeStats st = v.stats[base + tp.child_start + j];
          const unsigned long long key =
              rank_key(ucb_score(st, np, v.c_puct, v.vl_value, v.enable_vl), j);
          best = key > best ? key : best;
        }
        best = warp_max_u64(best);
        final_node = tp.child_start + key_slot(best);
        ext = (e.depth + 1 < v.max_depth) ? 1 : 0;
        if (lane == 0 && v.enable_vl) v.stats[base + final_node].VL += 1;
      }
    }
    if (lane == 0) lf[i] = make_int2(final_node, ext << 30);
    __syncwarp();
  }
  if (slices > 1) return;  // k_expand_commit finishes the sliced expansion
  __syncthreads();
  if (tid == 0) {
    H->num_nodes = num_nodes + total;
    if (!root_mode) {
      s_fbase = atomicAdd(&v.q_count[1], nleaf);
      H->fin_off = s_fbase;
      H->fin_cnt = nleaf;
    }
  }
  __syncthreads();
  if (!root_mode) {
    for (int i = tid; i < nleaf; i += blockDim.x) {
      const int2 x = lf[i];
      v.q_entries[1][s_fbase + i] = make_int2(r, x.x);
      lf[i] = make_int2(x.x, (s_fbase + i) | (x.y & (1 << 30)));
    }
  }
}

// The end of a sliced k_expand: the tree's node count and its final-node queue entries (the
// single-CTA k_expand does this itself).
__global__ void k_expand_commit(EngineView v, int root_mode) {
  const int r = blockIdx.x, tid = threadIdx.x;
  TreeHeader* H = &v.hdr[r];
  if (H->status != OMQ_OK) return;
  const int nleaf = H->nleaves;
  int2* lf = v.leaf_final + (size_t)r * v.WCAP;
  __shared__ int s_fbase;
  if (tid == 0) {
    H->num_nodes += H->exp_total;
    H->exp_total = 0;
    if (!root_mode) {
      s_fbase = atomicAdd(&v.q_count[1], nleaf);
      H->fin_off = s_fbase;
      H->fin_cnt = nleaf;
    }
  }
  __syncthreads();
  if (!root_mode) {
    for (int i = tid; i < nleaf; i += blockDim.x) {
      const int2 x = lf[i];
      v.q_entries[1][s_fbase + i] = make_int2(r, x.x);
      lf[i] = make_int2(x.x, (s_fbase + i) | (x.y & (1 << 30)));
    }
  }
}

// ---------------------------------------------------------------------------------------------
// backup + virtual-loss revert
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void backup_node(const EngineView& v, size_t base, const float* sv,
                                            const Visit& x) {
  NodeStats st = v.stats[base + x.node];
  st.N += x.k;
  float w = st.W;
  const bool even = (x.depth % 2) == 0;
  for (int s = x.lo; s < x.lo + x.k; ++s) {
    const float val = sv[s];
    w = __fadd_rn(w, even ? val : -val);
  }
  st.W = w;
  if (x.depth >= 1 && v.enable_vl) st.VL = max(st.VL - x.k, 0);
  v.stats[base + x.node] = st;
}

__global__ void __launch_bounds__(kThreads) k_backup(EngineView v) {
  const int r = blockIdx.x, tid = threadIdx.x;
  TreeHeader* H = &v.hdr[r];
  if (H->status != OMQ_OK) return;
  const size_t base = (size_t)r * v.T;
  const int nleaf = H->nleaves, nlog = H->nlog;
  const Visit* leaves = v.leaves + (size_t)r * v.WCAP;
  const int2* lf = v.leaf_final + (size_t)r * v.WCAP;
  float* sv = v.simval + (size_t)r * v.WCAP;
  for (int i = tid; i < nleaf; i += blockDim.x) {
    const Visit e = leaves[i];
    const float val = v.q_value[1][lf[i].y & ((1 << 30) - 1)];
    for (int s = e.lo; s < e.lo + e.k; ++s) sv[s] = val;
  }
  __syncthreads();
  const Visit* log = v.vlog + (size_t)r * v.LOGCAP;
  for (int i = tid; i < nlog; i += blockDim.x) backup_node(v, base, sv, log[i]);
  for (int i = tid; i < nleaf; i += blockDim.x) {
    if (lf[i].y & (1 << 30)) {
      const Visit e = leaves[i];
      backup_node(v, base, sv, Visit{lf[i].x, e.lo, e.k, e.depth + 1});
    }
  }
}

// ---------------------------------------------------------------------------------------------
// readouts
// ---------------------------------------------------------------------------------------------
__global__ void k_root_visits(EngineView v, int32_t* visits, float* nw) {
  const int r = blockIdx.x, tid = threadIdx.x;
  const size_t base = (size_t)r * v.T;
  for (int a = tid; a < v.A; a += blockDim.x) visits[(size_t)r * v.A + a] = 0;
  __syncthreads();
  const NodeTopo t = v.topo[base];
  const int n = topo_count(t);
  for (int j = tid; j < n; j += blockDim.x) {
    const int c = t.child_start + j;
    visits[(size_t)r * v.A + topo_action(v.topo[base + c])] = v.stats[base + c].N;
  }
  if (tid == 0 && nw) {
    nw[2 * r] = (float)v.stats[base].N;
    nw[2 * r + 1] = v.stats[base].W;
  }
}

__global__ void k_export(EngineView v, int tree, int count, int32_t* N, float* W, float* P,
                         int32_t* VL, int32_t* parent, int32_t* action, uint8_t* terminal) {
  const size_t base = (size_t)tree * v.T;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
    const NodeStats s = v.stats[base + i];
    const NodeTopo t = v.topo[base + i];
    if (N) N[i] = s.N;
    if (W) W[i] = s.W;
    if (P) P[i] = s.P;
    if (VL) VL[i] = s.VL;
    if (parent) parent[i] = t.parent;
    if (action) action[i] = topo_action(t);
    if (terminal) terminal[i] = (topo_flags(t) & kFlagTerminal) ? 1 : 0;
  }
}

__global__ void k_status(EngineView v, int32_t* status, int32_t* num_nodes) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < v.R) {
    if (status) status[r] = v.hdr[r].status;
    if (num_nodes) num_nodes[r] = v.hdr[r].num_nodes;
  }
}

// ---------------------------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------------------------
// SMs of the device (every device of the pool is the same part)
static int device_sms() {
  static std::atomic<int> sms{0};
  int n = sms.load(std::memory_order_relaxed);
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    sms.store(n, std::memory_order_relaxed);
  }
  return n;
}

static int tree_threads(const EngineView& v) {
  const int sms = device_sms();
  return v.R >= 2 * sms ? 256 : kThreads;
}

static size_t select_smem(const EngineView& v) {
  int p2 = 1;
  while (p2 < v.max_children) p2 <<= 1;
  return ((sizeof(SelectShared) + 15) & ~(size_t)15) + (size_t)(tree_threads(v) / 32) * p2 * 8 +
         (size_t)v.WCAP * sizeof(Visit) + (size_t)v.WCAP * sizeof(int);
}

void launch_begin(const EngineView& v, const int8_t* boards, int search_id, cudaStream_t s) {
  count_launches(1);
  k_begin<<<v.R, tree_threads(v), 0, s>>>(v, boards, search_id);
}

void launch_begin_chess(const EngineView& v, const void* records, const int32_t* nprior, int search_id,
                        cudaStream_t s) {
  count_launches(1);
  k_begin_chess<<<v.R, 256, 0, s>>>(v, reinterpret_cast<const ChessRec*>(records), nprior, search_id);
}

void launch_begin_go(const EngineView& v, const int8_t* history, const int32_t* meta,
                     const uint64_t* keys, const int32_t* nkeys, int search_id, cudaStream_t s) {
  count_launches(1);
  k_begin_go<<<v.R, 256, 0, s>>>(v, history, meta, keys, nkeys, search_id);
}

void launch_select(const EngineView& v, int wave, cudaStream_t s) {
  const size_t sm = select_smem(v);
  if (sm > 48 * 1024)
    cudaFuncSetAttribute(k_select, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  cudaMemsetAsync(v.q_count, 0, sizeof(int32_t), s);
  if (v.slices > 1) cudaMemsetAsync(v.sel_ctr, 0, (size_t)v.R * 4 * sizeof(int32_t), s);
  count_launches(1);
  k_select<<<dim3(v.R, v.slices), tree_threads(v), sm, s>>>(v, wave);
  if (v.slices > 1) {
    const int csm = (int)((size_t)v.WCAP * (sizeof(Visit) + sizeof(int)));
    if (csm > 48 * 1024) cudaFuncSetAttribute(k_select_commit, cudaFuncAttributeMaxDynamicSharedMemorySize, csm);
    count_launches(1);
    k_select_commit<<<v.R, tree_threads(v), csm, s>>>(v, wave);
  }
}

void launch_expand(const EngineView& v, int root_mode, cudaStream_t s) {
  if (!root_mode) cudaMemsetAsync(v.q_count + 1, 0, sizeof(int32_t), s);
  count_launches(1);
  const size_t extra = v.game == OMQ_GAME_GO ? sizeof(GoPos)
                       : v.game == OMQ_GAME_CHESS ? sizeof(ChessWarpSmem) : 0;
  // Go's per-warp scratch (board analysis with group keys) allows 16 warps per tree
  const int threads = v.game == OMQ_GAME_GO ? min(tree_threads(v), 512) : tree_threads(v);
  const int sm = (int)((threads / 32) * (sizeof(ExpandWarpSmem) + extra));
  cudaFuncSetAttribute(k_expand, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
  // few Gomoku trees: several CTAs (SMs) per tree, one leaf per warp at a full wave
  const int slices = v.game == OMQ_GAME_GOMOKU
                         ? max(1, min(v.slices, (v.WCAP + threads / 32 - 1) / (threads / 32)))
                         : 1;
  k_expand<<<dim3(v.R, slices), threads, sm, s>>>(v, root_mode);
  if (slices > 1) {
    count_launches(1);
    k_expand_commit<<<v.R, 256, 0, s>>>(v, root_mode);
  }
}

void launch_backup(const EngineView& v, cudaStream_t s) {
  count_launches(1);
  k_backup<<<v.R, tree_threads(v), 0, s>>>(v);
}

void launch_root_visits(const EngineView& v, int32_t* visits, float* nw, cudaStream_t s) {
  count_launches(1);
  k_root_visits<<<v.R, 256, 0, s>>>(v, visits, nw);
}

void launch_export(const EngineView& v, int tree, int count, int32_t* N, float* W, float* P,
                   int32_t* VL, int32_t* parent, int32_t* action, uint8_t* terminal,
                   cudaStream_t s) {
  const int blocks = max(1, min(1024, (count + 255) / 256));
  count_launches(1);
  k_export<<<blocks, 256, 0, s>>>(v, tree, count, N, W, P, VL, parent, action, terminal);
}

void launch_status(const EngineView& v, int32_t* status, int32_t* num_nodes, cudaStream_t s) {
  count_launches(1);
  k_status<<<(v.R + 255) / 256, 256, 0, s>>>(v, status, num_nodes);
}

// Self-test of the prior-normalisation sum: one warp per segment [offsets[s], offsets[s+1]) of x.
__global__ void k_selftest_prior_sum(const float* x, const int32_t* offsets, int segments, float* out) {
  const int seg = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (seg >= segments) return;
  const int lo = offsets[seg], n = offsets[seg + 1] - lo;
  const float r = warp_torch_sum(x + lo, n);
  if ((threadIdx.x & 31) == 0) out[seg] = r;
}

void launch_selftest_prior_sum(const float* x, const int32_t* offsets, int segments, float* out,
                               cudaStream_t s) {
  count_launches(1);
  k_selftest_prior_sum<<<(segments + 7) / 8, 256, 0, s>>>(x, offsets, segments, out);
}

}  // namespace omq
