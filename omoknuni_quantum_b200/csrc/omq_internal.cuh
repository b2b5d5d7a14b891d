// Internal definitions shared by the engine's CUDA translation units.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "omq_b200.h"

namespace omq {

// 16-bit storage of the ResNet's weights and activations: bf16 (OMQ_DTYPE_BF16) or fp16
// (OMQ_DTYPE_F16, the reference evaluator's autocast precision); the same bits feed tcgen05
// kind::f16. Conversions round to nearest even.
using h16 = uint16_t;

template <bool F16>
__device__ __forceinline__ uint32_t pack2_h16(float a, float b) {
  if constexpr (F16) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}
template <bool F16>
__device__ __forceinline__ float2 unpack2_h16(uint32_t u) {
  if constexpr (F16) return __half22float2(*reinterpret_cast<const __half2*>(&u));
  else return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}
__device__ __forceinline__ h16 to_h16(float a, bool f16) {
  return f16 ? __half_as_ushort(__float2half_rn(a)) : __bfloat16_as_ushort(__float2bfloat16_rn(a));
}
__device__ __forceinline__ float from_h16(h16 a, bool f16) {
  return f16 ? __half2float(__ushort_as_half(a)) : __bfloat162float(__ushort_as_bfloat16(a));
}

// Per-node statistics, one 16-byte vector load per child during selection.
// Fields mirror NodeDataManager's SoA arrays (python/mcts/gpu/node_data_manager.py:88-113):
// visit_counts (int32), value_sums (fp32), node_priors (fp32), virtual_loss_counts (int32).
struct __align__(16) NodeStats {
  int32_t N;
  float W;
  float P;
  int32_t VL;
};

// Per-node topology. Children of a node occupy the contiguous id range
// [child_start, child_start + count) in ascending action order, which is exactly the layout the
// reference produces (child ids assigned consecutively in action order, csr_tree.py:391-449), so
// the reference's dense children[node, action] table is implied and need not be stored.
struct __align__(16) NodeTopo {
  int32_t parent;       // -1 for the root (reference parent_indices; -2 = unused slot)
  int32_t act_depth;    // action (low 16 bits, signed) | depth (high 16 bits)
  int32_t child_start;
  int32_t cnt_flags;    // child count (low 16 bits) | flags (high 16 bits)
};

constexpr int kFlagTerminal = 1;

__host__ __device__ inline int topo_action(const NodeTopo& t) { return (int)(int16_t)(t.act_depth & 0xFFFF); }
__host__ __device__ inline int topo_depth(const NodeTopo& t) { return (t.act_depth >> 16) & 0xFFFF; }
__host__ __device__ inline int topo_count(const NodeTopo& t) { return t.cnt_flags & 0xFFFF; }
__host__ __device__ inline int topo_flags(const NodeTopo& t) { return (t.cnt_flags >> 16) & 0xFFFF; }
__host__ __device__ inline int pack_act_depth(int a, int d) { return (a & 0xFFFF) | (d << 16); }
__host__ __device__ inline int pack_cnt_flags(int c, int f) { return (c & 0xFFFF) | (f << 16); }

// One (node, simulation range, depth) record. Simulations reaching a node in a wave always form
// a contiguous index range [lo, lo + k): the reference hands the simulations at a parent (in
// ascending index) to its UCB-sorted children in rank order (wave_search.py:1300-1319).
struct __align__(16) Visit {
  int32_t node;
  int32_t lo;
  int32_t k;
  int32_t depth;
};

struct TreeHeader {
  int32_t num_nodes;
  int32_t status;
  int32_t root_player;
  int32_t root_mc;
  int32_t root_five;
  int32_t nleaves;
  int32_t nlog;
  int32_t exp_off;
  int32_t exp_cnt;
  int32_t fin_off;
  int32_t fin_cnt;
  int32_t wave;
  int32_t wave_idx;      // waves run in the current search (root-noise counter)
  int32_t search_idx;    // searches begun on this engine (root-noise counter)
  int32_t root_ko;       // Go: ko point of the root position (-1 none)
  int32_t root_passes;   // Go: consecutive passes that led to the root position
  int32_t root_prior;    // chess: earlier game positions stored with the root
  int32_t root_nkeys;    // Go: superko keys of the root's game (sorted in go_keys)
  // set by omq_reroot, consumed by the next begin: 0 fresh tree; 1 fresh tree whose root starts
  // with (carry_n, carry_w); 2 nodes [0, num_nodes) are the kept subtree of the new root
  int32_t kept;
  int32_t carry_n;
  float carry_w;
  int32_t exp_total;     // children created by the expansion in flight (sliced k_expand)
};

constexpr int kPlanes = 19;
constexpr int kFullHistoryGomoku = 250;
constexpr int kMaxCells = 361;
constexpr int kMaxWords = 6;  // ceil(361 / 64)

// Device-side view of one engine, passed by value to kernels.
struct EngineView {
  int game;              // OMQ_GAME_GOMOKU or OMQ_GAME_GO
  int R, T, S, C, A, WCAP, LOGCAP, max_depth, enable_vl;
  float c_puct, vl_value;
  float noise_alpha, noise_eps, noise_keep;  // keep = (float)(1 - (double)eps), as the reference rounds it
  uint64_t noise_seed;
  float* root_noise;     // [R][A] noise of the last wave, by action
  NodeStats* stats;      // [R*T]
  NodeTopo* topo;        // [R*T]
  int8_t* root_board;    // Gomoku [R][C]; Go [R][8][C] (root position and 7 earlier ones);
                         // chess [R][1 + 100] position records (root, then earlier positions)
  uint32_t* go_mask;     // per-leaf legal bits: Go [R][WCAP][32] (12 words, the leaf's passes at 12,
                         // 12 words of repetition-terminal child bits from 16),
                         // chess [R][WCAP][148]
  uint64_t* chess_prior_hash;  // chess: [R][100] placement hashes of the earlier positions
  int go_superko;              // Go: positional superko on
  int go_cycle;                // Go: third repetition (board, ko, side to move) ends the game
  uint64_t* go_keys;           // Go: [R][OMQ_GO_MAX_KEYS] the root game's position keys, sorted
  uint32_t* go_bloom;          // Go: [R][128] 4096-bit filter of those keys (key & 4095)
  int max_children;      // most children a node can have (sizes the selection sort)
  int16_t* leaf_paths;   // Gomoku: [R][WCAP][128] actions root -> leaf of each expandable leaf
                         // (slot 127: its depth), written and read by k_expand
  TreeHeader* hdr;       // [R]
  Visit* frontier;       // [R][2][WCAP]
  Visit* vlog;           // [R][LOGCAP]
  Visit* leaves;         // [R][WCAP]  (sorted ascending by node after selection)
  int2* leaf_final;      // [R][WCAP]  {final node, final-queue index | extended << 30}
  float* simval;         // [R][WCAP]
  int2* q_entries[2];    // [R*WCAP] {tree, node}
  float* q_policy[2];    // [R*WCAP][A]
  float* q_value[2];     // [R*WCAP]
  int32_t* q_count;      // [2]
  int slices;            // CTAs per tree of k_select (and of the Gomoku k_expand) when trees are few
  int32_t* sel_ctr;      // [R][4] sliced k_select: visit-log entries, leaves, overflow, 0
};

// UCB score of a child exactly as the reference evaluates it in fp32
// (wave_search.py:1287-1296 selection, :1059-1072 child pick; node_data_manager.py:379-390):
//   Ne = float(N + VL); We = W + float(VL) * (-|vl|); Q = We / Ne if Ne > 0 else 0;
//   U = ((c * P) * sqrt(max(float(N_parent), 1))) / (1 + Ne); score = Q + U
// Every operation is an explicitly rounded intrinsic so no contraction can change the result.
// The same with sq = sqrt(max(N_parent, 1)) computed once per parent. A child with N + VL = 0
// has Q = 0 and U = c*P*sq / 1, and the IEEE division by 1 is exact, so its score is c*P*sq
// without a divide.
__device__ __forceinline__ float ucb_score_sq(const NodeStats& s, float sq, float c_puct,
                                              float vl_value, int enable_vl) {
  const int32_t vl = enable_vl ? s.VL : 0;
  const float cps = __fmul_rn(__fmul_rn(c_puct, s.P), sq);
  if (s.N + vl == 0) return __fadd_rn(0.0f, cps);
  const float ne = __int2float_rn(s.N + vl);
  const float we = enable_vl ? __fadd_rn(s.W, __fmul_rn(__int2float_rn(s.VL), vl_value)) : s.W;
  const float q = ne > 0.0f ? __fdiv_rn(we, ne) : 0.0f;
  const float u = __fdiv_rn(cps, __fadd_rn(1.0f, ne));
  return __fadd_rn(q, u);
}

__device__ __forceinline__ float parent_sqrt(int32_t n_parent) {
  return __fsqrt_rn(fmaxf(__int2float_rn(n_parent), 1.0f));
}

__device__ __forceinline__ float ucb_score(const NodeStats& s, int32_t n_parent, float c_puct,
                                           float vl_value, int enable_vl) {
  return ucb_score_sq(s, parent_sqrt(n_parent), c_puct, vl_value, enable_vl);
}

// Order-preserving 32-bit image of a float (total order; +0 and -0 mapped together).
__device__ __forceinline__ uint32_t float_order(float f) {
  if (f == 0.0f) f = 0.0f;
  uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Sort key: score descending, then child slot ascending (the deterministic tie rule).
__device__ __forceinline__ unsigned long long rank_key(float score, int slot) {
  return ((unsigned long long)float_order(score) << 32) | (0xFFFFFFFFu - (uint32_t)slot);
}
__device__ __forceinline__ int key_slot(unsigned long long key) {
  return (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
}

__device__ __forceinline__ uint64_t mix64(uint64_t x) {  // SplitMix64 finaliser
  x ^= x >> 30; x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 27; x *= 0x94D049BB133111EBull;
  x ^= x >> 31;
  return x;
}

// Walk from `node` to the root collecting the actions on the path into acts[0..depth-1]
// (root-to-node order). Returns the node's depth. A hard bound guards against a corrupted
// parent chain: on violation the walk stops and -1 is returned.
__device__ __forceinline__ int path_actions(const NodeTopo* topo, int node, int max_depth,
                                            int16_t* acts) {
  const NodeTopo t0 = topo[node];
  const int d = topo_depth(t0);
  if (d >= max_depth + 1) return -1;
  int cur = node;
  for (int i = d - 1; i >= 0; --i) {
    const NodeTopo t = topo[cur];
    acts[i] = (int16_t)topo_action(t);
    cur = t.parent;
    if (cur < 0) return -1;
  }
  return d;
}

}  // namespace omq

struct omq_engine {
  omq_engine_config cfg;
  omq::EngineView v;
  int32_t wave;          // wave size of the wave in flight
  int32_t phase;         // 0 idle, 1 begun, 2 root expanded, 3 selected, 4 expanded
  int32_t searches;      // omq_begin calls so far
  uint64_t bytes;
  void* arena;           // single device allocation backing every buffer
  void* reroot_scratch;  // omq_reroot mode 2: node copies for reroot_chunk trees (lazy)
  int32_t reroot_chunk;
};

namespace omq {
// Makes `dev` current for the lifetime of the guard, restoring the caller's device after.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    // an invalid ordinal leaves the device unchanged; the caller's own checks report it, and the
    // failed call's error is cleared so that a later cudaGetLastError does not pick it up
    if (prev != dev && cudaSetDevice(dev) != cudaSuccess) cudaGetLastError();
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

void set_error(const char* fmt, ...);
// Process-wide count of kernels this library has launched (reported by omq_kernel_launches).
void count_launches(int n);
int cuda_status(cudaError_t e, const char* what);

void launch_begin(const EngineView& v, const int8_t* boards, int search_id, cudaStream_t s);
void launch_begin_chess(const EngineView& v, const void* records, const int32_t* nprior, int search_id,
                        cudaStream_t s);
void launch_begin_go(const EngineView& v, const int8_t* history, const int32_t* meta,
                     const uint64_t* keys, const int32_t* nkeys, int search_id, cudaStream_t s);
void launch_select(const EngineView& v, int wave, cudaStream_t s);
void launch_reroot(const EngineView& v, const int32_t* actions, int mode, NodeStats* scratch_stats,
                   NodeTopo* scratch_topo, int chunk, cudaStream_t s);
void launch_expand(const EngineView& v, int root_mode, cudaStream_t s);
void launch_backup(const EngineView& v, cudaStream_t s);
void launch_root_visits(const EngineView& v, int32_t* visits, float* nw, cudaStream_t s);
void launch_export(const EngineView& v, int tree, int count, int32_t* N, float* W, float* P,
                   int32_t* VL, int32_t* parent, int32_t* action, uint8_t* terminal, cudaStream_t s);
void launch_status(const EngineView& v, int32_t* status, int32_t* num_nodes, cudaStream_t s);
void launch_selftest_prior_sum(const float* x, const int32_t* offsets, int segments, float* out,
                               cudaStream_t s);
void launch_features(const EngineView& v, int queue, float* out, cudaStream_t s);
void launch_synth_eval(const EngineView& v, int queue, cudaStream_t s);
// queue positions -> bf16 [count][P][in_pad] padded pixel layout (ResNet input)
void launch_pack_queue(const EngineView& v, int queue, int P, int in_pad, void* out, bool f16, cudaStream_t s);
// feature planes of the engine's game (19 Gomoku, 17 Go)
inline int engine_planes(const EngineView& v) {
  return v.game == OMQ_GAME_GO ? 17 : v.game == OMQ_GAME_CHESS ? 119 : 19;
}
}  // namespace omq
