// Leaf-queue evaluation kernels: the reference feature tensor and the built-in synthetic
// evaluator.
//
// Positions are never stored per node. A queued node's board is rebuilt from its tree's root
// board plus the actions on its parent chain (at most max_depth dependent loads), which is all
// the reference's features carry: occupancy, the side to move, and the last move (child states
// do not inherit full_move_history, python/mcts/gpu/gpu_game_states.py:325-327, 443-446).
#include <cuda_bf16.h>

#include "chess_device.cuh"
#include "go_device.cuh"
#include "omq_internal.cuh"

namespace omq {

constexpr int kEvalDepthCap = 128;

// Planes of the reference's 8-move history block (gpu_game_states.py:560-600) that hold this
// state's single recorded move, as a bitmask over the 19 planes. A state made by apply_moves
// records only its own move at index move_count-1; the clamp of :568 makes that entry reappear
// for k >= 1 when move_count == 1.
__device__ __forceinline__ uint32_t history_planes(int mc, int depth, int full_history) {
  uint32_t m = 0;
  if (depth < 1) return 0;
  for (int k = 0; k < 8; ++k) {
    int idx = mc - 1 - k;
    idx = idx < 0 ? 0 : idx;
    idx = idx > full_history - 1 ? full_history - 1 : idx;
    if (idx < mc && idx == mc - 1) m |= 1u << ((k % 2 == 0) ? 2 + k / 2 : 10 + k / 2);
  }
  return m;
}

struct WarpPos {
  int16_t acts[kEvalDepthCap];
  int8_t board[kMaxCells + 3];
  uint64_t words[kMaxWords];
};

// Rebuild the board of `node` of tree r into wp.board. Returns depth (or -1 on a bad chain).
__device__ int warp_rebuild(const EngineView& v, int r, int node, WarpPos& wp) {
  const int lane = threadIdx.x & 31;
  int d = 0;
  if (lane == 0) d = path_actions(v.topo + (size_t)r * v.T, node, kEvalDepthCap - 1, wp.acts);
  d = __shfl_sync(0xFFFFFFFFu, d, 0);
  if (d < 0) return -1;
  const TreeHeader& H = v.hdr[r];
  for (int c = lane; c < v.C; c += 32) wp.board[c] = v.root_board[(size_t)r * v.C + c];
  __syncwarp();
  for (int j = lane; j < d; j += 32)
    wp.board[wp.acts[j]] = (int8_t)((j % 2 == 0) ? H.root_player : 3 - H.root_player);
  __syncwarp();
  return d;
}

__device__ __forceinline__ int64_t exp_step(uint64_t r) {
  const int64_t s = (int64_t)(r & 0xFFFF) + (int64_t)((r >> 16) & 0xFFFF) +
                    (int64_t)((r >> 32) & 0xFFFF) + (int64_t)((r >> 48) & 0xFFFF) - 131072;
  return (s * 160) >> 16;
}

// In global memory, read through the read-only cache: lanes index it with different values,
// which the constant cache would serialise.
__device__ const uint32_t c_exp2[64] = {
    1048576u,1059994u,1071537u,1083205u,1095000u,1106924u,1118978u,1131163u,1143480u,1155932u,
    1168519u,1181244u,1194106u,1207109u,1220254u,1233542u,1246974u,1260553u,1274279u,1288155u,
    1302182u,1316362u,1330696u,1345187u,1359835u,1374642u,1389611u,1404743u,1420040u,1435503u,
    1451135u,1466937u,1482910u,1499058u,1515382u,1531883u,1548564u,1565427u,1582474u,1599706u,
    1617125u,1634735u,1652536u,1670531u,1688722u,1707110u,1725700u,1744491u,1763488u,1782691u,
    1802103u,1821727u,1841564u,1861617u,1881889u,1902381u,1923097u,1944038u,1965207u,1986607u,
    2008240u,2030108u,2052214u,2074562u};

// floor(n / d) for 0 < d and n < 2^53: an fp64 estimate from rd = 1.0 / d (relative error a few
// ulps, so at most one off for quotients below 2^20), corrected by integer products - the same
// quotient as the integer division, without a 64-bit divide per action.
__device__ __forceinline__ uint64_t div_floor53(uint64_t n, uint64_t d, double rd) {
  uint64_t q = (uint64_t)__dmul_rn((double)n, rd);
  if (q * d > n) --q;
  else if ((q + 1) * d <= n) ++q;
  return q;
}

__device__ __forceinline__ uint64_t exp2_fixed(int64_t t) {
  return (uint64_t)__ldg(&c_exp2[t & 63]) << ((t >> 6) + 6);
}

// Built-in synthetic evaluator (integer-exact definition: policy on a 2^-24 grid with distinct
// legal priors, value tanh(z/2) on a 2^-12 grid), keyed by a 64-bit hash of the reference feature
// planes of the position. One warp per queued position.
constexpr int kSynthWarps = 4;
constexpr int kMaxActionsPerLane = 12;  // ceil(362 / 32)

// Policy (queue 0) and value of queue entry q from the position hash h; legal = empty points of
// `board` plus any action past the board (Go pass). Warp-collective.
template <class Occupied>
__device__ void synth_emit(const EngineView& v, int queue, int q, uint64_t h, const Occupied& occupied) {
  const int lane = threadIdx.x & 31;
  if (queue == 0) {
    uint64_t wv[kMaxActionsPerLane];
    uint64_t tot = 0;
#pragma unroll
    for (int t = 0; t < kMaxActionsPerLane; ++t) {
      const int a = t * 32 + lane;
      wv[t] = 0;
      if (a < v.A && (a >= v.C || !occupied(a))) {
        wv[t] = exp2_fixed(exp_step(mix64(h + 0x9E3779B97F4A7C15ull * (uint64_t)(a + 1))));
        tot += wv[t];
      }
    }
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xFFFFFFFFu, tot, o);
    const double rtot = tot ? 1.0 / (double)tot : 0.0;
    int idx_base = 0;
    float* out = v.q_policy[0] + (size_t)q * v.A;
#pragma unroll
    for (int t = 0; t < kMaxActionsPerLane; ++t) {
      const int a = t * 32 + lane;
      const bool legal = a < v.A && (a >= v.C || !occupied(a));
      const unsigned m = __ballot_sync(0xFFFFFFFFu, legal);
      if (a < v.A) {
        float p = 0.0f;
        if (legal) {
          const uint64_t idx = (uint64_t)(idx_base + __popc(m & ((1u << lane) - 1)));
          const uint64_t qa = 512ull * div_floor53(wv[t] * 32640ull, tot, rtot) + idx;
          p = __fmul_rn(__ull2float_rn(qa), 1.0f / 16777216.0f);
        }
        out[a] = p;
      }
      idx_base += __popc(m);
    }
  }
  if (lane == 0) {
    const int64_t e = (int64_t)exp2_fixed(exp_step(mix64(h ^ 0xD1B54A32D192ED03ull)));
    const int64_t dd = (int64_t)1 << 26;
    const int64_t val = ((e - dd) * 4096) / (e + dd);
    v.q_value[queue][q] = __fmul_rn(__ll2float_rn(val), 1.0f / 4096.0f);
  }
}

// Positions per warp in k_synth (at most): the boards are rebuilt one after another by the whole
// warp, then lane i runs position i's hash chain (a serial chain per position), then the policies
// are emitted one position at a time. Small queues take fewer per warp (`group`), so that more
// warps share the work; every position's result is the same either way.
constexpr int kSynthGroup = 8;

__global__ void __launch_bounds__(kSynthWarps * 32) k_synth(EngineView v, int queue, int group) {
  __shared__ WarpPos wps[kSynthWarps];
  __shared__ uint64_t gwords[kSynthWarps][kSynthGroup][kMaxWords];  // occupancy bit boards
  __shared__ int gmeta[kSynthWarps][kSynthGroup][4];                 // player, move count, depth, last
  __shared__ uint64_t ghash[kSynthWarps][kSynthGroup];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int q0 = (blockIdx.x * kSynthWarps + wl) * group;
  const int count = v.q_count[queue];
  if (q0 >= count) return;
  const int ng = min(group, count - q0);
  WarpPos& wp = wps[wl];
  const int nwords = (v.C + 63) / 64;
  for (int i = 0; i < ng; ++i) {
    const int2 ent = v.q_entries[queue][q0 + i];
    const int r = ent.x;
    const int d = warp_rebuild(v, r, ent.y, wp);
    if (d < 0) {
      if (lane == 0) { v.hdr[r].status = OMQ_BAD_ARG; gmeta[wl][i][2] = -1; }
      __syncwarp();
      continue;
    }
    // occupancy words: bit b of word j is cell 64 j + b
    for (int c0 = 0, k = 0; c0 < v.C; c0 += 32, ++k) {
      const unsigned m = __ballot_sync(0xFFFFFFFFu, c0 + lane < v.C && wp.board[c0 + lane] != 0);
      if (lane == 0) {
        if (k & 1) gwords[wl][i][k >> 1] |= (uint64_t)m << 32;
        else gwords[wl][i][k >> 1] = m;
      }
    }
    if (lane == 0) {
      const TreeHeader& H = v.hdr[r];
      gmeta[wl][i][0] = (d % 2 == 0) ? H.root_player : 3 - H.root_player;
      gmeta[wl][i][1] = H.root_mc + d;
      gmeta[wl][i][2] = d;
      gmeta[wl][i][3] = d >= 1 ? wp.acts[d - 1] : -1;
    }
    __syncwarp();
  }
  // the hash of the reference feature planes, one chain per lane
  if (lane < ng && gmeta[wl][lane][2] >= 0) {
    const uint64_t* w = gwords[wl][lane];
    const int player = gmeta[wl][lane][0], mc = gmeta[wl][lane][1], d = gmeta[wl][lane][2];
    const int last = gmeta[wl][lane][3];
    uint64_t h = 0x243F6A8885A308D3ull;
    for (int j = 0; j < nwords; ++j) h = mix64(h ^ w[j]);
    h = mix64(h ^ (uint64_t)player);
    const uint32_t hp = history_planes(mc, d, kFullHistoryGomoku);
    for (int c = 2; c < kPlanes; ++c)
      for (int j = 0; j < nwords; ++j) {
        uint64_t word = 0;
        if ((hp >> c) & 1u) {
          if (last >= 64 * j && last < 64 * j + 64) word = 1ull << (last - 64 * j);
        }
        h = mix64(h ^ word);
      }
    ghash[wl][lane] = h;
  }
  __syncwarp();
  for (int i = 0; i < ng; ++i) {
    if (gmeta[wl][i][2] < 0) continue;
    const uint64_t* w = gwords[wl][i];
    synth_emit(v, queue, q0 + i, ghash[wl][i],
               [w](int a) { return ((w[a >> 6] >> (a & 63)) & 1ull) != 0; });
  }
}

// Reference feature tensor, fp32 [count][19][C]. One warp per queued position.
__global__ void __launch_bounds__(kSynthWarps * 32) k_features(EngineView v, int queue, float* out) {
  __shared__ WarpPos wps[kSynthWarps];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int q = blockIdx.x * kSynthWarps + wl;
  const int count = v.q_count[queue];
  if (q >= count) return;
  WarpPos& wp = wps[wl];
  const int2 ent = v.q_entries[queue][q];
  const int r = ent.x;
  const int d = warp_rebuild(v, r, ent.y, wp);
  if (d < 0) { if (lane == 0) v.hdr[r].status = OMQ_BAD_ARG; return; }
  const TreeHeader& H = v.hdr[r];
  const float player = (float)((d % 2 == 0) ? H.root_player : 3 - H.root_player);
  const uint32_t hp = history_planes(H.root_mc + d, d, kFullHistoryGomoku);
  const int last = d >= 1 ? wp.acts[d - 1] : -1;
  float* o = out + (size_t)q * kPlanes * v.C;
  for (int c = lane; c < v.C; c += 32) {
    o[c] = wp.board[c] != 0 ? 1.0f : 0.0f;
    o[v.C + c] = player;
    for (int p = 2; p < kPlanes; ++p)
      o[(size_t)p * v.C + c] = (((hp >> p) & 1u) && c == last) ? 1.0f : 0.0f;
  }
}

// 16-bit encodings of 1.0 and 2.0 (the only feature values of Gomoku and Go planes)
__device__ __forceinline__ uint16_t one_h16(bool f16) { return f16 ? 0x3C00 : 0x3F80; }
constexpr uint16_t kTwoH16 = 0x4000;  // 2.0 in both bf16 and fp16

// ResNet input: the same planes as k_features, bf16 or fp16 (the net's dtype), channels padded to
// 64, in the padded pixel space [(S+1) x (S+1)] whose last row and column stay zero. One warp per
// queued position.
__global__ void __launch_bounds__(kSynthWarps * 32) k_pack_queue(EngineView v, int queue, int P, bool f16,
                                                                 uint4* out) {
  __shared__ WarpPos wps[kSynthWarps];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int q = blockIdx.x * kSynthWarps + wl;
  const int count = v.q_count[queue];
  if (q >= count) return;
  WarpPos& wp = wps[wl];
  const int2 ent = v.q_entries[queue][q];
  const int r = ent.x;
  const int d = warp_rebuild(v, r, ent.y, wp);
  if (d < 0) { if (lane == 0) v.hdr[r].status = OMQ_BAD_ARG; return; }
  const TreeHeader& H = v.hdr[r];
  const uint16_t one = one_h16(f16);
  const uint16_t player = ((d % 2 == 0) ? H.root_player : 3 - H.root_player) == 1 ? one : kTwoH16;
  const uint32_t hp = history_planes(H.root_mc + d, d, kFullHistoryGomoku);
  const int last = d >= 1 ? wp.acts[d - 1] : -1;
  const int S = v.S;
  uint4* o = out + (size_t)q * P * 8;
  for (int i = lane; i < P * 8; i += 32) {
    const int pix = i >> 3, chunk = i & 7;
    const int y = pix / (S + 1), x = pix - y * (S + 1);
    uint16_t h[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (y < S && x < S) {
      const int c = y * S + x;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int ch = chunk * 8 + e;
        if (ch == 0) h[e] = wp.board[c] != 0 ? one : 0;
        else if (ch == 1) h[e] = player;
        else if (ch < kPlanes) h[e] = (((hp >> ch) & 1u) && c == last) ? one : 0;
      }
    }
    o[i] = *reinterpret_cast<uint4*>(h);
  }
}

// ---------------------------------------------------------------------------------------------
// Go: 17 history planes from the replayed position (go_device.cuh)
// ---------------------------------------------------------------------------------------------
struct GoWarpPos {
  GoPos pos;
  int8_t ring[kGoHistory * kMaxCells];
  uint64_t words[kGoPlanes * kMaxWords];
};

// Bit of plane p at cell c of the Go features (planes 0-7 own stones k plies ago, 8-15 the
// opponent's, 16 black to move).
__device__ __forceinline__ bool go_plane_bit(const EngineView& v, int r, const GoWarpPos& w, int p,
                                             int c) {
  if (p == 16) return w.pos.player == 1;
  const int k = p & 7;
  const int8_t s = go_hist_board(v, r, w.pos, w.ring, k)[c];
  return s == (p < 8 ? w.pos.player : 3 - w.pos.player);
}

__device__ int go_queue_replay(const EngineView& v, int queue, int q, GoWarpPos& w, int& r) {
  const int2 ent = v.q_entries[queue][q];
  r = ent.x;
  const int d = warp_go_replay(v, r, ent.y, w.pos, w.ring);
  if (d < 0 && (threadIdx.x & 31) == 0) v.hdr[r].status = OMQ_BAD_ARG;
  return d;
}

constexpr int kGoWarps = 4;

// Synthetic evaluator on Go positions: hash folded over the 17 binarised planes, plane by plane,
// 64-cell words in order (oracle_feature_hash_go); legal = empty points plus pass.
__global__ void __launch_bounds__(kGoWarps * 32) k_synth_go(EngineView v, int queue) {
  __shared__ GoWarpPos wps[kGoWarps];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int q = blockIdx.x * kGoWarps + wl;
  if (q >= v.q_count[queue]) return;
  GoWarpPos& w = wps[wl];
  int r;
  if (go_queue_replay(v, queue, q, w, r) < 0) return;
  const int nwords = (v.C + 63) / 64;
  for (int i = lane; i < kGoPlanes * nwords; i += 32) {
    const int p = i / nwords, j = i - p * nwords;
    uint64_t word = 0;
    for (int b = 0; b < 64; ++b) {
      const int c = j * 64 + b;
      if (c < v.C && go_plane_bit(v, r, w, p, c)) word |= 1ull << b;
    }
    w.words[i] = word;
  }
  __syncwarp();
  uint64_t h = 0;
  if (lane == 0) {
    h = 0x243F6A8885A308D3ull;
    for (int i = 0; i < kGoPlanes * nwords; ++i) h = mix64(h ^ w.words[i]);
  }
  h = __shfl_sync(0xFFFFFFFFu, h, 0);
  const int8_t* board = w.pos.board;
  synth_emit(v, queue, q, h, [board](int a) { return board[a] != 0; });
}

__global__ void __launch_bounds__(kGoWarps * 32) k_features_go(EngineView v, int queue, float* out) {
  __shared__ GoWarpPos wps[kGoWarps];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int q = blockIdx.x * kGoWarps + wl;
  if (q >= v.q_count[queue]) return;
  GoWarpPos& w = wps[wl];
  int r;
  if (go_queue_replay(v, queue, q, w, r) < 0) return;
  float* o = out + (size_t)q * kGoPlanes * v.C;
  for (int p = 0; p < kGoPlanes; ++p)
    for (int c = lane; c < v.C; c += 32) o[(size_t)p * v.C + c] = go_plane_bit(v, r, w, p, c) ? 1.0f : 0.0f;
}

// ResNet input for Go: the 17 planes as bf16 or fp16, channels padded to 64, padded pixel layout.
__global__ void __launch_bounds__(kGoWarps * 32) k_pack_queue_go(EngineView v, int queue, int P, bool f16,
                                                                 uint4* out) {
  __shared__ GoWarpPos wps[kGoWarps];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int q = blockIdx.x * kGoWarps + wl;
  if (q >= v.q_count[queue]) return;
  GoWarpPos& w = wps[wl];
  int r;
  if (go_queue_replay(v, queue, q, w, r) < 0) return;
  const int S = v.S;
  uint4* o = out + (size_t)q * P * 8;
  for (int i = lane; i < P * 8; i += 32) {
    const int pix = i >> 3, chunk = i & 7;
    const int y = pix / (S + 1), x = pix - y * (S + 1);
    uint16_t h[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (y < S && x < S && chunk < 3) {
      const int c = y * S + x;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int ch = chunk * 8 + e;
        if (ch < kGoPlanes) h[e] = go_plane_bit(v, r, w, ch, c) ? one_h16(f16) : 0;
      }
    }
    o[i] = *reinterpret_cast<uint4*>(h);
  }
}

// ---------------------------------------------------------------------------------------------
// Chess: 119 planes from the replayed position (chess_device.cuh)
// ---------------------------------------------------------------------------------------------
constexpr int kChessWarps = 4;

__device__ int chess_queue_replay(const EngineView& v, int queue, int q, ChessReplay& w, int& r) {
  const int2 ent = v.q_entries[queue][q];
  r = ent.x;
  const int d = warp_ch_replay(v, r, ent.y, w, true);
  if (d < 0 && (threadIdx.x & 31) == 0) v.hdr[r].status = OMQ_BAD_ARG;
  return d;
}

// Synthetic evaluator on chess positions: hash folded over the 119 binarised planes (one 64-bit
// word per plane, oracle_feature_hash_chess); the policy covers all 4672 actions, so action a
// has rank a among the "legal" ones.
__global__ void __launch_bounds__(kChessWarps * 32) k_synth_chess(EngineView v, int queue) {
  __shared__ ChessReplay wps[kChessWarps];
  __shared__ uint64_t words[kChessWarps][kChessPlanes];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int q = blockIdx.x * kChessWarps + wl;
  if (q >= v.q_count[queue]) return;
  ChessReplay& w = wps[wl];
  int r;
  if (chess_queue_replay(v, queue, q, w, r) < 0) return;
  for (int c = lane; c < kChessPlanes; c += 32) {
    uint64_t word = 0;
    for (int s = 0; s < 64; ++s)
      if (ch_plane(v, r, w, c, s) != 0.0f) word |= 1ull << s;
    words[wl][c] = word;
  }
  __syncwarp();
  uint64_t h = 0;
  if (lane == 0) {
    h = 0x243F6A8885A308D3ull;
    for (int c = 0; c < kChessPlanes; ++c) h = mix64(h ^ words[wl][c]);
  }
  h = __shfl_sync(0xFFFFFFFFu, h, 0);
  if (queue == 0) {
    uint64_t tot = 0;
    for (int a = lane; a < kChessActions; a += 32)
      tot += exp2_fixed(exp_step(mix64(h + 0x9E3779B97F4A7C15ull * (uint64_t)(a + 1))));
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xFFFFFFFFu, tot, o);
    const double rtot = 1.0 / (double)tot;
    float* out = v.q_policy[0] + (size_t)q * v.A;
    for (int a = lane; a < kChessActions; a += 32) {
      const uint64_t wa = exp2_fixed(exp_step(mix64(h + 0x9E3779B97F4A7C15ull * (uint64_t)(a + 1))));
      const uint64_t qa = 512ull * div_floor53(wa * 32640ull, tot, rtot) + (uint64_t)a;
      out[a] = __fmul_rn(__ull2float_rn(qa), 1.0f / 16777216.0f);
    }
  }
  if (lane == 0) {
    const int64_t e = (int64_t)exp2_fixed(exp_step(mix64(h ^ 0xD1B54A32D192ED03ull)));
    const int64_t dd = (int64_t)1 << 26;
    const int64_t val = ((e - dd) * 4096) / (e + dd);
    v.q_value[queue][q] = __fmul_rn(__ll2float_rn(val), 1.0f / 4096.0f);
  }
}

__global__ void __launch_bounds__(kChessWarps * 32) k_features_chess(EngineView v, int queue, float* out) {
  __shared__ ChessReplay wps[kChessWarps];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int q = blockIdx.x * kChessWarps + wl;
  if (q >= v.q_count[queue]) return;
  ChessReplay& w = wps[wl];
  int r;
  if (chess_queue_replay(v, queue, q, w, r) < 0) return;
  float* o = out + (size_t)q * kChessPlanes * 64;
  for (int i = lane; i < kChessPlanes * 64; i += 32) o[i] = ch_plane(v, r, w, i >> 6, i & 63);
}

// ResNet input for chess: 119 planes as bf16 or fp16, channels padded to 128, padded 9x9 pixel grid.
__global__ void __launch_bounds__(kChessWarps * 32) k_pack_queue_chess(EngineView v, int queue, int P, bool f16,
                                                                       uint4* out) {
  __shared__ ChessReplay wps[kChessWarps];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int q = blockIdx.x * kChessWarps + wl;
  if (q >= v.q_count[queue]) return;
  ChessReplay& w = wps[wl];
  int r;
  if (chess_queue_replay(v, queue, q, w, r) < 0) return;
  uint4* o = out + (size_t)q * P * 16;
  for (int i = lane; i < P * 16; i += 32) {
    const int pix = i >> 4, chunk = i & 15;
    const int y = pix / 9, x = pix - y * 9;
    uint16_t h[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int ch = chunk * 8 + e;
      const float val = (y < 8 && x < 8 && ch < kChessPlanes) ? ch_plane(v, r, w, ch, y * 8 + x) : 0.0f;
      h[e] = to_h16(val, f16);
    }
    o[i] = *reinterpret_cast<uint4*>(h);
  }
}

void launch_pack_queue(const EngineView& v, int queue, int P, int in_pad, void* out, bool f16, cudaStream_t s) {
  if (v.game == OMQ_GAME_CHESS) {
    (void)in_pad;  // 128
    const int cap = v.R * v.WCAP;
    count_launches(1);
    k_pack_queue_chess<<<(cap + kChessWarps - 1) / kChessWarps, kChessWarps * 32, 0, s>>>(
        v, queue, P, f16, reinterpret_cast<uint4*>(out));
    return;
  }
  if (v.game == OMQ_GAME_GO) {
    const int cap = v.R * v.WCAP;
    count_launches(1);
    k_pack_queue_go<<<(cap + kGoWarps - 1) / kGoWarps, kGoWarps * 32, 0, s>>>(
        v, queue, P, f16, reinterpret_cast<uint4*>(out));
    return;
  }
  const int cap = v.R * v.WCAP;
  count_launches(1);
  k_pack_queue<<<(cap + kSynthWarps - 1) / kSynthWarps, kSynthWarps * 32, 0, s>>>(
      v, queue, P, f16, reinterpret_cast<uint4*>(out));
}

void launch_synth_eval(const EngineView& v, int queue, cudaStream_t s) {
  const int cap = v.R * v.WCAP;
  count_launches(1);
  if (v.game == OMQ_GAME_GO) {
    k_synth_go<<<(cap + kGoWarps - 1) / kGoWarps, kGoWarps * 32, 0, s>>>(v, queue);
    return;
  }
  if (v.game == OMQ_GAME_CHESS) {
    k_synth_chess<<<(cap + kChessWarps - 1) / kChessWarps, kChessWarps * 32, 0, s>>>(v, queue);
    return;
  }
  // 8 positions per warp once the queue's capacity fills the SMs with such warps, fewer below
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    cudaGetLastError();
    sms = 148;
  }
  const int group = max(1, min(kSynthGroup, cap / (sms * 2 * kSynthWarps)));
  const int per_block = kSynthWarps * group;
  k_synth<<<(cap + per_block - 1) / per_block, kSynthWarps * 32, 0, s>>>(v, queue, group);
}

void launch_features(const EngineView& v, int queue, float* out, cudaStream_t s) {
  const int cap = v.R * v.WCAP;
  count_launches(1);
  if (v.game == OMQ_GAME_GO) {
    k_features_go<<<(cap + kGoWarps - 1) / kGoWarps, kGoWarps * 32, 0, s>>>(v, queue, out);
    return;
  }
  if (v.game == OMQ_GAME_CHESS) {
    k_features_chess<<<(cap + kChessWarps - 1) / kChessWarps, kChessWarps * 32, 0, s>>>(v, queue, out);
    return;
  }
  k_features<<<(cap + kSynthWarps - 1) / kSynthWarps, kSynthWarps * 32, 0, s>>>(v, queue, out);
}

}  // namespace omq
