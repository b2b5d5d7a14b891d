// Self-play move step on the device (Gomoku): after a batched search of every game's position,
// one kernel records each live game's training example (position, root visit counts, root
// value), chooses its move, plays it, and applies the game-end and resignation rules, without a
// host round trip. It follows SelfPlayGame.play_single_move
// (python/mcts/neural_networks/self_play_manager.py:218-370): temperature sampling from the
// visit distribution while move_number < temperature_threshold, arg-max afterwards
// (_get_temperature, :466-470); the game ends on five in a row or a full board; after the move,
// the player who moved resigns when the search's root value is below the threshold and more than
// resign_min_move moves have been played (:350-365).
//
// The reference samples with numpy's global generator. Here the draw is a counter-based hash of
// (seed, game, move), so a run is reproducible and the host can replay it exactly
// (omoknuni_quantum_b200.selfplay.counter_draw): the sampled action is the first one whose
// cumulative visit count exceeds floor(u * total) with u = hash / 2^64, i.e. visit-proportional.
#include "omq_internal.cuh"

namespace omq {

constexpr int kSelfplayThreads = 256;

__device__ __forceinline__ uint64_t selfplay_hash(uint64_t seed, int game, int move) {
  return mix64(mix64(mix64(seed) + (uint64_t)game) + (uint64_t)move);
}

// Five (or more) in a row anywhere on the board (the rule of roots.has_five and of the
// reference's terminal check, fast_terminal_check.py:233-332).
__device__ bool block_has_five(const int8_t* b, int S, int* flag) {
  if (threadIdx.x == 0) *flag = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < S * S; i += blockDim.x) {
    const int p = b[i];
    if (p == 0) continue;
    const int r0 = i / S, c0 = i - (i / S) * S;
    const int dr[4] = {0, 1, 1, 1}, dc[4] = {1, 0, 1, -1};
    for (int d = 0; d < 4; ++d) {
      int s = 1;
      for (; s < 5; ++s) {
        const int r = r0 + dr[d] * s, c = c0 + dc[d] * s;
        if (r < 0 || r >= S || c < 0 || c >= S || b[r * S + c] != p) break;
      }
      if (s == 5) { *flag = 1; break; }
    }
  }
  __syncthreads();
  return *flag != 0;
}

// One block per game. game[g] = {finished, winner (+1 black, -1 white, 0 draw), resigned, error,
// moves played, 0, 0, 0}.
__global__ void __launch_bounds__(kSelfplayThreads) k_selfplay_move(EngineView v, omq_selfplay_step_config c,
                                                                    int8_t* boards, int32_t* game,
                                                                    int32_t* actions, int32_t* moves_hist,
                                                                    int32_t* visits_hist, float* values_hist,
                                                                    int8_t* states_hist) {
  __shared__ int8_t board[kMaxCells];
  __shared__ int s_total, s_action, s_flag, s_stones;
  __shared__ int s_chunk[kSelfplayThreads];
  const int g = blockIdx.x, tid = threadIdx.x;
  int32_t* st = game + 8 * (size_t)g;
  if (st[0]) {  // finished: no move, and the next search starts a fresh tree for it
    if (tid == 0) actions[g] = -1;
    return;
  }
  const int C = v.C, A = v.A, m = c.move_number;
  const size_t slot = (size_t)g * c.max_moves + m;
  int32_t* vis = visits_hist + slot * A;
  const size_t base = (size_t)g * v.T;
  // position and root visit counts of this move's search (MCTS._extract_policy, mcts.py:1069)
  if (tid == 0) { s_total = 0; s_stones = 0; }
  for (int i = tid; i < C; i += blockDim.x) {
    board[i] = boards[(size_t)g * C + i];
    states_hist[slot * C + i] = board[i];
  }
  for (int a = tid; a < A; a += blockDim.x) vis[a] = 0;
  __syncthreads();
  const NodeTopo rt = v.topo[base];
  const int n = topo_count(rt);
  int local = 0, stones = 0;
  for (int j = tid; j < n; j += blockDim.x) {
    const int32_t cnt = v.stats[base + rt.child_start + j].N;
    vis[topo_action(v.topo[base + rt.child_start + j])] = cnt;
    local += cnt;
  }
  for (int i = tid; i < C; i += blockDim.x) stones += board[i] != 0;
  atomicAdd(&s_total, local);
  atomicAdd(&s_stones, stones);
  __syncthreads();
  const int total = s_total;
  const int player = (s_stones % 2 == 0) ? 1 : 2;
  // root value W / N from the side to move's perspective (MCTS.get_root_value)
  const NodeStats rs = v.stats[base];
  const float value = rs.N > 0 ? __fdiv_rn(rs.W, __int2float_rn(rs.N)) : 0.0f;
  // the move: sampled in proportion to the visits (temperature 1) or the first most-visited
  if (m < c.temperature_threshold && c.temperature > 0.0f) {
    const uint64_t h = selfplay_hash(c.seed, g, m);
    if (total == 0) {
      if (tid == 0) s_action = (int)__umul64hi(h, (uint64_t)A);  // uniform policy
    } else {
      const int64_t target = (int64_t)__umul64hi(h, (uint64_t)total);  // in [0, total)
      // block-wide inclusive scan of the visits in action order, chunk by chunk
      const int per = (A + blockDim.x - 1) / blockDim.x;
      int sum = 0;
      for (int a = tid * per; a < min(A, (tid + 1) * per); ++a) sum += vis[a];
      s_chunk[tid] = sum;
      __syncthreads();
      if (tid == 0) {
        int64_t acc = 0;
        int t = 0;
        for (; t < (int)blockDim.x; ++t) {
          if (acc + s_chunk[t] > target) break;
          acc += s_chunk[t];
        }
        int a = t * per;
        for (; a < A; ++a) {
          acc += vis[a];
          if (acc > target) break;
        }
        s_action = a;
      }
    }
  } else {
    if (tid == 0) {
      int best = 0, bv = vis[0];
      for (int a = 1; a < A; ++a)
        if (vis[a] > bv) { bv = vis[a]; best = a; }
      s_action = best;
    }
  }
  __syncthreads();
  const int action = s_action;
  if (action < 0 || action >= C || board[action] != 0) {  // an illegal move ends the game with an error
    if (tid == 0) { st[0] = 1; st[3] = OMQ_BAD_ARG; actions[g] = -1; }
    return;
  }
  if (tid == 0) board[action] = (int8_t)player;
  __syncthreads();
  const bool five = block_has_five(board, v.S, &s_flag);
  if (tid == 0) {
    boards[(size_t)g * C + action] = (int8_t)player;
    actions[g] = action;
    moves_hist[slot] = action;
    values_hist[slot] = value;
    st[4] = m + 1;
    if (five) { st[0] = 1; st[1] = player == 1 ? 1 : -1; }
    else if (s_stones + 1 >= C) { st[0] = 1; st[1] = 0; }
    // resignation after the move, also when the move ended the game (it then decides the winner)
    if (c.enable_resign && m + 1 > c.resign_min_move && (double)value < (double)c.resign_threshold) {
      st[0] = 1;
      st[2] = 1;
      st[1] = player == 1 ? -1 : 1;
    }
  }
}

}  // namespace omq

using namespace omq;

extern "C" int omq_selfplay_move(omq_engine* e, const omq_selfplay_step_config* cfg, int8_t* d_boards,
                                 int32_t* d_game, int32_t* d_actions, int32_t* d_moves_hist,
                                 int32_t* d_visits_hist, float* d_values_hist, int8_t* d_states_hist,
                                 void* stream) {
  if (!e || !cfg || !d_boards || !d_game || !d_actions || !d_moves_hist || !d_visits_hist || !d_values_hist ||
      !d_states_hist) {
    set_error("null argument");
    return OMQ_BAD_ARG;
  }
  if (e->v.game != OMQ_GAME_GOMOKU) { set_error("device self-play moves are Gomoku only"); return OMQ_BAD_ARG; }
  const omq_selfplay_step_config c = *cfg;
  if (c.move_number < 0 || c.move_number >= c.max_moves || !(c.temperature == 0.0f || c.temperature == 1.0f)) {
    set_error("bad self-play step (move %d of %d, temperature %g: 0 or 1 on the device)", c.move_number,
              c.max_moves, (double)c.temperature);
    return OMQ_BAD_ARG;
  }
  DeviceGuard g(e->cfg.device);
  count_launches(1);
  k_selfplay_move<<<e->v.R, kSelfplayThreads, 0, (cudaStream_t)stream>>>(
      e->v, c, d_boards, d_game, d_actions, d_moves_hist, d_visits_hist, d_values_hist, d_states_hist);
  return cuda_status(cudaGetLastError(), "k_selfplay_move");
}
