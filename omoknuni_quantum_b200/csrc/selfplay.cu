// Self-play move step on the device (Gomoku, chess and Go): after a batched search of every game's position,
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
#include "chess_device.cuh"
#include "go_device.cuh"
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

// Root visit counts of game g's search by action into vis[A] (zeroed first) and their total,
// and the root value W / N from the side to move's perspective (MCTS._extract_policy,
// mcts.py:1069; MCTS.get_root_value). Block-collective; *s_total must be 0 on entry.
__device__ float block_root_visits(const EngineView& v, int g, int32_t* vis, int* s_total) {
  const int tid = threadIdx.x;
  const size_t base = (size_t)g * v.T;
  for (int a = tid; a < v.A; a += blockDim.x) vis[a] = 0;
  __syncthreads();
  const NodeTopo rt = v.topo[base];
  const int n = topo_count(rt);
  int local = 0;
  for (int j = tid; j < n; j += blockDim.x) {
    const int32_t cnt = v.stats[base + rt.child_start + j].N;
    vis[topo_action(v.topo[base + rt.child_start + j])] = cnt;
    local += cnt;
  }
  atomicAdd(s_total, local);
  const NodeStats rs = v.stats[base];
  return rs.N > 0 ? __fdiv_rn(rs.W, __int2float_rn(rs.N)) : 0.0f;
}

// The move of game g at move m (block-collective, after the visits are complete): sampled in
// proportion to the visits (temperature 1, while m < temperature_threshold) or the first
// most-visited action. s_chunk holds blockDim.x ints.
__device__ int block_choose(const omq_selfplay_step_config& c, int g, int m, const int32_t* vis, int A,
                            int total, int* s_chunk, int* s_action) {
  const int tid = threadIdx.x;
  if (m < c.temperature_threshold && c.temperature > 0.0f) {
    const uint64_t h = selfplay_hash(c.seed, g, m);
    if (total == 0) {
      if (tid == 0) *s_action = (int)__umul64hi(h, (uint64_t)A);  // uniform policy
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
        *s_action = a;
      }
    }
  } else if (tid == 0) {
    int best = 0, bv = vis[0];
    for (int a = 1; a < A; ++a)
      if (vis[a] > bv) { bv = vis[a]; best = a; }
    *s_action = best;
  }
  __syncthreads();
  return *s_action;
}

// Resignation after the move (self_play_manager.py:350-365), also when the move ended the game
// (it then decides the winner): the player who moved (1 first, 2 second) resigns.
__device__ __forceinline__ void apply_resign(const omq_selfplay_step_config& c, int m, float value, int player,
                                             int32_t* st) {
  if (c.enable_resign && m + 1 > c.resign_min_move && (double)value < (double)c.resign_threshold) {
    st[0] = 1;
    st[2] = 1;
    st[1] = player == 1 ? -1 : 1;
  }
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
  if (tid == 0) { s_total = 0; s_stones = 0; }
  for (int i = tid; i < C; i += blockDim.x) {
    board[i] = boards[(size_t)g * C + i];
    states_hist[slot * C + i] = board[i];
  }
  __syncthreads();
  const float value = block_root_visits(v, g, vis, &s_total);
  int stones = 0;
  for (int i = tid; i < C; i += blockDim.x) stones += board[i] != 0;
  atomicAdd(&s_stones, stones);
  __syncthreads();
  const int player = (s_stones % 2 == 0) ? 1 : 2;
  const int action = block_choose(c, g, m, vis, A, s_total, s_chunk, &s_action);
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
    apply_resign(c, m, value, player, st);
  }
}

// Chess: the same step on the engine's root records (records[g][1 + 100] position records, the
// position then the earlier ones, most recent first; nprior[g] of them present). The move is
// played as ChessPosition.play / ChessState::makeMove: the played position becomes the most
// recent earlier one (the list keeps 100), and the new position's repetition count is 1 + the
// earlier positions with the same piece placement (compared square by square). The game ends as
// ChessState::getGameResult (chess_state.cpp:623-676): no legal move (mate: the side not to move
// wins; stalemate: draw), insufficient material, halfmove clock >= 100 or a third occurrence
// (draws). game[g] = {finished, winner (+1 white, -1 black, 0 draw), resigned, error, moves
// played, 0, 0, 0}; states_hist[g][move] holds the 80-byte record of the searched position.
__global__ void __launch_bounds__(kSelfplayThreads) k_selfplay_move_chess(
    EngineView v, omq_selfplay_step_config c, ChessRec* records, int32_t* nprior, int32_t* game,
    int32_t* actions, int32_t* moves_hist, int32_t* visits_hist, float* values_hist, ChessRec* states_hist) {
  __shared__ ChessRec s_rec[1 + kChessPrior];
  __shared__ ChessRec s_new;
  __shared__ uint32_t s_mask[kChessMaskWords];
  __shared__ ChessMoveList s_list;
  __shared__ int s_total, s_action, s_reps, s_legal;
  __shared__ int s_chunk[kSelfplayThreads];
  const int g = blockIdx.x, tid = threadIdx.x;
  int32_t* st = game + 8 * (size_t)g;
  if (st[0]) {
    if (tid == 0) actions[g] = -1;
    return;
  }
  const int A = v.A, m = c.move_number;
  const size_t slot = (size_t)g * c.max_moves + m;
  int32_t* vis = visits_hist + slot * A;
  ChessRec* rec = records + (size_t)g * (1 + kChessPrior);
  const int np = min(max(nprior[g], 0), kChessPrior);
  // the records as 8-byte words (ChessRec is 8-byte aligned, 80 bytes)
  constexpr int kW = (int)(sizeof(ChessRec) / 8);
  for (int i = tid; i < (1 + np) * kW; i += blockDim.x)
    reinterpret_cast<uint64_t*>(s_rec)[i] = reinterpret_cast<const uint64_t*>(rec)[i];
  if (tid == 0) { s_total = 0; s_reps = 0; }
  __syncthreads();
  if (tid < kW) reinterpret_cast<uint64_t*>(states_hist + slot)[tid] = reinterpret_cast<const uint64_t*>(s_rec)[tid];
  const float value = block_root_visits(v, g, vis, &s_total);
  __syncthreads();
  const int player = s_rec[0].side;
  const int action = block_choose(c, g, m, vis, A, s_total, s_chunk, &s_action);
  // the action must be a legal move of the position
  if (tid < 32) warp_ch_legal(s_rec[0], s_mask, s_list);
  __syncthreads();
  const bool legal = action >= 0 && action < kChessActions && ((s_mask[action >> 5] >> (action & 31)) & 1u);
  if (!legal) {
    if (tid == 0) { st[0] = 1; st[3] = OMQ_BAD_ARG; actions[g] = -1; }
    return;
  }
  if (tid == 0) {
    s_new = s_rec[0];
    ch_play(s_new, ch_move(s_rec[0], action));
  }
  __syncthreads();
  // repetitions among the new list of earlier positions: the played one, then the old list
  const int np2 = min(np + 1, kChessPrior);
  int same = 0;
  for (int i = tid; i < np2; i += blockDim.x) {
    const uint64_t* a = reinterpret_cast<const uint64_t*>(s_rec[i].sq);
    const uint64_t* b = reinterpret_cast<const uint64_t*>(s_new.sq);
    bool eq = true;
#pragma unroll
    for (int w = 0; w < 8; ++w) eq &= a[w] == b[w];
    same += eq;
  }
  atomicAdd(&s_reps, same);
  __syncthreads();
  if (tid == 0) {
    const int reps = 1 + s_reps;
    s_new.reps = (int8_t)(reps < 127 ? reps : 127);
  }
  __syncthreads();
  if (tid < 32) {
    const int n = warp_ch_legal(s_new, s_mask, s_list);
    if (tid == 0) s_legal = n;
  }
  __syncthreads();
  // the shifted list: record i + 1 = old record i, record 0 = the new position
  for (int i = tid; i < np2 * kW; i += blockDim.x)
    reinterpret_cast<uint64_t*>(rec + 1)[i] = reinterpret_cast<const uint64_t*>(s_rec)[i];
  if (tid < kW) reinterpret_cast<uint64_t*>(rec)[tid] = reinterpret_cast<const uint64_t*>(&s_new)[tid];
  if (tid == 0) {
    nprior[g] = np2;
    actions[g] = action;
    moves_hist[slot] = action;
    values_hist[slot] = value;
    st[4] = m + 1;
    if (s_legal == 0) {
      st[0] = 1;
      st[1] = ch_in_check(s_new, s_new.side) ? (s_new.side == chess::WHITE ? -1 : 1) : 0;
    } else if (ch_terminal(s_new, s_legal)) {
      st[0] = 1;
      st[1] = 0;
    }
    apply_resign(c, m, value, player, st);
  }
}

// Go: score of a finished game (GoRules::calculateScores / getTerritoryOwnership,
// go_rules.cpp:211-260, 343-380): every empty region bordered by one colour only counts for that
// colour; area scoring adds the stones on the board, territory scoring the prisoners; komi goes
// to white. No stones are marked dead. Returns +1 (black wins), -1 (white wins) or 0.
// Warp-collective; g.par / g.libs are used as the regions' union-find and border colours.
__device__ int warp_go_winner(const int8_t* b, int S, GoScratch& g, bool area, int prisoners_b,
                              int prisoners_w, float komi) {
  const int lane = threadIdx.x & 31, C = S * S;
  for (int c = lane; c < C; c += 32) { g.par[c] = c; g.libs[c] = 0; }
  __syncwarp();
  for (int c = lane; c < C; c += 32) {
    if (b[c]) continue;
    const int x = c % S;
    if (x < S - 1 && !b[c + 1]) go_unite(g.par, c, c + 1);
    if (c + S < C && !b[c + S]) go_unite(g.par, c, c + S);
  }
  __syncwarp();
  for (int c = lane; c < C; c += 32)
    if (!b[c]) g.par[c] = go_find(g.par, c);
  __syncwarp();
  int stones_b = 0, stones_w = 0;
  for (int c = lane; c < C; c += 32) {
    if (b[c]) { stones_b += b[c] == 1; stones_w += b[c] == 2; continue; }
    int nb[4];
    go_neighbours(c, S, nb);
    int col = 0;
    for (int k = 0; k < 4; ++k)
      if (nb[k] >= 0 && b[nb[k]]) col |= b[nb[k]];
    if (col) atomicOr(&g.libs[g.par[c]], col);
  }
  __syncwarp();
  int terr_b = 0, terr_w = 0;
  for (int c = lane; c < C; c += 32) {
    if (b[c]) continue;
    const int f = g.libs[g.par[c]];
    terr_b += f == 1;
    terr_w += f == 2;
  }
  for (int o = 16; o > 0; o >>= 1) {
    stones_b += __shfl_xor_sync(0xFFFFFFFFu, stones_b, o);
    stones_w += __shfl_xor_sync(0xFFFFFFFFu, stones_w, o);
    terr_b += __shfl_xor_sync(0xFFFFFFFFu, terr_b, o);
    terr_w += __shfl_xor_sync(0xFFFFFFFFu, terr_w, o);
  }
  const double black = (double)((area ? stones_b : prisoners_b) + terr_b);
  const double white = (double)((area ? stones_w : prisoners_w) + terr_w) + (double)komi;
  return black > white ? 1 : (white > black ? -1 : 0);
}

// Go: the same step on the engine's Go roots, updated in place (GoState::makeMove,
// go_state.cpp:227-356): hist[g][8][C] (the position, then the 7 before it), meta[g] = {side to
// move, ko point, consecutive passes}, keys[g][OMQ_GO_MAX_KEYS] / nkeys[g] the game's position
// keys in game order (after every non-pass move without the repetition rule - superko's
// history; after every move, with the side to move, under the repetition rule). The game ends
// after two consecutive passes (scored) or a third repetition (no result / draw: winner 0).
// game[g] = {finished, winner (+1 black, -1 white, 0 draw), resigned, error, moves played,
// black's prisoners, white's prisoners, repetition ended it}; states_hist[g][move] holds the
// searched position's 8 history boards.
__global__ void __launch_bounds__(kSelfplayThreads) k_selfplay_move_go(
    EngineView v, omq_selfplay_step_config c, float komi, int area, int8_t* hist, int32_t* meta, uint64_t* keys,
    int32_t* nkeys, int32_t* game, int32_t* actions, int32_t* moves_hist, int32_t* visits_hist,
    float* values_hist, int8_t* states_hist) {
  __shared__ int8_t s_hist[kGoHistory * kMaxCells];
  __shared__ int8_t s_board[kMaxCells + 3];
  __shared__ GoScratch s_g;
  __shared__ uint32_t s_mask[kGoMaskWords + 4];
  __shared__ uint64_t s_key;
  __shared__ int s_total, s_action, s_ok, s_ko, s_passes, s_captured;
  __shared__ int s_chunk[kSelfplayThreads];
  const int g = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  int32_t* st = game + 8 * (size_t)g;
  if (st[0]) {
    if (tid == 0) actions[g] = -1;
    return;
  }
  const int C = v.C, S = v.S, A = v.A, m = c.move_number;
  const size_t slot = (size_t)g * c.max_moves + m;
  int32_t* vis = visits_hist + slot * A;
  int8_t* H = hist + (size_t)g * kGoHistory * C;
  for (int i = tid; i < kGoHistory * C; i += blockDim.x) {
    s_hist[i] = H[i];
    states_hist[slot * kGoHistory * C + i] = s_hist[i];
  }
  if (tid == 0) s_total = 0;
  __syncthreads();
  const float value = block_root_visits(v, g, vis, &s_total);
  __syncthreads();
  const int player = meta[3 * g], ko0 = meta[3 * g + 1], passes0 = meta[3 * g + 2];
  const int repeated0 = st[7];  // read before thread 0 rewrites it below
  const int action = block_choose(c, g, m, vis, A, s_total, s_chunk, &s_action);
  uint64_t* K = keys + (size_t)g * OMQ_GO_MAX_KEYS;
  const int nk = min(max(nkeys[g], 0), OMQ_GO_MAX_KEYS);
  if (tid < 32) {
    // legality (GoState::isLegalMove): the basic rules, then positional superko
    for (int i = lane; i < C; i += 32) s_board[i] = s_hist[i];
    __syncwarp();
    bool ok = action >= 0 && action <= C;
    if (ok && action < C) {
      warp_go_analyze(s_board, S, s_g);
      warp_go_legal(s_board, S, player, ko0, s_g, s_mask);
      ok = (s_mask[action >> 5] >> (action & 31)) & 1u;
    }
    int opp_before = 0;
    for (int i = lane; i < C; i += 32) opp_before += s_board[i] == 3 - player;
    for (int o = 16; o > 0; o >>= 1) opp_before += __shfl_xor_sync(0xFFFFFFFFu, opp_before, o);
    int ko = ko0, passes = passes0;
    if (ok) warp_go_play(s_board, S, player, action, s_g, ko, passes);
    int opp_after = 0;
    for (int i = lane; i < C; i += 32) opp_after += s_board[i] == 3 - player;
    for (int o = 16; o > 0; o >>= 1) opp_after += __shfl_xor_sync(0xFFFFFFFFu, opp_after, o);
    const uint64_t key = warp_go_board_key(s_board, C) ^ (ko >= 0 ? go_ko_key(ko) : 0ull);
    if (ok && v.go_superko && action < C) {
      bool seen = false;
      for (int i = lane; i < nk; i += 32) seen |= K[i] == key;
      ok = !__any_sync(0xFFFFFFFFu, seen);
    }
    if (lane == 0) {
      s_ok = ok;
      s_ko = ko;
      s_passes = passes;
      s_captured = opp_before - opp_after;
      s_key = key;
    }
  }
  __syncthreads();
  if (!s_ok) {
    if (tid == 0) { st[0] = 1; st[3] = OMQ_BAD_ARG; actions[g] = -1; }
    return;
  }
  // the game's keys: superko history (non-pass moves) or the repetition rule's (every move)
  const bool cycle = v.go_cycle != 0;
  const bool add = cycle ? repeated0 == 0 : action < C;
  const uint64_t newkey = cycle ? (s_key ^ go_side_key(3 - player)) : s_key;
  int nk2 = nk;
  if (add) {
    if (nk == OMQ_GO_MAX_KEYS) {  // full: keep the most recent keys
      uint64_t tmp[(OMQ_GO_MAX_KEYS + kSelfplayThreads - 1) / kSelfplayThreads];
      int j = 0;
      for (int i = tid; i + 1 < nk; i += blockDim.x) tmp[j++] = K[i + 1];
      __syncthreads();
      j = 0;
      for (int i = tid; i + 1 < nk; i += blockDim.x) K[i] = tmp[j++];
      nk2 = nk - 1;
    }
    if (tid == 0) K[nk2] = newkey;
    ++nk2;
  }
  __syncthreads();
  int repeated = repeated0;
  if (cycle && add) {
    int cnt = 0;
    for (int i = tid; i < nk2; i += blockDim.x) cnt += K[i] == newkey;
    if (tid == 0) s_total = 0;
    __syncthreads();
    atomicAdd(&s_total, cnt);
    __syncthreads();
    repeated = s_total >= 3;
  }
  // history: the new board first, the 7 most recent before it
  for (int i = tid; i < (kGoHistory - 1) * C; i += blockDim.x) H[C + i] = s_hist[i];
  for (int i = tid; i < C; i += blockDim.x) H[i] = s_board[i];
  int winner = 0;
  const bool over = s_passes >= 2 || repeated;
  if (tid < 32 && over && !repeated)
    winner = warp_go_winner(s_board, S, s_g, area != 0, st[5] + (player == 1 ? s_captured : 0),
                            st[6] + (player == 2 ? s_captured : 0), komi);
  if (tid == 0) {
    nkeys[g] = nk2;
    meta[3 * g] = 3 - player;
    meta[3 * g + 1] = s_ko;
    meta[3 * g + 2] = s_passes;
    actions[g] = action;
    moves_hist[slot] = action;
    values_hist[slot] = value;
    st[4] = m + 1;
    st[player == 1 ? 5 : 6] += s_captured;
    st[7] = repeated;
    if (over) { st[0] = 1; st[1] = winner; }
    apply_resign(c, m, value, player, st);
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
  if (e->v.game != OMQ_GAME_GOMOKU) { set_error("omq_selfplay_move is for Gomoku engines (omq_selfplay_move_chess for chess)"); return OMQ_BAD_ARG; }
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

extern "C" int omq_selfplay_move_chess(omq_engine* e, const omq_selfplay_step_config* cfg, void* d_records,
                                       int32_t* d_nprior, int32_t* d_game, int32_t* d_actions,
                                       int32_t* d_moves_hist, int32_t* d_visits_hist, float* d_values_hist,
                                       void* d_states_hist, void* stream) {
  if (!e || !cfg || !d_records || !d_nprior || !d_game || !d_actions || !d_moves_hist || !d_visits_hist ||
      !d_values_hist || !d_states_hist) {
    set_error("null argument");
    return OMQ_BAD_ARG;
  }
  if (e->v.game != OMQ_GAME_CHESS) { set_error("omq_selfplay_move_chess on a non-chess engine"); return OMQ_BAD_ARG; }
  if ((reinterpret_cast<uintptr_t>(d_records) | reinterpret_cast<uintptr_t>(d_states_hist)) & 7) {
    set_error("chess records must be 8-byte aligned");
    return OMQ_BAD_ARG;
  }
  const omq_selfplay_step_config c = *cfg;
  if (c.move_number < 0 || c.move_number >= c.max_moves || !(c.temperature == 0.0f || c.temperature == 1.0f)) {
    set_error("bad self-play step (move %d of %d, temperature %g: 0 or 1 on the device)", c.move_number,
              c.max_moves, (double)c.temperature);
    return OMQ_BAD_ARG;
  }
  DeviceGuard g(e->cfg.device);
  count_launches(1);
  k_selfplay_move_chess<<<e->v.R, kSelfplayThreads, 0, (cudaStream_t)stream>>>(
      e->v, c, reinterpret_cast<ChessRec*>(d_records), d_nprior, d_game, d_actions, d_moves_hist, d_visits_hist,
      d_values_hist, reinterpret_cast<ChessRec*>(d_states_hist));
  return cuda_status(cudaGetLastError(), "k_selfplay_move_chess");
}

extern "C" int omq_selfplay_move_go(omq_engine* e, const omq_selfplay_step_config* cfg, float komi,
                                    int32_t area_scoring, int8_t* d_history, int32_t* d_meta, uint64_t* d_keys,
                                    int32_t* d_nkeys, int32_t* d_game, int32_t* d_actions, int32_t* d_moves_hist,
                                    int32_t* d_visits_hist, float* d_values_hist, int8_t* d_states_hist,
                                    void* stream) {
  if (!e || !cfg || !d_history || !d_meta || !d_keys || !d_nkeys || !d_game || !d_actions || !d_moves_hist ||
      !d_visits_hist || !d_values_hist || !d_states_hist) {
    set_error("null argument");
    return OMQ_BAD_ARG;
  }
  if (e->v.game != OMQ_GAME_GO) { set_error("omq_selfplay_move_go on a non-Go engine"); return OMQ_BAD_ARG; }
  const omq_selfplay_step_config c = *cfg;
  if (c.move_number < 0 || c.move_number >= c.max_moves || !(c.temperature == 0.0f || c.temperature == 1.0f)) {
    set_error("bad self-play step (move %d of %d, temperature %g: 0 or 1 on the device)", c.move_number,
              c.max_moves, (double)c.temperature);
    return OMQ_BAD_ARG;
  }
  DeviceGuard g(e->cfg.device);
  count_launches(1);
  k_selfplay_move_go<<<e->v.R, kSelfplayThreads, 0, (cudaStream_t)stream>>>(
      e->v, c, komi, area_scoring, d_history, d_meta, d_keys, d_nkeys, d_game, d_actions, d_moves_hist,
      d_visits_hist, d_values_hist, d_states_hist);
  return cuda_status(cudaGetLastError(), "k_selfplay_move_go");
}
