// Parity oracle - TEST INFRASTRUCTURE ONLY.
//
// A plain C++ restatement of the reference's deterministic CPU search path:
//   MCTS(MCTSConfig(backend='gpu', device='cpu', wave_async_expansion=False, dirichlet_epsilon=0,
//        enable_subtree_reuse=False, ...)).search(board)
// i.e. torch WaveSearch + CSRTree + GPUGameStates on the host. Only tests/, bench.py's CPU
// baseline leg and __graft_entry__.smoke() may load this library, and only as the checker.
// The product library never links or calls it.
//
// Each step cites the reference function it follows (paths relative to the reference project):
//   search driver  python/mcts/core/mcts.py:924-979, 1020-1063 (wave loop), 1069-1137 (policy)
//   root init      python/mcts/core/mcts.py:1495-1519 (numpy branch), 1659-1691 (force expand)
//   selection      python/mcts/core/wave_search.py:711-777, 1104-1335 (fallback branch 1279-1333)
//   expansion      python/mcts/core/wave_search.py:779-979; python/mcts/gpu/csr_tree.py:391-449
//   child pick     python/mcts/core/wave_search.py:981-1102
//   evaluation     python/mcts/core/wave_search.py:1337-1457
//   backup         python/mcts/gpu/mcts_gpu_accelerator.py:378-393
//   VL revert      python/mcts/core/wave_search.py:1513-1552; node_data_manager.py:366-390
#pragma once
#include <cstdint>

#include "chess_rules.h"

extern "C" {

// Evaluator callback: features [n, planes, cells] fp32 -> policy [n, actions], value [n].
typedef void (*oracle_eval_fn)(void* ctx, int n, const float* features, float* policy,
                               float* value);

typedef struct {
  int board_size;        // 15 for Gomoku
  int num_simulations;
  int max_wave_size;
  float c_puct;
  float virtual_loss;    // positive; applied as -|virtual_loss| (mcts.py:643)
  int enable_virtual_loss;
  int max_nodes;         // tree (and state pool) capacity
  int max_depth;         // paths buffer width (wave_search.py:414, default 100)
} oracle_config;

typedef struct {
  int status;            // 0 ok, 1 tree full, 2 bad argument
  int num_nodes;
  int waves;
  int boundary_ties;     // equal scores straddling a rank-assignment boundary (order-defined)
  int order_ties;        // equal scores among ranks that received simulations
  int eval_calls;
  long long eval_positions;
} oracle_result;

void* oracle_tree_create(int max_nodes, int board_size);
void oracle_tree_destroy(void* tree);

// Reset + root init + forced root expansion (mcts.py:947-949, 981-1018). eval == NULL selects
// the built-in synthetic evaluator.
int oracle_begin(void* tree, const oracle_config* cfg, const int8_t* root_board,
                 oracle_eval_fn eval, void* ctx);
// One run_wave(wave_size) (wave_search.py:555-615).
int oracle_wave(void* tree, int wave_size);
// Root Dirichlet noise for the next oracle_wave only (wave_search.py:1160-1170): the root's
// priors become keep * P + eps * noise[action] in fp32, where keep is (float)(1 - (double)eps) as
// the reference computes it in Python. Used to replay the noise a device run drew.
int oracle_set_root_noise(void* tree, float eps, float keep, const float* noise_by_action);
// Go root (go_rules.h): hist [8][board_size^2] (hist[0] = root position, hist[k] = k plies
// earlier), side to move, ko point (-1 none), consecutive passes. Actions = cells + 1 (pass last).
// Children are the rules' legal moves; a child whose pass makes two in a row is terminal.
int oracle_begin_go(void* tree, const oracle_config* cfg, const int8_t* hist, int to_move, int ko,
                    int passes, oracle_eval_fn eval, void* ctx);
// With positional superko (superko != 0): keys[0..nkeys) are the game's position keys recorded
// after each non-pass move before the root (go_rules.h go_key); inside the tree every position
// reached by a non-pass move is added along its path.
int oracle_begin_go_sk(void* tree, const oracle_config* cfg, const int8_t* hist, int to_move, int ko,
                       int passes, const uint64_t* keys, int nkeys, int superko,
                       oracle_eval_fn eval, void* ctx);
// With the Japanese / Korean repetition rule (cycle != 0): keys are those of every move of the
// game (board, ko point, side to move: go_key ^ mix64(0x3C6EF372FE94F82B ^ side)); a child whose
// position occurs for the third time (root keys + path) is terminal.
int oracle_begin_go_rules(void* tree, const oracle_config* cfg, const int8_t* hist, int to_move,
                          int ko, int passes, const uint64_t* keys, int nkeys, int superko,
                          int cycle, oracle_eval_fn eval, void* ctx);
int oracle_search_go(void* tree, const oracle_config* cfg, const int8_t* hist, int to_move, int ko,
                     int passes, oracle_eval_fn eval, void* ctx, oracle_result* out);
// Chess root (chess_rules.h): the root record (reps = occurrences so far, itself included) and
// the game's earlier positions, most recent first (history planes, repetition count). Board
// size 8; actions 4672 (the engine's AlphaZero encoding); children in ascending action order;
// a node's terminal status is found when it is first expanded (it then gets no children).
int oracle_begin_chess(void* tree, const oracle_config* cfg, const oracle_chess_pos* root,
                       const oracle_chess_pos* prior, int nprior, oracle_eval_fn eval, void* ctx);
// Action count of the last begun game (cells for Gomoku, cells + 1 for Go).
int oracle_actions(void* tree);
// Between searches: the root child reached by `action` becomes the next begin's root (which must
// be the position that move leads to). mode 1 keeps the child's visit count and value sum on a
// fresh root; mode 2 keeps its subtree in breadth-first order. Returns the mode applied (0: the
// move is not a root child, fresh tree).
int oracle_reroot(void* tree, int action, int mode);
// Full search = begin + ceil(sims / max_wave_size) waves.
int oracle_search(void* tree, const oracle_config* cfg, const int8_t* root_board,
                  oracle_eval_fn eval, void* ctx, oracle_result* out);
void oracle_get_result(void* tree, oracle_result* out);

// Node arrays (length num_nodes). Any pointer may be NULL.
int oracle_export(void* tree, int32_t* visits, float* value_sums, float* priors,
                  int32_t* virtual_loss, int32_t* parent, int32_t* action, uint8_t* terminal);
// Root policy N_child / sum N_child in fp64 over oracle_actions() actions (mcts.py:1069-1137).
int oracle_root_policy(void* tree, double* policy);
}
