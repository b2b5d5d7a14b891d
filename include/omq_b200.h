/*
 * omq_b200.h - C ABI of the B200-native wave-MCTS hot path (libomq_b200.so).
 *
 * Plain pointers, sizes and a caller-supplied cudaStream_t (passed as void*); no C++ or torch
 * types cross this boundary. Every function returns an omq_status. Device pointers are marked
 * d_; host pointers h_. Kernels launch on the given stream and never synchronize it unless the
 * comment says so (functions that report a device-side status read it back and therefore
 * synchronize that stream).
 *
 * Reference interfaces replaced (paths relative to the reference project):
 *   - pybind module mcts_cuda_kernels (python/mcts/gpu/mcts_kernels.cu:2342-2409) and
 *     fused_mcts_kernel.cu:252-254: per-op tensor kernels with silent early returns
 *     (mcts_kernels.cu:1437-1443). Here: explicit status codes, caller streams.
 *   - CSRTree / NodeDataManager storage (python/mcts/gpu/csr_tree.py:37-86,
 *     node_data_manager.py:88-113): device-resident trees owned by an omq_engine.
 *   - WaveSearch.run_wave (python/mcts/core/wave_search.py:555-615): omq_wave_* phases.
 *   - RequestBatchingCoordinator / GPUEvaluatorService (python/mcts/utils/
 *     batch_evaluation_coordinator.py:48-500): the engine's on-device leaf queues.
 *   - ResNetModel.forward (python/mcts/neural_networks/resnet_model.py:247-271) under
 *     ResNetEvaluator._forward_model (resnet_evaluator.py:231-265): omq_resnet_forward.
 */
#ifndef OMQ_B200_H
#define OMQ_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define OMQ_API __attribute__((visibility("default")))
#else
#define OMQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  OMQ_OK = 0,
  OMQ_TREE_FULL = 1,       /* capacity exhausted (reference: "Tree full", csr_tree.py:405) */
  OMQ_QUEUE_OVERFLOW = 2,  /* a per-wave scratch list overflowed (visit log, leaf queue) */
  OMQ_TIMEOUT = 3,         /* a bounded device wait ran out */
  OMQ_BAD_ARG = 4,
  OMQ_CUDA_ERROR = 5,
  OMQ_NOT_READY = 6        /* phase called out of order */
} omq_status;

/* Which on-device leaf queue an evaluation call refers to. */
typedef enum {
  OMQ_QUEUE_EXPAND = 0, /* leaves to expand: policy + value wanted (wave_search.py:866-871) */
  OMQ_QUEUE_FINAL = 1   /* picked children: value wanted (wave_search.py:1337-1457) */
} omq_queue;

/* Game of an engine. Gomoku: actions = n*n, 19 feature planes (the reference's basic
 * representation). Go: actions = n*n + 1 (pass last, the reference's NN action space for Go),
 * 17 feature planes; rules of GoState (src/games/go/go_state.cpp:227-420, 502-506): Chinese
 * rules with positional superko (go_superko), or Japanese / Korean rules (go_cycle). Chess:
 * the rules of the reference's ChessState, standard or Chess960. */
typedef enum {
  OMQ_GAME_GOMOKU = 0,
  OMQ_GAME_GO = 1,
  OMQ_GAME_CHESS = 2  /* board_size 8; 4672 actions (8x8x73, mover's frame); 119 planes */
} omq_game;

typedef struct omq_engine omq_engine;

/* omq_reroot modes. */
#define OMQ_REROOT_CARRY 1  /* next root starts with the chosen child's visit count and value sum */
#define OMQ_REROOT_KEEP 2   /* keep the chosen child's whole subtree */

typedef struct {
  int32_t num_trees;        /* independent trees searched in lockstep (one root each) */
  int32_t board_size;       /* Gomoku: 15 */
  int32_t capacity;         /* nodes per tree (reference max_tree_nodes / initial_tree_nodes) */
  int32_t max_wave_size;    /* simulations per wave (reference MCTSConfig.max_wave_size) */
  int32_t max_depth;        /* path buffer width (reference wave_search.py:414, 100) */
  float c_puct;
  float virtual_loss;       /* positive; applied as -|virtual_loss| (mcts.py:643) */
  int32_t enable_virtual_loss;
  int32_t device;           /* CUDA device ordinal */
  /* Root Dirichlet noise (wave_search.py:1160-1170): when dirichlet_epsilon > 0, every wave's
   * root selection mixes one fresh Dirichlet(alpha) vector into the root priors,
   * P' = (1 - eps) * P + eps * noise. Drawn on the device from a counter-based generator keyed by
   * (noise_seed, search, wave, tree, child); 0 disables. */
  float dirichlet_alpha;
  float dirichlet_epsilon;
  uint64_t noise_seed;
  int32_t game;             /* omq_game */
  /* Go: positional superko (GoState::isLegalMove with enforce_superko, go_state.cpp:359-418, the
   * reference's default): a move is refused when the position it makes - board after captures
   * plus the new ko point - has the key of a position recorded after an earlier non-pass move of
   * the game (the root's history keys, see omq_begin_go) or of the path from the root. Keys are
   * 64-bit Zobrist hashes: XOR over stones of mix64(0x6A09E667F3BCC909 ^ (cell * 4 + colour)),
   * ^ mix64(0xBB67AE8584CAA73B ^ ko) with a ko point (mix64 = the SplitMix64 finaliser). */
  int32_t go_superko;
  /* Go: Japanese / Korean repetition rule (GoState::makeMove, go_state.cpp:342-356; isTerminal
   * :502-513): a position - board, ko point and side to move, key ^ mix64(0x3C6EF372FE94F82B ^
   * side) - reached for the third time (counting every move, passes included) ends the game.
   * With go_cycle the root keys passed to omq_begin_go are those of every move of the game.
   * The reference turns superko off under these rules; set go_superko = 0 with go_cycle = 1. */
  int32_t go_cycle;
} omq_engine_config;

OMQ_API const char* omq_status_string(int status);
OMQ_API const char* omq_last_error(void); /* thread-local detail for the last non-OK status */
/* Number of kernels this library has launched in the calling process so far. */
OMQ_API int omq_kernel_launches(uint64_t* h_count);
/* sizeof(omq_engine_config) and sizeof(omq_resnet_config) as this library was compiled: a binding
 * checks its own struct declarations against them (host only, no device needed). */
OMQ_API int omq_abi_struct_sizes(uint32_t* h_engine_config, uint32_t* h_resnet_config);
/* Adjust that count by delta: a CUDA graph capture records launches without running them (-n),
 * each replay of the graph runs them (+n). */
OMQ_API int omq_kernel_launches_add(int64_t delta);

/* Allocates all device memory of the engine (trees + per-wave scratch + queues).
 * Replaces CSRTree(CSRTreeConfig) (csr_tree.py:86) and WaveSearch.allocate_buffers (:414). */
OMQ_API int omq_engine_create(const omq_engine_config* cfg, omq_engine** out);
OMQ_API int omq_engine_destroy(omq_engine* e);
/* Bytes of device memory held by the engine. */
OMQ_API int omq_engine_memory(const omq_engine* e, uint64_t* h_bytes);

/* Between searches: tree r's root child reached by the move d_actions[r] (int32 [num_trees], the
 * engine's action space; -1 = none) becomes the root of the next search, which must begin from
 * the position that move leads to. Replaces MCTS.update_root with subtree reuse
 * (mcts.py:1205-1246). OMQ_REROOT_CARRY restates what the reference's use_gpu_tree_reuse path
 * (mcts.py:1929-2005, compact_subtree.py:195-313) leaves behind: a fresh tree whose root starts
 * with the child's visit count and value sum. OMQ_REROOT_KEEP keeps the child's subtree,
 * renumbered breadth-first with children in action order - what CSRTree.shift_root
 * (csr_tree.py:1020-1229) describes, which the reference never reaches (its call raises and the
 * tree is reset); a kept root that is already expanded is not expanded again. A move that is not
 * a root child, or a tree with an error status, gives a fresh tree. Mode KEEP allocates (once)
 * node copies for a chunk of trees, about 1 GiB at most. */
OMQ_API int omq_reroot(omq_engine* e, const int32_t* d_actions, int mode, void* stream);

/* Reset every tree and set its root from d_boards[num_trees][n][n] (int8, 0/1/2); the side to
 * move is black when the stone count is even (mcts.py:1509-1519). Queues the roots for their
 * forced expansion (mcts.py:1659-1691): evaluate OMQ_QUEUE_EXPAND, then call
 * omq_root_expand. */
OMQ_API int omq_begin(omq_engine* e, const int8_t* d_boards, void* stream);
/* Chess engines: reset every tree and set its root from d_records, 80-byte position records
 * [num_trees][101] (record 0 = the root, records 1..100 = the game's earlier positions, most
 * recent first; layout: int8 squares[64] (rank 0 = the eighth rank; 0 empty, piece type 1..6 =
 * P N B R Q K, +8 for black), int8 side (1 white, 2 black), int8 castling bits (1 K, 2 Q, 4 k,
 * 8 q), int8 en-passant square (-1 none), int8 occurrences of the position so far, int16 halfmove
 * clock, int16 fullmove number, int8 Chess960 flag, int8 original rook files [4] (white kingside,
 * white queenside, black kingside, black queenside; 7 0 7 0 in standard chess), 3 pad bytes) and
 * d_nprior int32 [num_trees] (earlier positions present).
 * Replaces MCTS._initialize_root for GameType.CHESS (mcts.py:1495-1519) with the rules of the
 * reference's ChessState (chess_state.cpp, chess_rules.cpp) in place of the placeholder
 * gpu_game_states.py:397-405. A node's terminal status is found when it is first expanded. */
OMQ_API int omq_begin_chess(omq_engine* e, const void* d_records, const int32_t* d_nprior,
                            void* stream);
/* Go engines: reset every tree and set its root from d_history int8 [num_trees][8][n][n]
 * (index 0 = the root position, index k = the position k plies earlier, all-zero before the
 * game started; they feed the 17 history planes) and d_meta int32 [num_trees][3] = {side to move
 * (1 black, 2 white), ko point (-1 none), consecutive passes}. Replaces MCTS._initialize_root
 * for GameType.GO (mcts.py:1495-1519), which takes the GoState. Then as omq_begin. */
OMQ_API int omq_begin_go(omq_engine* e, const int8_t* d_history, const int32_t* d_meta,
                         const uint64_t* d_keys, const int32_t* d_nkeys, void* stream);
/* d_keys uint64 [num_trees][OMQ_GO_MAX_KEYS] and d_nkeys int32 [num_trees] (both may be NULL):
 * the position keys of each root's game so far, one per non-pass move, for superko. When a game
 * has more, pass its most recent OMQ_GO_MAX_KEYS. */
#define OMQ_GO_MAX_KEYS 512
OMQ_API int omq_root_expand(omq_engine* e, void* stream);

/* One wave of `wave_size` simulations in every tree (wave_search.py:555-615), in phases:
 *   omq_wave_select  : selection with virtual loss (wave_search.py:711-777, 1104-1335) and the
 *                      expansion queue (unique leaves, ascending node id per tree);
 *   <evaluate OMQ_QUEUE_EXPAND>
 *   omq_wave_expand  : children in action order, prefix-scan child ids (wave_search.py:779-979,
 *                      csr_tree.py:391-449), child pick (wave_search.py:981-1102) and the final
 *                      queue;
 *   <evaluate OMQ_QUEUE_FINAL>
 *   omq_wave_backup  : sign-alternating backup in the reference's per-simulation order
 *                      (mcts_gpu_accelerator.py:378-393) and virtual-loss revert
 *                      (wave_search.py:1513-1552). */
OMQ_API int omq_wave_select(omq_engine* e, int32_t wave_size, void* stream);
OMQ_API int omq_wave_expand(omq_engine* e, void* stream);
OMQ_API int omq_wave_backup(omq_engine* e, void* stream);

/* Device buffers of a leaf queue: entries int32 [cap][2] = {tree, node}; policy fp32
 * [cap][actions] (probabilities, as evaluate_batch returns them); value fp32 [cap]; and the
 * device int32 entry count. An external evaluator fills policy/value for the first count
 * entries. */
OMQ_API int omq_queue_buffers(omq_engine* e, int32_t queue, int32_t** d_entries, float** d_policy,
                      float** d_value, int32_t** d_count, int32_t* h_capacity);
/* Synchronizes the stream and returns the entry count. */
OMQ_API int omq_queue_count(omq_engine* e, int32_t queue, int32_t* h_count, void* stream);

/* Feature tensor of the queue entries into d_out (capacity rows): Gomoku, the reference's
 * (gpu_game_states.py:534-600) fp32 [count][19][n][n]; Go, fp32 [count][17][n][n] with planes
 * 0-7 the side to move's stones now and 1..7 plies ago, 8-15 the opponent's, 16 all ones when
 * black is to move; chess, fp32 [count][119][8][8] in the mover's frame: for k = 0..7 plies ago
 * planes 14k+0..5 the mover's P N B R Q K, 14k+6..11 the opponent's, 14k+12/13 position seen
 * >= 2 / >= 3 times; then white to move, fullmove / 100, mover's castling K/Q, opponent's K/Q,
 * halfmove / 100. */
OMQ_API int omq_queue_features(omq_engine* e, int32_t queue, float* d_out, void* stream);
/* Built-in integer-exact synthetic evaluator on the queue (policy for OMQ_QUEUE_EXPAND, value
 * for both). */
OMQ_API int omq_queue_eval_synthetic(omq_engine* e, int32_t queue, void* stream);

/* Whole search with the built-in synthetic evaluator: omq_search with net == NULL (begin, forced
 * root expansion and ceil(num_simulations / max_wave_size) waves, mcts.py:1020-1063).
 * Synchronizes the stream once at the end to report device status. */
OMQ_API int omq_search_synthetic(omq_engine* e, const int8_t* d_boards, int32_t num_simulations,
                         void* stream);
/* The same for chess engines, with the roots of omq_begin_chess. */
OMQ_API int omq_search_synthetic_chess(omq_engine* e, const void* d_records, const int32_t* d_nprior,
                                       int32_t num_simulations, void* stream);
/* The same for Go engines, with the roots of omq_begin_go. */
OMQ_API int omq_search_synthetic_go(omq_engine* e, const int8_t* d_history, const int32_t* d_meta,
                                    const uint64_t* d_keys, const int32_t* d_nkeys,
                                    int32_t num_simulations, void* stream);

/* Root statistics: visit counts of the root's children scattered by action,
 * d_visits int32 [num_trees][actions] (0 for illegal actions), and the root's own N and W
 * (d_root_nw float [num_trees][2]). Replaces tree_ops.get_root_children_info
 * (tree_operations.py:154-187). */
OMQ_API int omq_root_visits(omq_engine* e, int32_t* d_visits, float* d_root_nw, void* stream);

/* The Dirichlet noise the last wave mixed into each root's priors, scattered by action:
 * d_noise fp32 [num_trees][actions] (0 where the root has no child or noise is off). */
OMQ_API int omq_root_noise(omq_engine* e, float* d_noise, void* stream);

/* Device status word and node count of each tree: d_status int32 [num_trees],
 * d_num_nodes int32 [num_trees]. */
OMQ_API int omq_tree_status(omq_engine* e, int32_t* d_status, int32_t* d_num_nodes, void* stream);

/* Node arrays of tree `tree` in creation order, `count` nodes from index 0 (the layout the
 * reference's NodeDataManager holds: visit_counts, value_sums, node_priors,
 * virtual_loss_counts, parent_indices, parent_actions). Any pointer may be NULL. */
OMQ_API int omq_export_tree(omq_engine* e, int32_t tree, int32_t count, int32_t* d_visits,
                    float* d_value_sums, float* d_priors, int32_t* d_virtual_loss,
                    int32_t* d_parent, int32_t* d_action, uint8_t* d_terminal, void* stream);

/* One self-play move of every game on the device (Gomoku; chess and Go below), after a search of all the engine's
 * trees, tree g = game g (SelfPlayGame.play_single_move, self_play_manager.py:218-370). */
typedef struct {
  int32_t move_number;            /* 0-based index of this move in every game */
  int32_t max_moves;              /* history rows per game in the arrays below */
  int32_t temperature_threshold;  /* sample while move_number < this, arg-max afterwards */
  float temperature;              /* 1: sample in proportion to the visit counts; 0: arg-max */
  int32_t enable_resign;
  int32_t resign_min_move;        /* resignation only when move_number + 1 > this */
  float resign_threshold;         /* the player who moved resigns when the root value < this */
  uint64_t seed;                  /* draws: hash(seed, game, move), see selfplay.counter_draw */
} omq_selfplay_step_config;
/* For every live game g (d_game[8g] == 0): records the position (d_states_hist[g][move][C]),
 * the root visit counts by action (d_visits_hist[g][move][A]) and the root value W/N
 * (d_values_hist[g][move]); chooses the move (first action whose cumulative visit count exceeds
 * floor(hash / 2^64 * total) while sampling; the first most-visited action otherwise), plays it on
 * d_boards[g], writes it to d_moves_hist[g][move] and d_actions[g] (-1 for finished games, the
 * input of omq_reroot for subtree reuse), and updates d_game[g][8] = {finished, winner (+1
 * black, -1 white, 0 draw), resigned, error, moves played, 0, 0, 0}. No host synchronisation. */
OMQ_API int omq_selfplay_move(omq_engine* e, const omq_selfplay_step_config* cfg, int8_t* d_boards,
                              int32_t* d_game, int32_t* d_actions, int32_t* d_moves_hist,
                              int32_t* d_visits_hist, float* d_values_hist, int8_t* d_states_hist,
                              void* stream);
/* The same step for chess engines, on the roots of omq_search_chess: d_records [G][1 + 100]
 * 80-byte position records (the position, then the earlier ones, most recent first) and d_nprior
 * int32 [G], both updated in place so that they are the next search's roots; d_states_hist
 * [G][max_moves] records of the searched positions (8-byte aligned, as d_records). The move is
 * played as ChessState::makeMove (chess_state.cpp:1232-1346) and the game ends as
 * ChessState::getGameResult (chess_state.cpp:623-676); d_game[g][1] is +1 white, -1 black, 0
 * draw. An action that is not a legal move ends the game with d_game[g][3] = OMQ_BAD_ARG. */
OMQ_API int omq_selfplay_move_chess(omq_engine* e, const omq_selfplay_step_config* cfg, void* d_records,
                                    int32_t* d_nprior, int32_t* d_game, int32_t* d_actions,
                                    int32_t* d_moves_hist, int32_t* d_visits_hist, float* d_values_hist,
                                    void* d_states_hist, void* stream);
/* The same step for Go engines, on the roots of omq_search_go, updated in place as the next
 * search's roots: d_history int8 [G][8][n][n], d_meta int32 [G][3] = {side to move, ko point,
 * consecutive passes}, d_keys uint64 [G][OMQ_GO_MAX_KEYS] with d_nkeys int32 [G] the game's
 * position keys in game order (a full list drops its oldest key). The move is played as
 * GoState::makeMove (go_state.cpp:227-356; captures, ko point, superko refusal under the engine's
 * go_superko, the repetition rule under go_cycle). Two consecutive passes end the game, scored
 * by area (area_scoring = 1, Chinese) or by territory and prisoners (0, Japanese / Korean) with
 * `komi` for white (go_rules.cpp:211-260, 343-380); a third repetition ends it with winner 0.
 * d_game[g] = {finished, winner (+1 black, -1 white, 0), resigned, error, moves played, black's
 * prisoners, white's prisoners, ended by repetition}; d_states_hist [G][max_moves][8][n][n]. */
OMQ_API int omq_selfplay_move_go(omq_engine* e, const omq_selfplay_step_config* cfg, float komi,
                                 int32_t area_scoring, int8_t* d_history, int32_t* d_meta, uint64_t* d_keys,
                                 int32_t* d_nkeys, int32_t* d_game, int32_t* d_actions, int32_t* d_moves_hist,
                                 int32_t* d_visits_hist, float* d_values_hist, int8_t* d_states_hist,
                                 void* stream);


/* ---------------------------------------------------------------------------------------------
 * ResNet policy/value evaluator (reference: ResNetModel, python/mcts/neural_networks/
 * resnet_model.py:26-271; ResNetEvaluator._forward_model, resnet_evaluator.py:231-265).
 * bf16 weights/activations, fp32 accumulation, BatchNorm folded (eval mode).
 * ------------------------------------------------------------------------------------------- */
typedef struct omq_resnet omq_resnet;

typedef struct {
  int32_t board_size;        /* 15 Gomoku */
  int32_t input_channels;    /* feature planes: 19 Gomoku, 17 Go, 119 chess; <= 128 */
  int32_t num_blocks;        /* residual blocks */
  int32_t filters;           /* 128 or 256 */
  int32_t num_actions;       /* policy size (225 Gomoku, 362 Go 19x19, 4672 chess), <= 5000 */
  int32_t fc_policy_hidden;  /* PolicyHead fc1 width (reference default 256) */
  int32_t fc_value_hidden;   /* ValueHead fc1 width (reference default 256) */
  int32_t max_batch;         /* positions per forward call (activation buffers are sized for it) */
  int32_t device;
  int32_t dtype;             /* OMQ_DTYPE_BF16 (0, default) or OMQ_DTYPE_F16: the 16-bit type of the
                                conv weights, activations and dense-layer operands (fp32 accumulate);
                                F16 is the precision of the reference evaluator's fp16 autocast */
  int32_t trunk_per_layer;   /* 0 (default): the whole trunk in one kernel where it applies (15x15
                                boards, 128 filters); 1: one launch per conv everywhere (same
                                results; for comparisons) */
} omq_resnet_config;

enum { OMQ_DTYPE_BF16 = 0, OMQ_DTYPE_F16 = 1 };

OMQ_API int omq_resnet_create(const omq_resnet_config* cfg, omq_resnet** out);
OMQ_API int omq_resnet_destroy(omq_resnet* net);
OMQ_API int omq_resnet_memory(const omq_resnet* net, uint64_t* h_bytes);
/* Kernel launches of the convolution trunk per forward call: 1 when the whole trunk runs as one
 * kernel (15x15 boards with 128 filters: every conv of a position in one CTA), else 1 + 2 x
 * num_blocks (one per conv). */
OMQ_API int omq_resnet_trunk_launches(const omq_resnet* net, int32_t* h_launches);
/* Element counts of the three packed parameter blobs omq_resnet_load expects:
 *  conv_w (16-bit, the config's dtype): input conv [F][9][Cin_pad] (input channels zero-padded to 64, or to 128 for
 *                 more than 64 planes), then per block
 *                 conv1 [F][9][F], conv2 [F][9][F]; K index = tap * Cin + channel, tap = 3*ky+kx;
 *                 BatchNorm scale folded in.
 *  conv_b (fp32): folded BatchNorm shift, [1 + 2*num_blocks][F].
 *  head   (fp32): w1x1 [3][F] (policy ch0, policy ch1, value), b1x1 [3], policy fc1^T [2*HW][Hp],
 *                 b [Hp], policy fc2^T [Hp][A], b [A], value fc1^T [HW][Hv], b [Hv],
 *                 value fc2 [Hv], b [1]. */
OMQ_API int omq_resnet_param_sizes(const omq_resnet* net, uint64_t* conv_w, uint64_t* conv_b,
                                   uint64_t* head);
/* Copies the blobs in. When the fully connected widths allow it (policy fc1 width a multiple of
 * 64, value fc1 width <= 256, a multiple of 16) the heads then run on the tensor cores from bf16
 * copies of the fc weights made here; otherwise (and in omq_resnet_forward_noalloc) in fp32. */
OMQ_API int omq_resnet_load(omq_resnet* net, const uint16_t* d_conv_w, const float* d_conv_b,
                            const float* d_head, void* stream);
/* Forward on reference-layout features fp32 [batch][input_channels][n][n]
 * -> policy probabilities fp32 [batch][num_actions], value fp32 [batch]. */
OMQ_API int omq_resnet_forward_features(omq_resnet* net, const float* d_features, int32_t batch,
                                        float* d_policy, float* d_value, void* stream);
/* Forward on an already packed bf16 input [batch][(n+1)^2][64] (the padded pixel layout; NULL
 * = the net's own input buffer). The batch is *d_count when d_count is not NULL (clamped to
 * `batch`), which keeps the call free of host synchronisation. */
OMQ_API int omq_resnet_forward_packed(omq_resnet* net, const uint16_t* d_input,
                                      const int32_t* d_count, int32_t batch, float* d_policy,
                                      float* d_value, void* stream);
OMQ_API int omq_resnet_input_buffer(omq_resnet* net, uint16_t** d_input);
/* Evaluate an engine leaf queue in place: the queued positions are packed on the device and
 * the queue's policy/value buffers are written; no host synchronisation. Queue 1 (the final
 * nodes, whose policies the search never reads: wave_search.py:1337-1457 keeps only the values)
 * gets its values only; its policy buffer is left as it was. */
OMQ_API int omq_resnet_forward_queue(omq_resnet* net, omq_engine* engine, int32_t queue,
                                     void* stream);
/* Whole search in one call, the native counterpart of MCTS.search / _run_search
 * (python/mcts/core/mcts.py:924-979, 1020-1063; mcts_search in the survey's C-ABI list): begin
 * on the roots, forced root expansion, then ceil(num_simulations / max_wave_size) waves of
 * select / evaluate / expand / evaluate / backup, every evaluation done by `net` on the engine's
 * leaf queues in place (net == NULL: the built-in synthetic evaluator). The net's max_batch must
 * cover the engine's queue capacity (num_trees x max_wave_size), and its board size, planes and
 * actions must be the engine's. Synchronizes the stream once, at the end, to report the trees'
 * status (OMQ_TREE_FULL, ...). Roots as for omq_begin / omq_begin_go / omq_begin_chess. */
OMQ_API int omq_search(omq_engine* e, omq_resnet* net, const int8_t* d_boards, int32_t num_simulations,
                       void* stream);
OMQ_API int omq_search_go(omq_engine* e, omq_resnet* net, const int8_t* d_history, const int32_t* d_meta,
                          const uint64_t* d_keys, const int32_t* d_nkeys, int32_t num_simulations,
                          void* stream);
OMQ_API int omq_search_chess(omq_engine* e, omq_resnet* net, const void* d_records,
                             const int32_t* d_nprior, int32_t num_simulations, void* stream);
/* Record CUDA events around the convolution trunk of the next `capacity` forward calls
 * (0 disables; re-arming resets). omq_resnet_profile_read synchronizes on the last event and
 * returns, per call, the trunk's device time in ms and the number of positions evaluated. */
OMQ_API int omq_resnet_profile(omq_resnet* net, int32_t capacity);
OMQ_API int omq_resnet_profile_read(omq_resnet* net, int32_t* h_calls, float* h_trunk_ms,
                                    int32_t* h_counts, int32_t max);
/* ResNet forward that allocates nothing (no counterpart in the reference). For callers that must
 * not let a library allocate device memory: a process whose own allocator owns the whole device
 * heap, or a latency-critical thread where cudaMalloc/cudaFree would synchronise the device.
 * Same computation as omq_resnet_forward_features, but the caller passes the packed parameter
 * blobs (layouts as for omq_resnet_load), the features and the outputs, and the activations live
 * in one fixed 8 MiB device array built into the library, held by every GPU that loads it until
 * the process exits. Batches beyond what that array holds (36 positions at 128 filters, 19 at
 * 256, for 15x15) are rejected with OMQ_BAD_ARG. The first call on a device looks up the
 * array's device address; make that first call before any stream capture. All calls share the
 * array: calls that overlap on the GPU (other streams, other threads) race and must be
 * serialised by the caller. */
OMQ_API int omq_resnet_forward_noalloc(const omq_resnet_config* cfg, const uint16_t* d_conv_w,
                                       const float* d_conv_b, const float* d_head,
                                       const float* d_features, int32_t batch, float* d_policy,
                                       float* d_value, void* stream);
/* Error word of the last omq_resnet_forward_noalloc call on `device`: OMQ_OK, or OMQ_TIMEOUT when
 * a kernel's bounded wait gave up (the outputs of that call are then incomplete). Waits for the
 * work queued on `stream` and allocates nothing (no counterpart in the reference; the companion
 * of omq_resnet_forward_noalloc). The next forward clears the word. */
OMQ_API int omq_resnet_noalloc_error(int32_t device, int32_t* h_error, void* stream);
/* Self-test of the bounded device waits: launches a kernel whose mbarrier wait can never complete;
 * after limit_ns (at most 1 s) it gives up and writes OMQ_TIMEOUT to d_status (int32, device). */
OMQ_API int omq_selftest_wait_timeout(uint64_t limit_ns, int32_t* d_status, void* stream);
/* Self-test of the sum behind the prior normalisation p / (sum(p) + 1e-8) that expansion runs
 * (wave_search.py:894-895, summed in torch's CPU order): writes the sum of each segment
 * d_x[d_offsets[s] .. d_offsets[s+1]) to d_out[s] (device pointers; no counterpart in the
 * reference, which has no device sum of its own). */
OMQ_API int omq_selftest_prior_sum(const float* d_x, const int32_t* d_offsets, int32_t segments,
                                   float* d_out, void* stream);
/* Device error word of the net (OMQ_TIMEOUT after a bounded wait gave up); synchronizes. */
OMQ_API int omq_resnet_error(omq_resnet* net, int32_t* h_error, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* OMQ_B200_H */
