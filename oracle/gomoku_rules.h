// Parity oracle (TEST INFRASTRUCTURE ONLY). Gomoku state rules and the reference's basic
// 19-plane feature encoding, restated from python/mcts/gpu/gpu_game_states.py and
// python/mcts/utils/fast_terminal_check.py.
#pragma once
#include <cstdint>

namespace oracle {
constexpr int kPlanes = 19;
constexpr int kFullHistoryGomoku = 250;  // gpu_game_states.py:157 (max_game_length)

// fast_terminal_check.py:233-332: five (or more) in a row of one player anywhere, or a full board.
bool gomoku_terminal(const int8_t* board, int size);

// gpu_game_states.py:534-600 (basic representation). Child states never inherit the parent's
// full_move_history (clone_states copies it only with enhanced features, :325-327), so a state
// created by apply_moves holds exactly one history entry: its own last move at index
// move_count-1 (:443-446). The clamp of :568 is reproduced, including the artefact that
// repeats that entry for move_count == 1. last_action < 0 marks the root (no history written).
void gomoku_features(const int8_t* board, int size, int player, int move_count, int last_action,
                     float* out /* [19, size*size] */);
}  // namespace oracle
