// Parity oracle (TEST INFRASTRUCTURE ONLY). Go rules restated from the reference's C++ engine
// (src/games/go/go_state.cpp, go_rules.cpp) with Chinese rules and positional superko off:
// captures of opponent groups left without liberties (go_state.cpp:283-316), no suicide
// (go_rules.cpp:34-110), simple ko - a move that captures exactly one stone forbids the
// immediate play on that point (go_state.cpp:318-321, 371-374) - and pass always legal.
// Actions are y * n + x; action n * n is pass.
#pragma once
#include <cstdint>

namespace oracle {
// Plays `action` for `player` on board b (n x n). Returns false (and leaves out untouched) if the
// move is illegal. ko: the current ko point or -1. ko_out: the ko point after the move.
bool go_play(const int8_t* b, int n, int player, int action, int ko, int8_t* out, int* ko_out);
// mask[n * n + 1]: legal actions of `player` (pass included).
void go_legal(const int8_t* b, int n, int player, int ko, uint8_t* mask);

// Network input for Go, 17 planes of `cells` (AlphaGo Zero layout; the reference has no Go
// encoding of this size, so this is the engine's own definition): plane k (k = 0..7) holds the
// side to move's stones k plies ago, plane 8 + k the opponent's, plane 16 is 1 when black
// (player 1) is to move. hist[k] is the board k plies before the position (all-zero boards
// before the game started).
constexpr int kGoPlanes = 17;
void go_features(const int8_t* const* hist, int cells, int to_move, float* out);
}  // namespace oracle

extern "C" {
// ctypes entry points for the rule tests
int oracle_go_play(const int8_t* b, int n, int player, int action, int ko, int8_t* out, int* ko_out);
void oracle_go_legal(const int8_t* b, int n, int player, int ko, uint8_t* mask);
}
