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

// Positional superko (GoState with enforce_superko, go_state.cpp:359-418): a move is refused when
// the position it makes - board after captures plus the new ko point - equals one recorded after
// an earlier non-pass move of the game (position_history_, pushed at :333). Positions are keyed by
// a 64-bit Zobrist hash: stone keys mix64(0x6A09E667F3BCC909 ^ (cell * 4 + colour)) and ko keys
// mix64(0xBB67AE8584CAA73B ^ cell), the keys the device engine uses.
uint64_t go_key(const int8_t* b, int n, int ko);
// go_legal minus the moves whose resulting key is in hist[0..nhist).
void go_legal_superko(const int8_t* b, int n, int player, int ko, const uint64_t* hist, int nhist,
                      uint8_t* mask);

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
uint64_t oracle_go_key(const int8_t* b, int n, int ko);
void oracle_go_legal_superko(const int8_t* b, int n, int player, int ko, const uint64_t* hist,
                             int nhist, uint8_t* mask);
}
