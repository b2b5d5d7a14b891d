// Parity oracle (TEST INFRASTRUCTURE ONLY). Chess rules as the reference's C++ engine implements
// them (src/games/chess/chess_state.cpp, chess_rules.cpp; standard chess, not Chess960),
// including its behaviours that differ from FIDE rules:
//   * isSquareAttacked (chess_rules.cpp:135-150) looks for an attacking pawn on the mirrored
//     side (a white pawn is looked for one rank *towards* white's promotion rank from the
//     square), so kings can step into real pawn attacks and be captured; a side without a king
//     is never in check and keeps playing;
//   * a double pawn push always sets the en-passant square (chess_state.cpp:1262-1268);
//   * the repetition key is the piece placement alone: the position hash is computed in full
//     once (updateHash, :1414-1453) and afterwards only updated for piece changes (setPiece ->
//     updateHashIncrementally, :255-267, 1455-1471), so side to move, castling rights and the
//     en-passant square never change it;
//   * terminal (ChessState::isTerminal, :623-676): no legal move (draw unless in check), then the
//     insufficient-material table of chess_rules.cpp:236-394, then halfmove clock >= 100, then
//     the position's third occurrence.
// Chess960 (the reference's chess960_ mode): castling takes the king two files towards the rook
// (king file +- 2, chess_rules.cpp:619-680, 735-749) and puts the rook on the king's other side
// (chess_state.cpp:1296-1312); the original rook files come from the start position. Where
// king file +- 2 leaves the board (king on the b- or g-file) the reference computes an off-board
// target; no such castling move is generated here.
// Squares are rank * 8 + file with rank 0 = the eighth rank (black's back rank); white pawns move
// towards rank 0. Moves use the reference encoding (promotion << 12) | (from << 6) | to with
// promotion 1 queen, 2 rook, 3 bishop, 4 knight (chess_state.cpp:1474-1507).
#pragma once
#include <cstdint>

extern "C" {
// Position record shared with the device engine (80 bytes).
typedef struct {
  int8_t sq[64];     // 0 empty; piece type 1..6 (P N B R Q K), +8 for black
  int8_t side;       // 1 white, 2 black
  int8_t castle;     // 1 white kingside, 2 white queenside, 4 black kingside, 8 black queenside
  int8_t ep;         // en-passant square or -1
  int8_t reps;       // occurrences of this position so far, itself included (repetition planes)
  int16_t halfmove;
  int16_t fullmove;
  int8_t c960;       // Chess960 castling (the reference's chess960_ flag)
  int8_t rook_file[4];  // original rook files: white kingside, white queenside, black k, black q
  int8_t pad[3];
} oracle_chess_pos;

int oracle_chess_from_fen(const char* fen, oracle_chess_pos* out);  // 0 ok
// The same for a Chess960 game: castling letters may name rook files (Shredder FEN).
int oracle_chess_from_fen960(const char* fen, oracle_chess_pos* out);
// Legal moves (reference encoding) into moves[256]; returns the count.
int oracle_chess_legal(const oracle_chess_pos* p, int32_t* moves);
// ChessState::makeMove (chess_state.cpp:1232-1346) for a move of the reference encoding.
void oracle_chess_play(oracle_chess_pos* p, int32_t move);
// Terminal test with `reps` occurrences of the position (itself included); *result is the
// reference's GameResult (0 ongoing, 1 white wins, 2 black wins, 3 draw).
int oracle_chess_terminal(const oracle_chess_pos* p, int reps, int* result);
// Same position for repetition purposes: the piece placement (see above).
int oracle_chess_same(const oracle_chess_pos* a, const oracle_chess_pos* b);

// Engine action space: 4672 = 64 from-squares x 73 move planes (AlphaZero encoding), in the
// mover's frame (ranks mirrored for black). Plane: queen-like moves dir * 7 + (distance - 1)
// with dir 0..7 = N, NE, E, SE, S, SW, W, NW (N = towards the mover's promotion rank), knight
// moves 56 + k, under-promotions 64 + 3 * (knight 0, bishop 1, rook 2) + (file step + 1).
// Queen promotions use the queen-like planes. Action = from_in_frame * 73 + plane.
int oracle_chess_action(const oracle_chess_pos* p, int32_t move);  // -> 0..4671
int32_t oracle_chess_move(const oracle_chess_pos* p, int action);  // inverse

// Network input, 119 planes of 8x8 in the mover's frame: for k = 0..7 (k plies ago, zeros where
// hist[k] is null) planes 14k + 0..5 the mover's P N B R Q K, 14k + 6..11 the opponent's,
// 14k + 12 reps >= 2, 14k + 13 reps >= 3; then 112 white to move, 113 fullmove / 100,
// 114/115 mover's kingside/queenside right, 116/117 opponent's, 118 halfmove / 100.
void oracle_chess_features(const oracle_chess_pos* const* hist, float* out);
}

namespace oracle {
constexpr int kChessActions = 4672;
constexpr int kChessPlanes = 119;
}
