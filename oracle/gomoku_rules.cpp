// Parity oracle (TEST INFRASTRUCTURE ONLY). See gomoku_rules.h.
#include "gomoku_rules.h"
#include <cstring>

namespace oracle {

bool gomoku_terminal(const int8_t* b, int n) {
  static const int dr[4] = {0, 1, 1, 1}, dc[4] = {1, 0, 1, -1};
  bool full = true;
  for (int r = 0; r < n; ++r)
    for (int c = 0; c < n; ++c) {
      int p = b[r * n + c];
      if (p == 0) { full = false; continue; }
      for (int d = 0; d < 4; ++d) {
        int k = 1;
        for (; k < 5; ++k) {
          int rr = r + dr[d] * k, cc = c + dc[d] * k;
          if (rr < 0 || rr >= n || cc < 0 || cc >= n || b[rr * n + cc] != p) break;
        }
        if (k == 5) return true;
      }
    }
  return full;
}

void gomoku_features(const int8_t* b, int n, int player, int mc, int last_action, float* out) {
  const int cells = n * n;
  std::memset(out, 0, sizeof(float) * kPlanes * cells);
  for (int i = 0; i < cells; ++i) out[i] = b[i] != 0 ? 1.0f : 0.0f;
  for (int i = 0; i < cells; ++i) out[cells + i] = (float)player;
  for (int k = 0; k < 8; ++k) {
    int idx = mc - 1 - k;
    if (idx < 0) idx = 0;
    if (idx > kFullHistoryGomoku - 1) idx = kFullHistoryGomoku - 1;
    if (!(idx < mc)) continue;
    int mv = (last_action >= 0 && idx == mc - 1) ? last_action : -1;
    if (mv < 0) continue;
    int ch = (k % 2 == 0) ? 2 + k / 2 : 10 + k / 2;
    out[(size_t)ch * cells + mv] = 1.0f;
  }
}

}  // namespace oracle
