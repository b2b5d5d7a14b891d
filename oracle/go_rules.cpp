// Parity oracle (TEST INFRASTRUCTURE ONLY). See go_rules.h.
#include "go_rules.h"
#include "synth_eval.h"

#include <cstring>
#include <vector>

namespace oracle {
namespace {

// Stones of the group at p and whether it has a liberty (flood fill).
bool group_has_liberty(const int8_t* b, int n, int p, std::vector<int>* stones) {
  const int color = b[p];
  std::vector<char> seen(n * n, 0);
  std::vector<int> stack{p};
  seen[p] = 1;
  bool lib = false;
  while (!stack.empty()) {
    const int c = stack.back();
    stack.pop_back();
    if (stones) stones->push_back(c);
    const int y = c / n, x = c % n;
    const int nb[4] = {y > 0 ? c - n : -1, y < n - 1 ? c + n : -1, x > 0 ? c - 1 : -1, x < n - 1 ? c + 1 : -1};
    for (int q : nb) {
      if (q < 0 || seen[q]) continue;
      if (b[q] == 0) { lib = true; continue; }
      if (b[q] == color) { seen[q] = 1; stack.push_back(q); }
    }
  }
  return lib;
}

}  // namespace

bool go_play(const int8_t* b, int n, int player, int action, int ko, int8_t* out, int* ko_out) {
  const int cells = n * n;
  if (action == cells) {  // pass clears the ko point (go_state.cpp:278-283)
    std::memcpy(out, b, cells);
    *ko_out = -1;
    return true;
  }
  if (action < 0 || action > cells || b[action] != 0 || action == ko) return false;
  std::vector<int8_t> t(b, b + cells);
  t[action] = (int8_t)player;
  const int opp = 3 - player;
  const int y = action / n, x = action % n;
  const int nb[4] = {y > 0 ? action - n : -1, y < n - 1 ? action + n : -1,
                     x > 0 ? action - 1 : -1, x < n - 1 ? action + 1 : -1};
  int groups = 0, captured = 0, last = -1;
  for (int q : nb) {
    if (q < 0 || t[q] != opp) continue;
    std::vector<int> stones;
    if (!group_has_liberty(t.data(), n, q, &stones)) {
      ++groups;
      captured += (int)stones.size();
      for (int s : stones) t[s] = 0;
      last = stones[0];
    }
  }
  if (captured == 0 && !group_has_liberty(t.data(), n, action, nullptr)) return false;  // suicide
  std::memcpy(out, t.data(), cells);
  *ko_out = (groups == 1 && captured == 1) ? last : -1;
  return true;
}

void go_legal(const int8_t* b, int n, int player, int ko, uint8_t* mask) {
  const int cells = n * n;
  std::vector<int8_t> tmp(cells);
  int k;
  for (int a = 0; a < cells; ++a) mask[a] = go_play(b, n, player, a, ko, tmp.data(), &k) ? 1 : 0;
  mask[cells] = 1;
}

uint64_t go_key(const int8_t* b, int n, int ko) {
  uint64_t k = 0;
  for (int c = 0; c < n * n; ++c)
    if (b[c]) k ^= mix64(0x6A09E667F3BCC909ull ^ (uint64_t)(c * 4 + b[c]));
  if (ko >= 0) k ^= mix64(0xBB67AE8584CAA73Bull ^ (uint64_t)ko);
  return k;
}

void go_legal_superko(const int8_t* b, int n, int player, int ko, const uint64_t* hist, int nhist,
                      uint8_t* mask) {
  go_legal(b, n, player, ko, mask);
  std::vector<int8_t> t(n * n);
  for (int a = 0; a < n * n; ++a) {
    if (!mask[a]) continue;
    int k2 = -1;
    go_play(b, n, player, a, ko, t.data(), &k2);
    const uint64_t key = go_key(t.data(), n, k2);
    for (int i = 0; i < nhist; ++i)
      if (hist[i] == key) { mask[a] = 0; break; }
  }
}

void go_features(const int8_t* const* hist, int cells, int to_move, float* out) {
  const int opp = 3 - to_move;
  for (int k = 0; k < 8; ++k)
    for (int c = 0; c < cells; ++c) {
      out[(size_t)k * cells + c] = hist[k][c] == to_move ? 1.0f : 0.0f;
      out[(size_t)(8 + k) * cells + c] = hist[k][c] == opp ? 1.0f : 0.0f;
    }
  for (int c = 0; c < cells; ++c) out[(size_t)16 * cells + c] = to_move == 1 ? 1.0f : 0.0f;
}

}  // namespace oracle

extern "C" int oracle_go_play(const int8_t* b, int n, int player, int action, int ko, int8_t* out,
                              int* ko_out) {
  return oracle::go_play(b, n, player, action, ko, out, ko_out) ? 1 : 0;
}

extern "C" void oracle_go_legal(const int8_t* b, int n, int player, int ko, uint8_t* mask) {
  oracle::go_legal(b, n, player, ko, mask);
}

extern "C" uint64_t oracle_go_key(const int8_t* b, int n, int ko) { return oracle::go_key(b, n, ko); }

extern "C" void oracle_go_legal_superko(const int8_t* b, int n, int player, int ko,
                                        const uint64_t* hist, int nhist, uint8_t* mask) {
  oracle::go_legal_superko(b, n, player, ko, hist, nhist, mask);
}
