// Parity oracle (TEST INFRASTRUCTURE ONLY). Integer-exact synthetic evaluator; the definition is
// spelled out in synth_eval.h. Follows the evaluator protocol of the reference
// (python/mcts/core/wave_search.py:867-871 policy call, :1381-1383 value call).
#include "synth_eval.h"
#include <vector>

namespace oracle {

// round(2^(i/64) * 2^20), i = 0..63 (exact decimal evaluation; no entry is within 1e-6 of a tie).
const uint32_t kExp2Table[64] = {
    1048576u,1059994u,1071537u,1083205u,1095000u,1106924u,1118978u,1131163u,1143480u,1155932u,
    1168519u,1181244u,1194106u,1207109u,1220254u,1233542u,1246974u,1260553u,1274279u,1288155u,
    1302182u,1316362u,1330696u,1345187u,1359835u,1374642u,1389611u,1404743u,1420040u,1435503u,
    1451135u,1466937u,1482910u,1499058u,1515382u,1531883u,1548564u,1565427u,1582474u,1599706u,
    1617125u,1634735u,1652536u,1670531u,1688722u,1707110u,1725700u,1744491u,1763488u,1782691u,
    1802103u,1821727u,1841564u,1861617u,1881889u,1902381u,1923097u,1944038u,1965207u,1986607u,
    2008240u,2030108u,2052214u,2074562u};

static const uint64_t kHashSeed = 0x243F6A8885A308D3ull;
static const uint64_t kGolden = 0x9E3779B97F4A7C15ull;
static const uint64_t kValueSalt = 0xD1B54A32D192ED03ull;

uint64_t mix64(uint64_t x) {  // SplitMix64 finaliser (Steele, Lea & Flood 2014)
  x ^= x >> 30; x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 27; x *= 0x94D049BB133111EBull;
  x ^= x >> 31;
  return x;
}

// Irwin-Hall(4) draw folded to an exponent step t = floor(z * log2(e) * 64), z ~ N(0,1) approx.
static int64_t exp_step(uint64_t r) {
  int64_t s = (int64_t)(r & 0xFFFF) + (int64_t)((r >> 16) & 0xFFFF) +
              (int64_t)((r >> 32) & 0xFFFF) + (int64_t)((r >> 48) & 0xFFFF) - 131072;
  return (s * 160) >> 16;  // arithmetic shift = floor division
}

// 2^(t/64) scaled by 2^26.
static uint64_t exp2_fixed(int64_t t) {
  return (uint64_t)kExp2Table[t & 63] << ((t >> 6) + 6);
}

void synth_from_hash(uint64_t h, int actions, const uint8_t* legal, float* policy, float* value) {
  std::vector<uint64_t> w(actions, 0);
  uint64_t total = 0;
  for (int a = 0; a < actions; ++a) {
    if (!legal[a]) continue;
    w[a] = exp2_fixed(exp_step(mix64(h + kGolden * (uint64_t)(a + 1))));
    total += w[a];
  }
  uint32_t idx = 0;
  for (int a = 0; a < actions; ++a) {
    if (!legal[a]) { policy[a] = 0.0f; continue; }
    uint64_t m = (w[a] * 32640ull) / total;
    uint64_t q = 512ull * m + idx++;
    policy[a] = (float)q * (1.0f / 16777216.0f);
  }
  int64_t e = (int64_t)exp2_fixed(exp_step(mix64(h ^ kValueSalt)));
  const int64_t d = (int64_t)1 << 26;
  int64_t v = ((e - d) * 4096) / (e + d);  // C++ division truncates toward zero
  *value = (float)v * (1.0f / 4096.0f);
}

}  // namespace oracle

extern "C" uint64_t oracle_feature_hash(const float* f, int planes, int cells) {
  uint64_t h = oracle::kHashSeed;
  const int words = (cells + 63) / 64;
  for (int c = 0; c < planes; ++c) {
    const float* p = f + (size_t)c * cells;
    if (c == 1) {  // player plane: constant 1.0 or 2.0
      h = oracle::mix64(h ^ (uint64_t)(int64_t)p[0]);
      continue;
    }
    for (int j = 0; j < words; ++j) {
      uint64_t word = 0;
      for (int b = 0; b < 64 && 64 * j + b < cells; ++b)
        if (p[64 * j + b] != 0.0f) word |= 1ull << b;
      h = oracle::mix64(h ^ word);
    }
  }
  return h;
}

extern "C" void oracle_synth_eval(int n, int planes, int cells, int actions, const float* features,
                                  float* policy, float* value) {
  std::vector<uint8_t> legal(actions);
  for (int i = 0; i < n; ++i) {
    const float* f = features + (size_t)i * planes * cells;
    for (int a = 0; a < actions; ++a) legal[a] = (a >= cells) || (f[a] == 0.0f);
    uint64_t h = oracle_feature_hash(f, planes, cells);
    oracle::synth_from_hash(h, actions, legal.data(), policy + (size_t)i * actions, value + i);
  }
}

extern "C" uint64_t oracle_feature_hash_go(const float* f, int cells) {
  uint64_t h = oracle::kHashSeed;
  const int words = (cells + 63) / 64;
  for (int c = 0; c < 17; ++c) {
    const float* p = f + (size_t)c * cells;
    for (int j = 0; j < words; ++j) {
      uint64_t word = 0;
      for (int b = 0; b < 64 && 64 * j + b < cells; ++b)
        if (p[64 * j + b] != 0.0f) word |= 1ull << b;
      h = oracle::mix64(h ^ word);
    }
  }
  return h;
}

extern "C" void oracle_synth_eval_go(int n, int cells, int actions, const float* features,
                                     float* policy, float* value) {
  std::vector<uint8_t> legal(actions);
  for (int i = 0; i < n; ++i) {
    const float* f = features + (size_t)i * 17 * cells;
    for (int a = 0; a < actions; ++a)
      legal[a] = (a >= cells) || (f[a] == 0.0f && f[(size_t)8 * cells + a] == 0.0f);
    uint64_t h = oracle_feature_hash_go(f, cells);
    oracle::synth_from_hash(h, actions, legal.data(), policy + (size_t)i * actions, value + i);
  }
}

extern "C" uint64_t oracle_feature_hash_chess(const float* f) {
  uint64_t h = oracle::kHashSeed;
  for (int c = 0; c < 119; ++c) {
    uint64_t word = 0;
    for (int b = 0; b < 64; ++b)
      if (f[(size_t)c * 64 + b] != 0.0f) word |= 1ull << b;
    h = oracle::mix64(h ^ word);
  }
  return h;
}

extern "C" void oracle_synth_eval_chess(int n, const float* features, float* policy, float* value) {
  std::vector<uint8_t> legal(4672, 1);
  for (int i = 0; i < n; ++i) {
    const uint64_t h = oracle_feature_hash_chess(features + (size_t)i * 119 * 64);
    oracle::synth_from_hash(h, 4672, legal.data(), policy + (size_t)i * 4672, value + i);
  }
}
