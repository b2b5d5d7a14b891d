// Parity oracle (TEST INFRASTRUCTURE ONLY - never linked into the product library).
//
// Deterministic synthetic evaluator used by the parity gate (benchmark config 0):
// "policy logits ~N(0,1) over the actions, seeded by a 64-bit hash of the position, masked to
// legal moves and softmaxed; value = tanh of a hash-seeded N(0,0.5) draw".
//
// The evaluator is defined on the reference's feature tensor (the only thing the reference's
// evaluator protocol sees: python/mcts/core/wave_search.py:867-871, 1381-1383) and is built from
// integer arithmetic only, so that numpy (reference harness), this C file and the CUDA kernels
// produce bit-identical outputs:
//   * hash   : SplitMix64 finaliser folded over the binarised feature planes (plane 1, the
//              player plane, is folded in as its integer value instead);
//   * normal : Irwin-Hall sum of four 16-bit uniforms -> exponent step t (1/64 octave units);
//   * exp    : 2^(t/64) from a 64-entry integer table;
//   * policy : weights quantised to q_a = 512*m_a + idx_a (idx_a = rank of a among legal moves),
//              so every legal prior is distinct and every partial sum is an exact fp32 integer
//              multiple of 2^-24 (the reference's priors.sum() is then order-independent);
//   * value  : tanh(z/2) = (e^z-1)/(e^z+1) on a 2^-12 grid, so fp32 value sums are exact for
//              |W| < 4096 in any summation order.
#pragma once
#include <cstdint>

extern "C" {
uint64_t oracle_feature_hash(const float* features, int planes, int cells);
// features [n, planes, cells] fp32 -> policy [n, actions] fp32 (0 on illegal), value [n] fp32.
// Legal = plane-0 cell empty (Gomoku/Go board actions); actions beyond `cells` count as legal.
void oracle_synth_eval(int n, int planes, int cells, int actions, const float* features,
                       float* policy, float* value);
// Go variant on the 17-plane Go features [n, 17, cells]: the hash folds all 17 planes binarised
// (no special plane), and the legal set is the empty points (planes 0 and 8 clear) plus pass
// (action == cells). Expansion renormalises over the rules' legal set afterwards.
uint64_t oracle_feature_hash_go(const float* features, int cells);
void oracle_synth_eval_go(int n, int cells, int actions, const float* features, float* policy,
                          float* value);
// Chess variant on the 119-plane features [n, 119, 64]: the hash folds all 119 planes binarised
// (value != 0), one 64-bit word per plane; the policy covers all 4672 actions (the features do
// not carry legality; expansion renormalises over the legal moves).
uint64_t oracle_feature_hash_chess(const float* features);
void oracle_synth_eval_chess(int n, const float* features, float* policy, float* value);
}

namespace oracle {
uint64_t mix64(uint64_t x);
// Evaluate one position given its hash and legal mask (used by the oracle directly).
void synth_from_hash(uint64_t h, int actions, const uint8_t* legal, float* policy, float* value);
extern const uint32_t kExp2Table[64];
}
