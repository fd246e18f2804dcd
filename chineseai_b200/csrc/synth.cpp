// synth.cpp - deterministic synthetic workloads for the evaluator (host).
//
// The generator is the reference's SplitMix64 (src/az.rs:3146-3176): each draw
// replaces the state by splitmix64(state), so the stream is a chain of mixes,
// not the usual counter-based SplitMix64.  unit() follows SplitMix64::unit_f32
// (53 high bits scaled into [0,1)).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "../../include/cnnue.h"

namespace {

inline uint64_t mix(uint64_t value) {
  value += 0x9E3779B97F4A7C15ull;
  uint64_t m = value;
  m = (m ^ (m >> 30)) * 0xBF58476D1CE4E5B9ull;
  m = (m ^ (m >> 27)) * 0x94D049BB133111EBull;
  return m ^ (m >> 31);
}

struct Rng {
  uint64_t state;
  uint64_t next() {
    state = mix(state);
    return state;
  }
  uint32_t below(uint32_t bound) { return (uint32_t)(next() % bound); }
  double unit53() { return (double)(next() >> 11) * (1.0 / 9007199254740992.0); }
  // Box-Muller, one normal per two draws.
  double normal() {
    const double u1 = ((double)(next() >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    const double u2 = unit53();
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
  }
};

// n unique values uniform in [0, bound), sorted ascending, appended to out.
void unique_sorted(Rng& rng, uint32_t n, uint32_t bound, std::vector<uint8_t>& mark,
                   uint16_t* out) {
  uint32_t got = 0;
  while (got < n) {
    const uint32_t v = rng.below(bound);
    if (mark[v]) continue;
    mark[v] = 1;
    out[got++] = (uint16_t)v;
  }
  std::sort(out, out + n);
  for (uint32_t i = 0; i < n; ++i) mark[out[i]] = 0;
}

}  // namespace

extern "C" {

uint64_t cnnue_splitmix64_next(uint64_t* state) {
  *state = mix(*state);
  return *state;
}

int cnnue_synth_positions(uint64_t seed, int64_t n_positions, uint32_t n_features,
                          uint32_t min_active, uint32_t max_active, uint16_t* h_indices,
                          uint32_t* h_offsets, uint32_t* n_indices) {
  if (n_positions < 0 || !h_offsets || !n_indices || n_features == 0 || n_features > 65536 ||
      min_active > max_active || max_active > n_features || (n_positions > 0 && !h_indices))
    return CNNUE_ERR_INVALID_ARG;
  Rng rng{seed};
  std::vector<uint8_t> mark(n_features, 0);
  uint32_t pos = 0;
  h_offsets[0] = 0;
  for (int64_t p = 0; p < n_positions; ++p) {
    for (int s = 0; s < 2; ++s) {
      const uint32_t n = min_active + rng.below(max_active - min_active + 1);
      unique_sorted(rng, n, n_features, mark, h_indices + pos);
      pos += n;
      h_offsets[2 * p + s + 1] = pos;
    }
  }
  *n_indices = pos;
  return CNNUE_OK;
}

int cnnue_synth_q_weights(uint64_t seed, int16_t* ft_weight, int16_t* ft_bias, int8_t* l1_weight,
                          int32_t* l1_bias, int8_t* l2_weight, int32_t* l2_bias,
                          int8_t* l3_weight, int32_t* l3_bias) {
  if (!ft_weight || !ft_bias || !l1_weight || !l1_bias || !l2_weight || !l2_bias || !l3_weight ||
      !l3_bias)
    return CNNUE_ERR_INVALID_ARG;
  Rng rng{seed};
  for (size_t i = 0; i < (size_t)CNNUE_Q_FEATURES * CNNUE_Q_COLS; ++i)
    ft_weight[i] = (int16_t)((int)rng.below(255) - 127);
  for (int i = 0; i < CNNUE_Q_COLS; ++i) ft_bias[i] = (int16_t)((int)rng.below(129) - 64);
  for (int i = 0; i < CNNUE_Q_BUCKETS * CNNUE_Q_L1 * CNNUE_Q_PACKED; ++i)
    l1_weight[i] = (int8_t)((int)rng.below(129) - 64);
  for (int i = 0; i < CNNUE_Q_BUCKETS * CNNUE_Q_L1; ++i) l1_bias[i] = (int)rng.below(129) - 64;
  for (int i = 0; i < CNNUE_Q_BUCKETS * CNNUE_Q_L2 * CNNUE_Q_L1; ++i)
    l2_weight[i] = (int8_t)((int)rng.below(129) - 64);
  for (int i = 0; i < CNNUE_Q_BUCKETS * CNNUE_Q_L2; ++i) l2_bias[i] = (int)rng.below(129) - 64;
  for (int i = 0; i < CNNUE_Q_BUCKETS * CNNUE_Q_L2; ++i)
    l3_weight[i] = (int8_t)((int)rng.below(129) - 64);
  for (int i = 0; i < CNNUE_Q_BUCKETS; ++i) l3_bias[i] = (int)rng.below(129) - 64;
  return CNNUE_OK;
}

int cnnue_synth_f_weights(uint64_t seed, float* ft_weight, float* ft_bias, float* l1_weight,
                          float* l1_bias, float* l2_weight, float* l2_bias, float* l3_weight,
                          float* l3_bias) {
  if (!ft_weight || !ft_bias || !l1_weight || !l1_bias || !l2_weight || !l2_bias || !l3_weight ||
      !l3_bias)
    return CNNUE_ERR_INVALID_ARG;
  Rng rng{seed};
  for (size_t i = 0; i < (size_t)CNNUE_F_FEATURES * CNNUE_F_COLS; ++i)
    ft_weight[i] = (float)(0.01 * rng.normal());
  for (int i = 0; i < CNNUE_F_COLS; ++i) ft_bias[i] = 0.f;
  for (int i = 0; i < CNNUE_F_BUCKETS * 16 * 2 * CNNUE_F_COLS; ++i)
    l1_weight[i] = (float)(0.05 * rng.normal());
  for (int i = 0; i < CNNUE_F_BUCKETS * 16; ++i) l1_bias[i] = 0.f;
  for (int i = 0; i < CNNUE_F_BUCKETS * 32 * 16; ++i) l2_weight[i] = (float)(0.05 * rng.normal());
  for (int i = 0; i < CNNUE_F_BUCKETS * 32; ++i) l2_bias[i] = 0.f;
  for (int i = 0; i < CNNUE_F_BUCKETS * 32; ++i) l3_weight[i] = (float)(0.05 * rng.normal());
  for (int i = 0; i < CNNUE_F_BUCKETS; ++i) l3_bias[i] = 0.f;
  return CNNUE_OK;
}

int cnnue_synth_q_update(uint64_t seed, int64_t n_positions, int16_t* h_parent, uint8_t* h_flags,
                         uint16_t* h_rem, uint32_t* h_rem_offsets, uint32_t* n_rem,
                         uint16_t* h_add, uint32_t* h_add_offsets, uint32_t* n_add,
                         uint8_t* h_count0) {
  if (n_positions < 0 || !h_rem_offsets || !h_add_offsets || !n_rem || !n_add ||
      (n_positions > 0 && (!h_parent || !h_flags || !h_rem || !h_add || !h_count0)))
    return CNNUE_ERR_INVALID_ARG;
  Rng rng{seed};
  std::vector<uint8_t> mark(CNNUE_Q_FEATURES, 0);
  uint32_t nr = 0, na = 0;
  h_rem_offsets[0] = 0;
  h_add_offsets[0] = 0;
  for (int64_t p = 0; p < n_positions; ++p) {
    int16_t* par = h_parent + (size_t)p * 2 * CNNUE_Q_COLS;
    for (int j = 0; j < 2 * CNNUE_Q_COLS; ++j) par[j] = (int16_t)((int)rng.below(4001) - 2000);
    uint32_t child0 = 0;
    for (int s = 0; s < 2; ++s) {
      const int64_t ps = 2 * p + s;
      const bool refresh = rng.below(20) == 0;
      h_flags[ps] = refresh ? 1 : 0;
      uint32_t r = 0, a = 0;
      if (refresh) {
        a = 2 + rng.below(31);
        unique_sorted(rng, a, CNNUE_Q_FEATURES, mark, h_add + na);
        na += a;
      } else {
        r = 1 + rng.below(2);
        for (uint32_t i = 0; i < r; ++i) h_rem[nr++] = (uint16_t)rng.below(CNNUE_Q_FEATURES);
        a = 1 + rng.below(3);
        for (uint32_t i = 0; i < a; ++i) h_add[na++] = (uint16_t)rng.below(CNNUE_Q_FEATURES);
      }
      h_rem_offsets[ps + 1] = nr;
      h_add_offsets[ps + 1] = na;
      if (s == 0) {
        const uint32_t parent0 = 2 + rng.below(31);
        child0 = refresh ? a : parent0 - r + a;
      }
    }
    h_count0[p] = (uint8_t)child0;
  }
  *n_rem = nr;
  *n_add = na;
  return CNNUE_OK;
}

// bf16 value of f, round to nearest even (finite inputs).
static float bf16_value(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  u &= 0xffff0000u;
  std::memcpy(&f, &u, 4);
  return f;
}

int cnnue_synth_rn_weights(uint64_t seed, float* stem_w, float* stem_b, float* block_w, float* block_b,
                           float* policy_conv_w, float* policy_conv_b, float* policy_fc_w, float* policy_fc_b,
                           float* value_conv_w, float* value_conv_b, float* value_fc1_w, float* value_fc1_b,
                           float* value_fc2_w, float* value_fc2_b) {
  if (!stem_w || !stem_b || !block_w || !block_b || !policy_conv_w || !policy_conv_b || !policy_fc_w ||
      !policy_fc_b || !value_conv_w || !value_conv_b || !value_fc1_w || !value_fc1_b || !value_fc2_w ||
      !value_fc2_b)
    return CNNUE_ERR_INVALID_ARG;
  Rng rng{seed};
  auto fill = [&](float* dst, size_t n, double std) {
    for (size_t i = 0; i < n; ++i) dst[i] = bf16_value((float)(rng.normal() * std));
  };
  const int C = CNNUE_RN_CHANNELS;
  fill(stem_w, (size_t)C * CNNUE_RN_PLANES * 9, std::sqrt(2.0 / (CNNUE_RN_PLANES * 9)));
  fill(stem_b, C, 0.02);
  for (int j = 0; j < 2 * CNNUE_RN_BLOCKS; ++j)
    fill(block_w + (size_t)j * C * C * 9, (size_t)C * C * 9, std::sqrt(2.0 / (C * 9)) * (j % 2 ? 0.25 : 1.0));
  fill(block_b, (size_t)2 * CNNUE_RN_BLOCKS * C, 0.02);
  fill(policy_conv_w, 2 * C, std::sqrt(2.0 / C));
  fill(policy_conv_b, 2, 0.02);
  fill(policy_fc_w, (size_t)CNNUE_RN_MOVES * 180, std::sqrt(1.0 / 180));
  fill(policy_fc_b, CNNUE_RN_MOVES, 0.02);
  fill(value_conv_w, C, std::sqrt(2.0 / C));
  fill(value_conv_b, 1, 0.02);
  fill(value_fc1_w, (size_t)256 * 90, std::sqrt(1.0 / 90));
  fill(value_fc1_b, 256, 0.02);
  fill(value_fc2_w, 256, std::sqrt(1.0 / 256));
  fill(value_fc2_b, 1, 0.02);
  return CNNUE_OK;
}

int cnnue_synth_rn_planes(uint64_t seed, int64_t batch, uint16_t* planes) {
  if (batch < 0 || (batch > 0 && !planes)) return CNNUE_ERR_INVALID_ARG;
  std::memset(planes, 0, sizeof(uint16_t) * (size_t)batch * CNNUE_RN_PLANES * 90);
  Rng rng{seed};
  const uint16_t one = 0x3f80;  // bf16 1.0
  for (int64_t b = 0; b < batch; ++b) {
    uint16_t* pl = planes + (size_t)b * CNNUE_RN_PLANES * 90;
    bool used[90] = {};
    const uint32_t k = rng.below(33);
    for (uint32_t i = 0; i < k; ++i) {
      uint32_t sq = rng.below(90);
      while (used[sq]) sq = (sq + 1) % 90;
      used[sq] = true;
      pl[rng.below(14) * 90 + sq] = one;
    }
    if (rng.below(2))
      for (int sq = 0; sq < 90; ++sq) pl[14 * 90 + sq] = one;
  }
  return CNNUE_OK;
}

}  // extern "C"
