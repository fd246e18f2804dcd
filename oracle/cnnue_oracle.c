/*
 * cnnue_oracle.c - CPU oracle for the NNUE evaluation hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the CUDA library is
 * compared against (tests/, the smoke check and bench.py's CPU-baseline leg).
 * It is never linked into the product library and the product never falls
 * back to it.
 *
 * Two halves:
 *
 * (1) Reference-native restatements, pinned to the reference's own code and
 *     tests (mycve/chineseai, Rust; cannot be compiled here - no cargo):
 *       oracle_feature_pool_fwd  <- FeaturePool::cpu_fwd
 *                                   src/az/fused_feature_pool.rs:169-198,
 *                                   item_rows :389-403
 *       oracle_feature_pool_bwd  <- FeaturePoolGrad::cpu_fwd
 *                                   src/az/fused_feature_pool.rs:231-260
 *       oracle_sparse_pool_fwd/bwd <- SparsePool / SparsePoolGrad cpu_fwd
 *                                   src/az/fused_feature_pool.rs:284-309, :342-370
 *     These are pinned against the reference tests' fixtures
 *     (src/az/fused_feature_pool.rs:611-686) in tests/test_oracle_pool.py.
 *       oracle_policy_fused_fwd/bwd <- FusedPolicy / FusedPolicyGrad cpu_fwd
 *                                   src/az/fused_policy.rs:178-241, :287-366
 *       oracle_policy_table_fwd/bwd <- SparsePolicy / SparsePolicyGrad cpu_fwd
 *                                   src/az/fused_sparse_policy.rs:86-107, :138-165
 *     The fused policy twin is checked against the reference test's inputs
 *     (src/az/fused_policy.rs:536-572) by hand-derived values in
 *     tests/test_oracle_policy.py.
 *
 * (2) The quantised and fp32 HalfKA networks.  The reference has no code for
 *     them (it has neither an int16 FT nor a pairwise pack nor bucket stacks);
 *     they are restated from the workload specification only, so their parity
 *     is UNPINNED by the reference.  Conventions fixed here (the specification
 *     leaves them open):
 *       - one FT table serves both perspectives; acc = bias + sum of rows with
 *         int16 wraparound (arithmetic mod 2^16);
 *       - pack: for perspective s and j < 512,
 *           u8[s*512 + j] = (clamp(acc_s[j],0,127) * clamp(acc_s[j+512],0,127)) >> 7
 *         (perspective 0 = side to move first);
 *       - bucket = min((max(n0,1) - 1) >> 1, 15) with n0 the perspective-0
 *         active count (16 buckets; 8 buckets with >> 2 for fp32);
 *       - L1 1024->16 int32 + bias, >> 6 (arithmetic), clamp [0,127];
 *         L2 16->32 the same; L3 32->1 int32 + bias, no shift;
 *       - fp32: clipped ReLU [0,1] on FT output and between layers, FT sum in
 *         index order starting from the bias.
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#ifdef __AVX2__
#include <immintrin.h>
#endif
#endif

#define Q_F 11340
#define Q_COLS 1024
#define Q_HALF 512
#define Q_NB 16
#define Q_L1 16
#define Q_L2 32

#define F_COLS 256
#define F_NB 8

static inline int32_t clampi(int32_t v, int32_t lo, int32_t hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}
static inline float clampf(float v, float lo, float hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}

int oracle_q_bucket(uint32_t n0) {
  uint32_t n = n0 < 1 ? 1 : n0;
  uint32_t b = (n - 1) >> 1;
  return (int)(b > 15 ? 15 : b);
}

int oracle_f_bucket(uint32_t n0) {
  uint32_t n = n0 < 1 ? 1 : n0;
  uint32_t b = (n - 1) >> 2;
  return (int)(b > 7 ? 7 : b);
}

/* acc[j] = bias[j] + sum rows, int16 wraparound. Returns 0, or 2 on a bad index. */
static int q_accumulate(const int16_t* ft, const int16_t* bias, const uint16_t* idx, uint32_t n,
                        int16_t* acc) {
  int status = 0;
  uint16_t tmp[Q_COLS];
  for (int j = 0; j < Q_COLS; ++j) tmp[j] = (uint16_t)bias[j];
  for (uint32_t i = 0; i < n; ++i) {
    uint32_t f = idx[i];
    if (f >= Q_F) { status = 2; continue; }
    const int16_t* row = ft + (size_t)f * Q_COLS;
    for (int j = 0; j < Q_COLS; ++j) tmp[j] = (uint16_t)(tmp[j] + (uint16_t)row[j]);
  }
  memcpy(acc, tmp, sizeof(tmp));
  return status;
}

static void q_pack(const int16_t* acc, uint8_t* out512) {
  for (int j = 0; j < Q_HALF; ++j) {
    int32_t a = clampi(acc[j], 0, 127);
    int32_t b = clampi(acc[j + Q_HALF], 0, 127);
    out512[j] = (uint8_t)((a * b) >> 7);
  }
}

static int32_t q_stack(const uint8_t* x, int bucket, const int8_t* l1w, const int32_t* l1b,
                       const int8_t* l2w, const int32_t* l2b, const int8_t* l3w,
                       const int32_t* l3b) {
  int32_t y1[Q_L1], y2[Q_L2];
  const int8_t* w1 = l1w + (size_t)bucket * Q_L1 * Q_COLS;
  for (int k = 0; k < Q_L1; ++k) {
    int32_t s = l1b[bucket * Q_L1 + k];
    for (int i = 0; i < Q_COLS; ++i) s += (int32_t)w1[k * Q_COLS + i] * (int32_t)x[i];
    y1[k] = clampi(s >> 6, 0, 127);
  }
  const int8_t* w2 = l2w + (size_t)bucket * Q_L2 * Q_L1;
  for (int m = 0; m < Q_L2; ++m) {
    int32_t s = l2b[bucket * Q_L2 + m];
    for (int k = 0; k < Q_L1; ++k) s += (int32_t)w2[m * Q_L1 + k] * y1[k];
    y2[m] = clampi(s >> 6, 0, 127);
  }
  int32_t s = l3b[bucket];
  for (int m = 0; m < Q_L2; ++m) s += (int32_t)l3w[bucket * Q_L2 + m] * y2[m];
  return s;
}

/* Offsets check shared by the batched oracles: 0 ok, 3 bad. */
static int check_offsets(const uint32_t* offsets, int64_t n_lists, uint32_t n_indices) {
  if (offsets[0] > n_indices) return 3;
  for (int64_t i = 0; i < n_lists; ++i) {
    if (offsets[i] > offsets[i + 1] || offsets[i + 1] > n_indices) return 3;
  }
  return 0;
}

/* Quantised forward over positions [begin, end). */
static int q_forward_range(const int16_t* ft, const int16_t* bias, const int8_t* l1w,
                           const int32_t* l1b, const int8_t* l2w, const int32_t* l2b,
                           const int8_t* l3w, const int32_t* l3b, const uint16_t* idx,
                           const uint32_t* offsets, int64_t begin, int64_t end, int32_t* scores,
                           int16_t* acc_out) {
  int status = 0;
  int16_t acc[2][Q_COLS];
  uint8_t x[Q_COLS];
  for (int64_t p = begin; p < end; ++p) {
    for (int s = 0; s < 2; ++s) {
      uint32_t b = offsets[2 * p + s], e = offsets[2 * p + s + 1];
      int st = q_accumulate(ft, bias, idx + b, e - b, acc[s]);
      if (st) status = st;
      q_pack(acc[s], x + s * Q_HALF);
    }
    if (acc_out) memcpy(acc_out + (size_t)p * 2 * Q_COLS, acc, sizeof(acc));
    uint32_t n0 = offsets[2 * p + 1] - offsets[2 * p];
    scores[p] = q_stack(x, oracle_q_bucket(n0), l1w, l1b, l2w, l2b, l3w, l3b);
  }
  return status;
}

int oracle_q_forward(const int16_t* ft, const int16_t* bias, const int8_t* l1w,
                     const int32_t* l1b, const int8_t* l2w, const int32_t* l2b,
                     const int8_t* l3w, const int32_t* l3b, const uint16_t* idx,
                     uint32_t n_indices, const uint32_t* offsets, int64_t n_positions,
                     int32_t* scores, int16_t* acc_out) {
  if (n_positions <= 0) return 0;
  if (check_offsets(offsets, 2 * n_positions, n_indices)) return 3;
  return q_forward_range(ft, bias, l1w, l1b, l2w, l2b, l3w, l3b, idx, offsets, 0, n_positions,
                         scores, acc_out);
}

#ifdef __AVX2__
/* The timed CPU baseline's hand-written AVX2 path (the reference's own
 * evaluator adds int8/int16 rows with 256-bit integer adds, src/az.rs:
 * 2616-2654); every result is bit-identical to the scalar forward above.
 *   - accumulation in 4 column tiles of 256 int16: a tile lives in 16 ymm
 *     registers while every row of the list is added (_mm256_add_epi16:
 *     int16 wraparound);
 *   - pack: clamp by max/min, 16-bit products (at most 127 * 127), >> 7,
 *     unsigned saturating narrow (no saturation: results are at most 126);
 *   - L1: _mm256_maddubs_epi16 of the packed uint8 (<= 126) with the int8
 *     weights (pair sums within +-2 * 126 * 128, inside int16, so exact),
 *     _mm256_madd_epi16 with ones to int32. */
static int q_accumulate_avx2(const int16_t* ft, const int16_t* bias, const uint16_t* idx, uint32_t n,
                             int16_t* acc) {
  int status = 0;
  for (int t = 0; t < Q_COLS; t += 256) {
    __m256i r[16];
    for (int k = 0; k < 16; ++k) r[k] = _mm256_loadu_si256((const __m256i*)(bias + t + 16 * k));
    for (uint32_t i = 0; i < n; ++i) {
      const uint32_t f = idx[i];
      if (f >= Q_F) {
        status = 2;
        continue;
      }
      const int16_t* row = ft + (size_t)f * Q_COLS + t;
      for (int k = 0; k < 16; ++k) r[k] = _mm256_add_epi16(r[k], _mm256_loadu_si256((const __m256i*)(row + 16 * k)));
    }
    for (int k = 0; k < 16; ++k) _mm256_storeu_si256((__m256i*)(acc + t + 16 * k), r[k]);
  }
  return status;
}

static void q_pack_avx2(const int16_t* acc, uint8_t* out512) {
  const __m256i zero = _mm256_setzero_si256(), top = _mm256_set1_epi16(127);
  for (int j = 0; j < Q_HALF; j += 32) {
    __m256i a0 = _mm256_loadu_si256((const __m256i*)(acc + j));
    __m256i a1 = _mm256_loadu_si256((const __m256i*)(acc + j + 16));
    __m256i b0 = _mm256_loadu_si256((const __m256i*)(acc + j + Q_HALF));
    __m256i b1 = _mm256_loadu_si256((const __m256i*)(acc + j + Q_HALF + 16));
    a0 = _mm256_min_epi16(_mm256_max_epi16(a0, zero), top);
    a1 = _mm256_min_epi16(_mm256_max_epi16(a1, zero), top);
    b0 = _mm256_min_epi16(_mm256_max_epi16(b0, zero), top);
    b1 = _mm256_min_epi16(_mm256_max_epi16(b1, zero), top);
    const __m256i p0 = _mm256_srli_epi16(_mm256_mullo_epi16(a0, b0), 7);
    const __m256i p1 = _mm256_srli_epi16(_mm256_mullo_epi16(a1, b1), 7);
    /* packus interleaves the 128-bit lanes: restore the column order */
    const __m256i u8 = _mm256_permute4x64_epi64(_mm256_packus_epi16(p0, p1), 0xd8);
    _mm256_storeu_si256((__m256i*)(out512 + j), u8);
  }
}

static int32_t q_stack_avx2(const uint8_t* x, int bucket, const int8_t* l1w, const int32_t* l1b,
                            const int8_t* l2w, const int32_t* l2b, const int8_t* l3w, const int32_t* l3b) {
  int32_t y1[Q_L1], y2[Q_L2];
  const int8_t* w1 = l1w + (size_t)bucket * Q_L1 * Q_COLS;
  const __m256i ones = _mm256_set1_epi16(1);
  for (int k = 0; k < Q_L1; ++k) {
    __m256i s = _mm256_setzero_si256();
    for (int i = 0; i < Q_COLS; i += 32) {
      const __m256i xv = _mm256_loadu_si256((const __m256i*)(x + i));
      const __m256i wv = _mm256_loadu_si256((const __m256i*)(w1 + k * Q_COLS + i));
      s = _mm256_add_epi32(s, _mm256_madd_epi16(_mm256_maddubs_epi16(xv, wv), ones));
    }
    __m128i h = _mm_add_epi32(_mm256_castsi256_si128(s), _mm256_extracti128_si256(s, 1));
    h = _mm_add_epi32(h, _mm_shuffle_epi32(h, 0x4e));
    h = _mm_add_epi32(h, _mm_shuffle_epi32(h, 0xb1));
    y1[k] = clampi((l1b[bucket * Q_L1 + k] + _mm_cvtsi128_si32(h)) >> 6, 0, 127);
  }
  const int8_t* w2 = l2w + (size_t)bucket * Q_L2 * Q_L1;
  for (int m = 0; m < Q_L2; ++m) {
    int32_t s = l2b[bucket * Q_L2 + m];
    for (int k = 0; k < Q_L1; ++k) s += (int32_t)w2[m * Q_L1 + k] * y1[k];
    y2[m] = clampi(s >> 6, 0, 127);
  }
  int32_t s = l3b[bucket];
  for (int m = 0; m < Q_L2; ++m) s += (int32_t)l3w[bucket * Q_L2 + m] * y2[m];
  return s;
}

static int q_forward_range_avx2(const int16_t* ft, const int16_t* bias, const int8_t* l1w, const int32_t* l1b,
                                const int8_t* l2w, const int32_t* l2b, const int8_t* l3w, const int32_t* l3b,
                                const uint16_t* idx, const uint32_t* offsets, int64_t begin, int64_t end,
                                int32_t* scores) {
  int status = 0;
  int16_t acc[2][Q_COLS];
  uint8_t x[Q_COLS];
  for (int64_t p = begin; p < end; ++p) {
    for (int s = 0; s < 2; ++s) {
      uint32_t b = offsets[2 * p + s], e = offsets[2 * p + s + 1];
      int st = q_accumulate_avx2(ft, bias, idx + b, e - b, acc[s]);
      if (st) status = st;
      q_pack_avx2(acc[s], x + s * Q_HALF);
    }
    uint32_t n0 = offsets[2 * p + 1] - offsets[2 * p];
    scores[p] = q_stack_avx2(x, oracle_q_bucket(n0), l1w, l1b, l2w, l2b, l3w, l3b);
  }
  return status;
}
#define Q_FORWARD_RANGE_FAST(...) q_forward_range_avx2(__VA_ARGS__)
#else
#define Q_FORWARD_RANGE_FAST(...) q_forward_range(__VA_ARGS__, NULL)
#endif

int oracle_q_has_avx2(void) {
#ifdef __AVX2__
  return 1;
#else
  return 0;
#endif
}

/* Multi-threaded variant (OpenMP, static split) used as the timed CPU
 * baseline: the AVX2 path when the library is built for it. */
int oracle_q_forward_mt(const int16_t* ft, const int16_t* bias, const int8_t* l1w,
                        const int32_t* l1b, const int8_t* l2w, const int32_t* l2b,
                        const int8_t* l3w, const int32_t* l3b, const uint16_t* idx,
                        uint32_t n_indices, const uint32_t* offsets, int64_t n_positions,
                        int32_t* scores, int n_threads) {
  if (n_positions <= 0) return 0;
  if (check_offsets(offsets, 2 * n_positions, n_indices)) return 3;
  int status = 0;
#ifdef _OPENMP
  if (n_threads < 1) n_threads = omp_get_max_threads();
#pragma omp parallel num_threads(n_threads) reduction(| : status)
  {
    int t = omp_get_thread_num(), nt = omp_get_num_threads();
    int64_t chunk = (n_positions + nt - 1) / nt;
    int64_t b = t * chunk, e = b + chunk < n_positions ? b + chunk : n_positions;
    if (b < e)
      status |= Q_FORWARD_RANGE_FAST(ft, bias, l1w, l1b, l2w, l2b, l3w, l3b, idx, offsets, b, e, scores);
  }
#else
  (void)n_threads;
  status = Q_FORWARD_RANGE_FAST(ft, bias, l1w, l1b, l2w, l2b, l3w, l3b, idx, offsets, 0, n_positions, scores);
#endif
  return status;
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Incremental update + stack (the same conventions as the forward). */
static int q_update_range(const int16_t* ft, const int16_t* bias, const int8_t* l1w,
                          const int32_t* l1b, const int8_t* l2w, const int32_t* l2b,
                          const int8_t* l3w, const int32_t* l3b, const int16_t* parent,
                          const uint8_t* flags, const uint16_t* rem, const uint32_t* rem_off,
                          const uint16_t* add, const uint32_t* add_off, const uint8_t* count0,
                          int64_t begin, int64_t end, int16_t* child, int32_t* scores) {
  int status = 0;
  uint8_t x[Q_COLS];
  for (int64_t p = begin; p < end; ++p) {
    for (int s = 0; s < 2; ++s) {
      int64_t ps = 2 * p + s;
      uint16_t acc[Q_COLS];
      const int16_t* par = parent + (size_t)ps * Q_COLS;
      int refresh = flags[ps] & 1;
      for (int j = 0; j < Q_COLS; ++j) acc[j] = (uint16_t)(refresh ? bias[j] : par[j]);
      if (!refresh) {
        for (uint32_t i = rem_off[ps]; i < rem_off[ps + 1]; ++i) {
          uint32_t f = rem[i];
          if (f >= Q_F) { status = 2; continue; }
          const int16_t* row = ft + (size_t)f * Q_COLS;
          for (int j = 0; j < Q_COLS; ++j) acc[j] = (uint16_t)(acc[j] - (uint16_t)row[j]);
        }
      }
      for (uint32_t i = add_off[ps]; i < add_off[ps + 1]; ++i) {
        uint32_t f = add[i];
        if (f >= Q_F) { status = 2; continue; }
        const int16_t* row = ft + (size_t)f * Q_COLS;
        for (int j = 0; j < Q_COLS; ++j) acc[j] = (uint16_t)(acc[j] + (uint16_t)row[j]);
      }
      int16_t* out = child + (size_t)ps * Q_COLS;
      memcpy(out, acc, sizeof(acc));
      q_pack(out, x + s * Q_HALF);
    }
    scores[p] = q_stack(x, oracle_q_bucket(count0[p]), l1w, l1b, l2w, l2b, l3w, l3b);
  }
  return status;
}

int oracle_q_update(const int16_t* ft, const int16_t* bias, const int8_t* l1w, const int32_t* l1b,
                    const int8_t* l2w, const int32_t* l2b, const int8_t* l3w, const int32_t* l3b,
                    const int16_t* parent, const uint8_t* flags, const uint16_t* rem,
                    uint32_t n_rem, const uint32_t* rem_off, const uint16_t* add, uint32_t n_add,
                    const uint32_t* add_off, const uint8_t* count0, int64_t n_positions,
                    int16_t* child, int32_t* scores, int n_threads) {
  if (n_positions <= 0) return 0;
  if (check_offsets(rem_off, 2 * n_positions, n_rem)) return 3;
  if (check_offsets(add_off, 2 * n_positions, n_add)) return 3;
  int status = 0;
#ifdef _OPENMP
  if (n_threads < 1) n_threads = 1;
#pragma omp parallel num_threads(n_threads) reduction(| : status)
  {
    int t = omp_get_thread_num(), nt = omp_get_num_threads();
    int64_t chunk = (n_positions + nt - 1) / nt;
    int64_t b = t * chunk, e = b + chunk < n_positions ? b + chunk : n_positions;
    if (b < e)
      status |= q_update_range(ft, bias, l1w, l1b, l2w, l2b, l3w, l3b, parent, flags, rem,
                               rem_off, add, add_off, count0, b, e, child, scores);
  }
#else
  (void)n_threads;
  status = q_update_range(ft, bias, l1w, l1b, l2w, l2b, l3w, l3b, parent, flags, rem, rem_off,
                          add, add_off, count0, 0, n_positions, child, scores);
#endif
  return status;
}

/* fp32 forward. The FT sum runs in index order from the bias; the stack
 * layers are plain sequential dot products in double-free fp32. */
int oracle_f_forward(const float* ft, const float* bias, const float* l1w, const float* l1b,
                     const float* l2w, const float* l2b, const float* l3w, const float* l3b,
                     const uint16_t* idx, uint32_t n_indices, const uint32_t* offsets,
                     int64_t n_positions, float* out, float* acc_out) {
  if (n_positions <= 0) return 0;
  if (check_offsets(offsets, 2 * n_positions, n_indices)) return 3;
  int status = 0;
  float acc[2][F_COLS], x[2 * F_COLS], h1[16], h2[32];
  for (int64_t p = 0; p < n_positions; ++p) {
    for (int s = 0; s < 2; ++s) {
      for (int j = 0; j < F_COLS; ++j) acc[s][j] = bias[j];
      for (uint32_t i = offsets[2 * p + s]; i < offsets[2 * p + s + 1]; ++i) {
        uint32_t f = idx[i];
        if (f >= Q_F) { status = 2; continue; }
        const float* row = ft + (size_t)f * F_COLS;
        for (int j = 0; j < F_COLS; ++j) acc[s][j] += row[j];
      }
      for (int j = 0; j < F_COLS; ++j) x[s * F_COLS + j] = clampf(acc[s][j], 0.f, 1.f);
    }
    if (acc_out) memcpy(acc_out + (size_t)p * 2 * F_COLS, acc, sizeof(acc));
    int bucket = oracle_f_bucket(offsets[2 * p + 1] - offsets[2 * p]);
    for (int k = 0; k < 16; ++k) {
      float s = l1b[bucket * 16 + k];
      const float* w = l1w + ((size_t)bucket * 16 + k) * 2 * F_COLS;
      for (int i = 0; i < 2 * F_COLS; ++i) s += w[i] * x[i];
      h1[k] = clampf(s, 0.f, 1.f);
    }
    for (int m = 0; m < 32; ++m) {
      float s = l2b[bucket * 32 + m];
      const float* w = l2w + ((size_t)bucket * 32 + m) * 16;
      for (int k = 0; k < 16; ++k) s += w[k] * h1[k];
      h2[m] = clampf(s, 0.f, 1.f);
    }
    float s = l3b[bucket];
    for (int m = 0; m < 32; ++m) s += l3w[bucket * 32 + m] * h2[m];
    out[p] = s;
  }
  return status;
}

/* ---- reference-native feature pool ------------------------------------- */
#define POOL_ROWS 1545
#define POOL_PAD 0xffffffffu

/* item_rows, src/az/fused_feature_pool.rs:389-403.  Returns 1 when every row
 * lies inside the 1545-row table (the reference indexes the table with these
 * rows unchecked, so a row past the end is an index panic there). */
static int pool_item_rows(uint32_t packed, uint32_t rows[6]) {
  uint32_t feature = packed & 0x7ffu;
  uint32_t us = (packed >> 11) & 0xfu;
  uint32_t them = (packed >> 15) & 0xfu;
  uint32_t piece = feature / 90u, square = feature % 90u;
  rows[0] = feature;
  rows[1] = 1260u + piece;
  rows[2] = 1274u + square / 9u;
  rows[3] = 1284u + square % 9u;
  rows[4] = 1293u + us * 14u + piece;
  rows[5] = 1293u + (9u + them) * 14u + piece;
  for (int r = 0; r < 6; ++r)
    if (rows[r] >= POOL_ROWS) return 0;
  return 1;
}

/* FeaturePool::cpu_fwd, src/az/fused_feature_pool.rs:169-198: for every item
 * in order, for every h, out += the six rows in order.  Returns 2 when a row
 * falls outside the table (the reference would panic on the slice index). */
int oracle_feature_pool_fwd(const float* tables, const uint32_t* items, int64_t batch,
                            int64_t item_count, int64_t hidden, float* out) {
  int status = 0;
  for (int64_t i = 0; i < batch * hidden; ++i) out[i] = 0.f;
  for (int64_t b = 0; b < batch; ++b) {
    for (int64_t i = 0; i < item_count; ++i) {
      uint32_t packed = items[b * item_count + i];
      if (packed == POOL_PAD) continue;
      uint32_t rows[6];
      if (!pool_item_rows(packed, rows)) { status = 2; continue; }
      for (int64_t h = 0; h < hidden; ++h) {
        float* o = &out[b * hidden + h];
        for (int r = 0; r < 6; ++r) *o += tables[(int64_t)rows[r] * hidden + h];
      }
    }
  }
  return status;
}

/* FeaturePoolGrad::cpu_fwd, src/az/fused_feature_pool.rs:231-260: for every
 * (b, item) in order, for every slot row, grad[row] += grad_out[b]. */
int oracle_feature_pool_bwd(const uint32_t* items, const float* grad_out, int64_t batch,
                            int64_t item_count, int64_t hidden, float* grad_tables) {
  int status = 0;
  for (int64_t i = 0; i < (int64_t)POOL_ROWS * hidden; ++i) grad_tables[i] = 0.f;
  for (int64_t b = 0; b < batch; ++b) {
    for (int64_t i = 0; i < item_count; ++i) {
      uint32_t packed = items[b * item_count + i];
      if (packed == POOL_PAD) continue;
      uint32_t rows[6];
      if (!pool_item_rows(packed, rows)) { status = 2; continue; }
      for (int r = 0; r < 6; ++r)
        for (int64_t h = 0; h < hidden; ++h)
          grad_tables[(int64_t)rows[r] * hidden + h] += grad_out[b * hidden + h];
    }
  }
  return status;
}

/* SparsePool::cpu_fwd, src/az/fused_feature_pool.rs:284-309. */
int oracle_sparse_pool_fwd(const float* table, int64_t rows, const uint32_t* items, int64_t batch,
                           int64_t item_count, int64_t hidden, float* out) {
  int status = 0;
  for (int64_t i = 0; i < batch * hidden; ++i) out[i] = 0.f;
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t i = 0; i < item_count; ++i) {
      uint32_t item = items[b * item_count + i];
      if (item == POOL_PAD) continue;
      if ((int64_t)item >= rows) { status = 2; continue; }
      for (int64_t h = 0; h < hidden; ++h) out[b * hidden + h] += table[(int64_t)item * hidden + h];
    }
  return status;
}

/* SparsePoolGrad::cpu_fwd, src/az/fused_feature_pool.rs:342-370. */
int oracle_sparse_pool_bwd(const uint32_t* items, const float* grad_out, int64_t rows,
                           int64_t batch, int64_t item_count, int64_t hidden, float* grad_table) {
  int status = 0;
  for (int64_t i = 0; i < rows * hidden; ++i) grad_table[i] = 0.f;
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t i = 0; i < item_count; ++i) {
      uint32_t item = items[b * item_count + i];
      if (item == POOL_PAD) continue;
      if ((int64_t)item >= rows) { status = 2; continue; }
      for (int64_t h = 0; h < hidden; ++h)
        grad_table[(int64_t)item * hidden + h] += grad_out[b * hidden + h];
    }
  return status;
}

/* ---- policy-head training ops ------------------------------------------- */
/* Item fields and table offsets, src/az/fused_policy.rs:10-35. */
#define POL_TABLE_LEN 182886
#define POL_CONSEQUENCE 40320
#define POL_BIAS 40352
#define POL_CONTEXT 42438
#define POL_ACC_FEATURE 75814
#define POL_ACC_MOVE 116134
#define POL_CTX 48

typedef struct {
  int policy, move, capture;
  int64_t mv, from, to, cap;
} pol_item;

static pol_item pol_decode(int64_t packed_s) {
  uint64_t p = (uint64_t)packed_s;
  pol_item it;
  it.policy = (int)((p >> 47) & 1u);
  it.move = (int)((p >> 45) & 1u);
  it.capture = (int)((p >> 46) & 1u);
  it.mv = (int64_t)(p & 0xfffu);
  it.from = (int64_t)((p >> 12) & 0x7ffu);
  it.to = (int64_t)((p >> 23) & 0x7ffu);
  it.cap = (int64_t)((p >> 34) & 0x7ffu);
  return it;
}

/* The Rust twin indexes its slices and panics past the end; here such an
 * item is skipped and reported (status 2). */
static int pol_in_range(const pol_item* it) {
  return it->mv < 2086 && (!it->move || (it->from < 1260 && it->to < 1260 && (!it->capture || it->cap < 1260)));
}

/* FusedPolicy::cpu_fwd, src/az/fused_policy.rs:178-241. */
int oracle_policy_fused_fwd(const float* t, const float* context, const int64_t* items, int64_t batch,
                            int64_t moves, float* out) {
  int status = 0;
  for (int64_t i = 0; i < batch * moves; ++i) {
    out[i] = 0.f;
    pol_item it = pol_decode(items[i]);
    if (!it.policy) continue;
    if (!pol_in_range(&it)) { status = 2; continue; }
    float value = t[POL_BIAS + it.mv];
    if (it.move) {
      const float* c = context + (i / moves) * POL_CTX;
      for (int h = 0; h < 32; ++h) {
        float delta = t[it.to * 32 + h] - t[it.from * 32 + h];
        if (it.capture) delta -= t[it.cap * 32 + h];
        value += delta * t[POL_CONSEQUENCE + h];
      }
      for (int h = 0; h < 16; ++h) value += c[h] * t[POL_CONTEXT + it.mv * 16 + h];
      for (int h = 0; h < 32; ++h) {
        float after = c[16 + h] + t[POL_ACC_FEATURE + it.to * 32 + h] - t[POL_ACC_FEATURE + it.from * 32 + h];
        if (it.capture) after -= t[POL_ACC_FEATURE + it.cap * 32 + h];
        value += after * t[POL_ACC_MOVE + it.mv * 32 + h];
      }
    }
    out[i] = value;
  }
  return status;
}

/* FusedPolicyGrad::cpu_fwd, src/az/fused_policy.rs:287-366: one pass over the
 * items in order, every contribution added as it is met. */
int oracle_policy_fused_bwd(const float* t, const float* context, const int64_t* items, const float* grad_out,
                            int64_t batch, int64_t moves, float* grad_t, float* grad_c) {
  int status = 0;
  for (int64_t i = 0; i < POL_TABLE_LEN; ++i) grad_t[i] = 0.f;
  for (int64_t i = 0; i < batch * POL_CTX; ++i) grad_c[i] = 0.f;
  for (int64_t i = 0; i < batch * moves; ++i) {
    pol_item it = pol_decode(items[i]);
    if (!it.policy) continue;
    if (!pol_in_range(&it)) { status = 2; continue; }
    const float g = grad_out[i];
    grad_t[POL_BIAS + it.mv] += g;
    if (!it.move) continue;
    const int64_t b = i / moves;
    const float* c = context + b * POL_CTX;
    float* gc = grad_c + b * POL_CTX;
    for (int h = 0; h < 32; ++h) {
      const float w = t[POL_CONSEQUENCE + h];
      float delta = t[it.to * 32 + h] - t[it.from * 32 + h];
      grad_t[it.to * 32 + h] += g * w;
      grad_t[it.from * 32 + h] -= g * w;
      if (it.capture) {
        delta -= t[it.cap * 32 + h];
        grad_t[it.cap * 32 + h] -= g * w;
      }
      grad_t[POL_CONSEQUENCE + h] += g * delta;
    }
    for (int h = 0; h < 16; ++h) {
      const int64_t ci = POL_CONTEXT + it.mv * 16 + h;
      grad_t[ci] += g * c[h];
      gc[h] += g * t[ci];
    }
    for (int h = 0; h < 32; ++h) {
      const int64_t mf = POL_ACC_MOVE + it.mv * 32 + h;
      const float w = t[mf];
      const int64_t ti = POL_ACC_FEATURE + it.to * 32 + h, fi = POL_ACC_FEATURE + it.from * 32 + h;
      float after = c[16 + h] + t[ti] - t[fi];
      gc[16 + h] += g * w;
      grad_t[ti] += g * w;
      grad_t[fi] -= g * w;
      if (it.capture) {
        const int64_t cpi = POL_ACC_FEATURE + it.cap * 32 + h;
        after -= t[cpi];
        grad_t[cpi] -= g * w;
      }
      grad_t[mf] += g * after;
    }
  }
  return status;
}

/* SparsePolicy::cpu_fwd, src/az/fused_sparse_policy.rs:86-107 (terms = 7 for
 * the sparse table, 2 for the tactical one).  Rust's f32 Sum folds from
 * -0.0, the exact additive identity. */
int oracle_policy_table_fwd(const float* table, int64_t table_len, const int64_t* indices, int64_t outputs,
                            int terms, float* out) {
  int status = 0;
  for (int64_t o = 0; o < outputs; ++o) {
    float s = -0.f;
    for (int k = 0; k < terms; ++k) {
      const int64_t j = indices[o * terms + k];
      if (j < 0 || j >= table_len) { status = 2; continue; }
      s += table[j];
    }
    out[o] = s;
  }
  return status;
}

/* SparsePolicyGrad::cpu_fwd, src/az/fused_sparse_policy.rs:138-165. */
int oracle_policy_table_bwd(const int64_t* indices, const float* grad_out, int64_t outputs, int terms,
                            int64_t table_len, float* grad_table) {
  int status = 0;
  for (int64_t j = 0; j < table_len; ++j) grad_table[j] = 0.f;
  for (int64_t o = 0; o < outputs; ++o)
    for (int k = 0; k < terms; ++k) {
      const int64_t j = indices[o * terms + k];
      if (j < 0 || j >= table_len) { status = 2; continue; }
      grad_table[j] += grad_out[o];
    }
  return status;
}

/* ---- AdamW (candle-nn AdamW::step, the AZ trainer's optimizer) ---------- */
/* Parity of this restatement with candle itself is unpinned (candle cannot be
 * run here); the CUDA kernel is held to it bit for bit.  Each "x*a + c" is one
 * of candle's fp32 affine maps; b^t by repeated squaring (the powi runtime). */
static double oracle_powi(double b, int64_t e) {
  double r = 1.0;
  for (;;) {
    if (e & 1) r *= b;
    e /= 2;
    if (e == 0) break;
    b *= b;
  }
  return r;
}

int oracle_adamw(float* p, float* m, float* v, const float* g, int64_t n, double lr, double beta1, double beta2,
                 double eps, double wd, int64_t step) {
  const float b1 = (float)beta1, omb1 = (float)(1.0 - beta1), b2 = (float)beta2, omb2 = (float)(1.0 - beta2);
  const float sm = (float)(1.0 / (1.0 - oracle_powi(beta1, step)));
  const float sv = (float)(1.0 / (1.0 - oracle_powi(beta2, step)));
  const float decay = (float)(1.0 - lr * wd), flr = (float)lr, feps = (float)eps;
  for (int64_t i = 0; i < n; ++i) {
    const float gi = g[i];
    const float nm = (m[i] * b1 + 0.f) + (gi * omb1 + 0.f);
    const float nv = (v[i] * b2 + 0.f) + ((gi * gi) * omb2 + 0.f);
    const float mh = nm * sm + 0.f, vh = nv * sv + 0.f;
    const float den = sqrtf(vh) * 1.f + feps;
    p[i] = (p[i] * decay + 0.f) - ((mh / den) * flr + 0.f);
    m[i] = nm;
    v[i] = nv;
  }
  return 0;
}

/* ---- training step (data-parallel shard of one rank) ------------------- */
/* Conventions fixed here (the workload specification leaves them open;
 * parity UNPINNED by the reference, whose trainer differs):
 *   - FT master weights fp32 [11340][1024], bias fp32 [1024]; the forward
 *     gathers their bf16 shadow (round-to-nearest-even), sums in fp32 in
 *     index order starting from the bias, and stores the activation a as bf16;
 *   - u = clamp(a, 0, 1); x[p*512+j] = bf16(u_p[j] * u_p[j+512]);
 *   - bucket = min((max(n0,1)-1)>>1, 15); stack fp32: z1 = W1 x + b1,
 *     h1 = clamp(z1,0,1); z2 = W2 h1 + b2, h2 = clamp(z2,0,1); s = W3 h2 + b3;
 *   - loss = mean over the rank's batch of (sigmoid(s/400) - t)^2;
 *   - clamp derivative 1 strictly inside (0,1), else 0; bf16 roundings pass
 *     gradients straight through; gradients are of the rank's mean loss;
 *   - Adam (Kingma & Ba): m = b1 m + (1-b1) g, v = b2 v + (1-b2) g^2,
 *     w -= lr * (m / (1-b1^t)) / (sqrt(v / (1-b2^t)) + eps). */
#define T_F 11340
#define T_COLS 1024
#define T_NB 16

/* float -> bfloat16 -> float, round to nearest even (NaN -> quiet NaN). */
static inline float bf16_round(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u)
    u = (u | 0x00400000u) & 0xffff0000u;
  else
    u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
  float r;
  memcpy(&r, &u, 4);
  return r;
}

void oracle_bf16_round_array(const float* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = bf16_round(in[i]);
}

static inline float dclampf01(float z) { return (z > 0.f && z < 1.f) ? 1.f : 0.f; }

/* Forward + backward of one rank's batch.  Gradients are written (not
 * accumulated) into g_* (same shapes as the parameters); loss_out gets the
 * mean loss; score_out [n] optional. */
int oracle_t_grad(const float* ft, const float* ft_bias, const float* w1, const float* b1,
                  const float* w2, const float* b2, const float* w3, const float* b3,
                  const uint16_t* idx, uint32_t n_indices, const uint32_t* offsets,
                  int64_t n, const float* target, float* g_ft, float* g_ft_bias, float* g_w1,
                  float* g_b1, float* g_w2, float* g_b2, float* g_w3, float* g_b3,
                  float* loss_out, float* score_out) {
  if (n <= 0) return 1;
  if (check_offsets(offsets, 2 * n, n_indices)) return 3;
  memset(g_ft, 0, sizeof(float) * (size_t)T_F * T_COLS);
  memset(g_ft_bias, 0, sizeof(float) * T_COLS);
  memset(g_w1, 0, sizeof(float) * T_NB * 16 * T_COLS);
  memset(g_b1, 0, sizeof(float) * T_NB * 16);
  memset(g_w2, 0, sizeof(float) * T_NB * 32 * 16);
  memset(g_b2, 0, sizeof(float) * T_NB * 32);
  memset(g_w3, 0, sizeof(float) * T_NB * 32);
  memset(g_b3, 0, sizeof(float) * T_NB);
  double loss = 0.0;
  float a[2 * T_COLS], x[T_COLS], dx[T_COLS], da[2 * T_COLS];
  int status = 0;
  for (int64_t b = 0; b < n; ++b) {
    for (int p = 0; p < 2; ++p) {
      float* ap = a + p * T_COLS;
      for (int j = 0; j < T_COLS; ++j) ap[j] = bf16_round(ft_bias[j]);
      for (uint32_t i = offsets[2 * b + p]; i < offsets[2 * b + p + 1]; ++i) {
        uint32_t f = idx[i];
        if (f >= T_F) { status = 2; continue; }
        const float* row = ft + (size_t)f * T_COLS;
        for (int j = 0; j < T_COLS; ++j) ap[j] += bf16_round(row[j]);
      }
      for (int j = 0; j < T_COLS; ++j) ap[j] = bf16_round(ap[j]);
      for (int j = 0; j < 512; ++j) x[p * 512 + j] = bf16_round(clampf(ap[j], 0.f, 1.f) * clampf(ap[j + 512], 0.f, 1.f));
    }
    const int bk = oracle_q_bucket(offsets[2 * b + 1] - offsets[2 * b]);
    float z1[16], h1[16], z2[32], h2[32];
    for (int k = 0; k < 16; ++k) {
      float s = b1[bk * 16 + k];
      const float* w = w1 + ((size_t)bk * 16 + k) * T_COLS;
      for (int i = 0; i < T_COLS; ++i) s += w[i] * x[i];
      z1[k] = s;
      h1[k] = clampf(s, 0.f, 1.f);
    }
    for (int m = 0; m < 32; ++m) {
      float s = b2[bk * 32 + m];
      for (int k = 0; k < 16; ++k) s += w2[(bk * 32 + m) * 16 + k] * h1[k];
      z2[m] = s;
      h2[m] = clampf(s, 0.f, 1.f);
    }
    float sc = b3[bk];
    for (int m = 0; m < 32; ++m) sc += w3[bk * 32 + m] * h2[m];
    if (score_out) score_out[b] = sc;
    const float sg = 1.f / (1.f + expf(-sc / 400.f));
    const float d = sg - target[b];
    loss += (double)d * d;
    const float gs = 2.f * d * sg * (1.f - sg) / 400.f / (float)n;
    float dh2[32], dh1[16];
    g_b3[bk] += gs;
    for (int m = 0; m < 32; ++m) {
      g_w3[bk * 32 + m] += gs * h2[m];
      dh2[m] = gs * w3[bk * 32 + m] * dclampf01(z2[m]);
      g_b2[bk * 32 + m] += dh2[m];
    }
    for (int k = 0; k < 16; ++k) {
      float s = 0.f;
      for (int m = 0; m < 32; ++m) {
        g_w2[(bk * 32 + m) * 16 + k] += dh2[m] * h1[k];
        s += w2[(bk * 32 + m) * 16 + k] * dh2[m];
      }
      dh1[k] = s * dclampf01(z1[k]);
      g_b1[bk * 16 + k] += dh1[k];
    }
    for (int i = 0; i < T_COLS; ++i) dx[i] = 0.f;
    for (int k = 0; k < 16; ++k) {
      const float* w = w1 + ((size_t)bk * 16 + k) * T_COLS;
      float* gw = g_w1 + ((size_t)bk * 16 + k) * T_COLS;
      for (int i = 0; i < T_COLS; ++i) {
        gw[i] += dh1[k] * x[i];
        dx[i] += w[i] * dh1[k];
      }
    }
    for (int p = 0; p < 2; ++p) {
      const float* ap = a + p * T_COLS;
      float* dap = da + p * T_COLS;
      for (int j = 0; j < 512; ++j) {
        const float g = dx[p * 512 + j];
        dap[j] = g * clampf(ap[j + 512], 0.f, 1.f) * dclampf01(ap[j]);
        dap[j + 512] = g * clampf(ap[j], 0.f, 1.f) * dclampf01(ap[j + 512]);
      }
      for (int j = 0; j < T_COLS; ++j) g_ft_bias[j] += dap[j];
      for (uint32_t i = offsets[2 * b + p]; i < offsets[2 * b + p + 1]; ++i) {
        uint32_t f = idx[i];
        if (f >= T_F) continue;
        float* g = g_ft + (size_t)f * T_COLS;
        for (int j = 0; j < T_COLS; ++j) g[j] += dap[j];
      }
    }
  }
  *loss_out = (float)(loss / (double)n);
  return status;
}

/* One Adam step over a flat parameter array (gradient scaled by grad_scale). */
void oracle_adam(float* w, float* m, float* v, const float* g, int64_t count, float grad_scale,
                 float lr, float beta1, float beta2, float eps, int step) {
  const float c1 = 1.f - powf(beta1, (float)step);
  const float c2 = 1.f - powf(beta2, (float)step);
  for (int64_t i = 0; i < count; ++i) {
    const float gi = g[i] * grad_scale;
    m[i] = beta1 * m[i] + (1.f - beta1) * gi;
    v[i] = beta2 * v[i] + (1.f - beta2) * gi * gi;
    w[i] -= lr * (m[i] / c1) / (sqrtf(v[i] / c2) + eps);
  }
}

/* ---- AZ-NNUE, the reference's own network (reference-native) ----------- */
/* Restates src/nnue.rs:25-43 (features), src/az.rs:155-203 (buckets,
 * structural rows), :1339-1431 (AzNnue::random), :2049-2076 + :1920-2042
 * (FT gather order: bias, every input row in feature order, then for every
 * feature its piece, rank, file, king(us), king(them) rows), :439-566
 * (incremental transition), :1903-1918 (rule context), :3020-3126 (ReLU,
 * RMSNorm eps 1e-6), :2133-2157 + :2563-2575 (value head, WDL softmax). */
#define AZ_SQ 90
#define AZ_INPUT 1260
#define AZ_ROWS 1545
#define AZ_VALUE 96

static uint64_t az_mix(uint64_t v) {
  v += 0x9E3779B97F4A7C15ull;
  uint64_t m = v;
  m = (m ^ (m >> 30)) * 0xBF58476D1CE4E5B9ull;
  m = (m ^ (m >> 27)) * 0x94D049BB133111EBull;
  return m ^ (m >> 31);
}

/* SplitMix64::unit_f32 / weight, src/az.rs:3161-3168. */
static float az_weight(uint64_t* st, float scale) {
  *st = az_mix(*st);
  const float u = (float)((double)(*st >> 11) * (1.0 / 9007199254740992.0));
  return (u * 2.0f - 1.0f) * scale;
}

/* Tensor element counts in az_weight_tensors! order (src/az.rs:241-278). */
int64_t oracle_az_tensor_elements(int i, int h) {
  static const int64_t fixed[22] = {0, 0, 0, 0, 0, 0, 0, 0, 96, 3 * 96, 57702LL * 64, 3 * 128,
                                    16 * 128, 2086, 32, 0, 2086 * 16, 0, 2086 * 32, 2396815,
                                    199458, 934976};
  switch (i) {
    case 0: return 1260LL * h;
    case 1: return 14LL * h;
    case 2: return 10LL * h;
    case 3: return 9LL * h;
    case 4: return 252LL * h;
    case 5: return 7LL * h;
    case 6: return h;
    case 7: return 96LL * h;
    case 15: return 16LL * h;
    case 17: return 32LL * h;
    default: return (i >= 0 && i < 22) ? fixed[i] : -1;
  }
}

/* AzNnue::random_with_arch, src/az.rs:1339-1431: tensors[i] must hold
 * oracle_az_tensor_elements(i, h) floats; draws in the reference's order. */
void oracle_az_random(int h, uint64_t seed, float** t) {
  for (int i = 0; i < 22; ++i) memset(t[i], 0, sizeof(float) * (size_t)oracle_az_tensor_elements(i, h));
  uint64_t st = seed;
  const float hs = sqrtf(2.0f / (float)(h > 1 ? h : 1)) * 0.5f;
  for (int64_t i = 0; i < 1260LL * h; ++i) t[0][i] = az_weight(&st, 0.015f);
  for (int64_t i = 0; i < 96LL * h; ++i) t[7][i] = az_weight(&st, hs);
  for (int64_t i = 0; i < 57702LL * 64; ++i) t[10][i] = az_weight(&st, 0.02f);
  for (int64_t i = 0; i < 16LL * h; ++i) t[15][i] = az_weight(&st, hs);
  for (int64_t i = 0; i < 32LL * h; ++i) t[17][i] = az_weight(&st, hs);
}

/* canonical_general_bucket, src/az.rs:194-203. */
static int az_bucket(int piece_index, int sq) {
  const int o = piece_index < 7 ? sq : AZ_SQ - 1 - sq;
  int f = o % 9, r = o / 9;
  f = f < 3 ? 3 : (f > 5 ? 5 : f);
  r = r < 7 ? 7 : (r > 9 ? 9 : r);
  return (r - 7) * 3 + (f - 3);
}

/* Features of one perspective (src/nnue.rs:25-43 with the perspective in
 * place of the side to move, as refresh_perspective does, src/az.rs:413-426),
 * packed feature | us << 11 | them << 15 with the king buckets of
 * canonical_general_buckets_from_features (src/az.rs:168-184).  board: 0
 * empty, +1..+7 Red kind+1, -1..-7 Black kind+1.  Returns the count. */
int oracle_az_features(const int8_t* board, int perspective, uint32_t* items) {
  int n = 0, us = 4, them = 4;
  uint32_t feat[AZ_SQ];
  for (int sq = 0; sq < AZ_SQ; ++sq) {
    const int v = board[sq];
    if (v == 0) continue;
    const int color = v > 0 ? 0 : 1, kind = (v > 0 ? v : -v) - 1;
    const int piece_index = (color == perspective ? 0 : 7) + kind;
    const int csq = perspective == 0 ? sq : AZ_SQ - 1 - sq;
    feat[n++] = (uint32_t)(piece_index * AZ_SQ + csq);
  }
  for (int i = 0; i < n; ++i) {
    const int pi = (int)feat[i] / AZ_SQ, s = (int)feat[i] % AZ_SQ;
    if (pi == 0) us = az_bucket(0, s);
    if (pi == 7) them = az_bucket(7, s);
  }
  for (int i = 0; i < n; ++i) items[i] = feat[i] | ((uint32_t)us << 11) | ((uint32_t)them << 15);
  return n;
}

/* The six trunk rows of an item (offsets into the concatenated [1545][H]
 * trunk table: input 0, piece 1260, rank 1274, file 1284, king-piece 1293). */
static int az_rows(uint32_t item, int rows[6]) {
  const int feature = item & 0x7ff, us = (item >> 11) & 0xf, them = (item >> 15) & 0xf;
  if (feature >= AZ_INPUT || us > 8 || them > 8) return 0;
  const int piece = feature / 90, sq = feature % 90;
  rows[0] = feature;
  rows[1] = 1260 + piece;
  rows[2] = 1274 + sq / 9;
  rows[3] = 1284 + sq % 9;
  rows[4] = 1293 + us * 14 + piece;
  rows[5] = 1293 + (9 + them) * 14 + piece;
  return 1;
}

/* input_embedding_linear_into_slice for each list: acc = bias, + input row of
 * every item, + its five structural rows per item (in item order).  table =
 * [1545][H] concatenation.  Returns 2 on a bad item (skipped). */
int oracle_az_refresh(const float* table, const float* bias, int h, const uint32_t* items,
                      const uint32_t* offsets, int64_t n_lists, float* acc) {
  int status = 0;
  for (int64_t l = 0; l < n_lists; ++l) {
    float* a = acc + l * h;
    for (int j = 0; j < h; ++j) a[j] = bias[j];
    for (uint32_t i = offsets[l]; i < offsets[l + 1]; ++i) {
      int r[6];
      if (!az_rows(items[i], r)) { status = 2; continue; }
      for (int j = 0; j < h; ++j) a[j] += table[(int64_t)r[0] * h + j];
    }
    for (uint32_t i = offsets[l]; i < offsets[l + 1]; ++i) {
      int r[6];
      if (!az_rows(items[i], r)) continue;
      for (int k = 1; k < 6; ++k)
        for (int j = 0; j < h; ++j) a[j] += table[(int64_t)r[k] * h + j];
    }
  }
  return status;
}

/* apply_transition_for_perspective (src/az.rs:439-485): refresh[l] -> the
 * refresh of list l; else child = parent - rows(from) - rows(captured)
 * + rows(to), each item's six rows in order (add_canonical_piece_contribution,
 * src/az.rs:509-566).  delta[3l..3l+2] = from, captured (or 0xffffffff), to. */
int oracle_az_transition(const float* table, const float* bias, int h, const float* parent,
                         const uint32_t* delta, const uint8_t* refresh, const uint32_t* items,
                         const uint32_t* offsets, int64_t n_lists, float* child) {
  int status = 0;
  for (int64_t l = 0; l < n_lists; ++l) {
    float* c = child + l * h;
    if (refresh[l] & 1) {
      status |= oracle_az_refresh(table, bias, h, items, offsets + l, 1, c);
      continue;
    }
    for (int j = 0; j < h; ++j) c[j] = parent[l * h + j];
    for (int q = 0; q < 3; ++q) {
      const uint32_t it = delta[3 * l + q];
      if (it == 0xffffffffu) continue;
      int r[6];
      if (!az_rows(it, r)) { status = 2; continue; }
      for (int k = 0; k < 6; ++k)
        for (int j = 0; j < h; ++j) {
          const float w = table[(int64_t)r[k] * h + j];
          c[j] = q < 2 ? c[j] - w : c[j] + w;
        }
    }
  }
  return status;
}

/* Value of side-to-move accumulators: + rule context (non-zero entries,
 * src/az.rs:1903-1918), ReLU, RMSNorm (eps 1e-6), value head 96 ReLU units,
 * 3 WDL logits + threat logits, softmax, q = W - L.  rule [n][7] and threat
 * [n][3] may be NULL. */
void oracle_az_value(const float* rule_rows, const float* vh, const float* vb, const float* vo, int h,
                     const float* hidden, const float* rule, const float* threat, int64_t n,
                     float* wdl, float* q, float* x_out) {
  float x[4096], v[AZ_VALUE];
  if (h > 4096) return;
  for (int64_t p = 0; p < n; ++p) {
    for (int j = 0; j < h; ++j) x[j] = hidden[p * h + j];
    if (rule)
      for (int k = 0; k < 7; ++k) {
        const float r = rule[p * 7 + k];
        if (r == 0.f) continue;
        for (int j = 0; j < h; ++j) x[j] += r * rule_rows[k * h + j];
      }
    float ss = 0.f;
    for (int j = 0; j < h; ++j) {
      x[j] = x[j] > 0.f ? x[j] : 0.f;
      ss += x[j] * x[j];
    }
    const float inv = 1.f / sqrtf(ss / (float)h + 1e-6f);
    for (int j = 0; j < h; ++j) x[j] *= inv;
    if (x_out) memcpy(x_out + p * h, x, sizeof(float) * h);
    for (int k = 0; k < AZ_VALUE; ++k) {
      float s = vb[k];
      for (int j = 0; j < h; ++j) s += vh[k * h + j] * x[j];
      v[k] = s > 0.f ? s : 0.f;
    }
    float lg[3];
    for (int o = 0; o < 3; ++o) {
      float s = 0.f;
      for (int k = 0; k < AZ_VALUE; ++k) s += vo[o * AZ_VALUE + k] * v[k];
      lg[o] = s + (threat ? threat[p * 3 + o] : 0.f);
    }
    float mx = lg[0] > lg[1] ? lg[0] : lg[1];
    mx = mx > lg[2] ? mx : lg[2];
    float e[3];
    for (int o = 0; o < 3; ++o) e[o] = expf(lg[o] - mx);
    float sum = e[0] + e[1] + e[2];
    if (sum < FLT_MIN) sum = FLT_MIN; /* .max(f32::MIN_POSITIVE) */
    for (int o = 0; o < 3; ++o) wdl[p * 3 + o] = e[o] / sum;
    q[p] = wdl[p * 3] - wdl[p * 3 + 2];
  }
}

/* ---- AZ-NNUE quantised policy accumulator (reference-native) ------------ */
/* dot_product (src/az.rs:2730-2766) as it runs on x86-64 with AVX2 and FMA:
 * length >= 64 -> 4 x 8-lane FMA accumulators over 32-float chunks, lanes
 * combined (a0+a1)+(a2+a3), summed left to right, then the tail with separate
 * multiply and add (dot_product_avx2_fma, :2880-2922); shorter -> 4 scalar
 * accumulators (sum0+sum1)+(sum2+sum3) then the tail. */
static float az_dot(const float* l, const float* r, int n) {
  if (n >= 64) {
    float acc[4][8];
    memset(acc, 0, sizeof(acc));
    const int chunks = n / 32;
    for (int c = 0; c < chunks; ++c)
      for (int a = 0; a < 4; ++a)
        for (int k = 0; k < 8; ++k) acc[a][k] = fmaf(l[c * 32 + a * 8 + k], r[c * 32 + a * 8 + k], acc[a][k]);
    float sum = 0.0f;
    for (int k = 0; k < 8; ++k) {
      const float v = (acc[0][k] + acc[1][k]) + (acc[2][k] + acc[3][k]);
      sum += v;
    }
    for (int i = chunks * 32; i < n; ++i) {
      const float p = l[i] * r[i];
      sum += p;
    }
    return sum;
  }
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  const int chunks = n / 4;
  for (int c = 0; c < chunks; ++c) {
    float p0 = l[4 * c] * r[4 * c], p1 = l[4 * c + 1] * r[4 * c + 1];
    float p2 = l[4 * c + 2] * r[4 * c + 2], p3 = l[4 * c + 3] * r[4 * c + 3];
    s0 += p0;
    s1 += p1;
    s2 += p2;
    s3 += p3;
  }
  float sum = (s0 + s1) + (s2 + s3);
  for (int i = chunks * 4; i < n; ++i) {
    const float p = l[i] * r[i];
    sum += p;
  }
  return sum;
}

/* Symmetric int8 quantisation of x[n] (src/az.rs:2250-2262): scale =
 * max(max|x| / 127, 1e-12), q = clamp(round(x / scale), -127, 127) with
 * round half away from zero and NaN -> 0. */
static float az_quantize(const float* x, int64_t n, int8_t* q) {
  float mx = 0.f;
  for (int64_t i = 0; i < n; ++i) {
    const float a = fabsf(x[i]);
    if (a > mx) mx = a; /* f32::max ignores NaN */
  }
  float scale = mx / 127.0f;
  if (!(scale >= 1.0e-12f)) scale = 1.0e-12f;
  for (int64_t i = 0; i < n; ++i) {
    float v = roundf(x[i] / scale);
    if (v != v) v = 0.f;
    v = v < -127.f ? -127.f : (v > 127.f ? 127.f : v);
    q[i] = (int8_t)v;
  }
  return scale;
}

/* is_valid_policy_move (src/az.rs:3178-3238) */
static int az_advisor_pos(int r, int f) {
  return (r == 0 && (f == 3 || f == 5)) || (r == 1 && f == 4) || (r == 2 && (f == 3 || f == 5)) ||
         (r == 7 && (f == 3 || f == 5)) || (r == 8 && f == 4) || (r == 9 && (f == 3 || f == 5));
}
static int az_elephant_pos(int r, int f) {
  return ((r == 0 || r == 9) && (f == 2 || f == 6)) || ((r == 2 || r == 7) && (f == 0 || f == 4 || f == 8)) ||
         ((r == 4 || r == 5) && (f == 2 || f == 6));
}
static int az_valid_move(int from, int to) {
  const int ff = from % 9, fr = from / 9, tf = to % 9, tr = to / 9;
  const int df = abs(tf - ff), dr = abs(tr - fr);
  if (df == 0 || dr == 0) return 1;
  if ((df == 1 && dr == 2) || (df == 2 && dr == 1)) return 1;
  if (df == 1 && dr == 1 && az_advisor_pos(fr, ff) && az_advisor_pos(tr, tf)) return 1;
  if (df == 2 && dr == 2 && az_elephant_pos(fr, ff) && az_elephant_pos(tr, tf)) return 1;
  return 0;
}

/* move_map (src/az.rs:3261-3285): dense index -> from * 90 + to. */
int oracle_az_dense_moves(uint16_t* dense_to_sparse) {
  int n = 0;
  for (int from = 0; from < 90; ++from)
    for (int to = 0; to < 90; ++to)
      if (from != to && az_valid_move(from, to)) dense_to_sparse[n++] = (uint16_t)(from * 90 + to);
  return n;
}

/* rebuild_policy_accumulator_quantization + rebuild_value_threat_quantization
 * (src/az.rs:2201-2342).  t = the 22 tensors.  Outputs: feature_q
 * [1546][32], move_q [2086][32], sparse_q [2396815], moved_delta / capture
 * [2086][14] (int32), threat_q [57702][64]; scales[4] = feature, move,
 * sparse, threat; flags[2] = value_threat_active, policy_tactical_active. */
int oracle_az_quantize(int h, const float* const* t, int8_t* feature_q, int8_t* move_q, int8_t* sparse_q,
                       int32_t* moved_delta, int32_t* capture, int8_t* threat_q, float* scales, int* flags) {
  const int rank = 32, moves = 2086;
  float* projected = (float*)malloc(sizeof(float) * 1546 * rank);
  if (!projected) return 1;
  const int tables[6] = {0, 1, 2, 3, 4, 6};
  const int rows_of[6] = {1260, 14, 10, 9, 252, 1};
  int64_t o = 0;
  for (int k = 0; k < 6; ++k)
    for (int r = 0; r < rows_of[k]; ++r)
      for (int j = 0; j < rank; ++j) projected[o++] = az_dot(t[tables[k]] + (int64_t)r * h, t[17] + (int64_t)j * h, h);
  scales[0] = az_quantize(projected, 1546 * rank, feature_q);
  free(projected);
  scales[1] = az_quantize(t[18], (int64_t)moves * rank, move_q);
  /* fold the sparse factors into the main table */
  const int64_t main_size = (int64_t)moves * 14 * 81, sparse_size = 2396815;
  float* folded = (float*)malloc(sizeof(float) * sparse_size);
  if (!folded) return 1;
  memcpy(folded, t[19], sizeof(float) * sparse_size);
  uint16_t d2s[2086];
  oracle_az_dense_moves(d2s);
  const int64_t mp = (int64_t)moves * 14, mk = (int64_t)moves * 81, pk = 14 * 81, dist = 14 * 6;
  for (int m = 0; m < moves; ++m) {
    const int from = d2s[m] / 90, to = d2s[m] % 90;
    for (int piece = 0; piece < 14; ++piece)
      for (int us = 0; us < 9; ++us)
        for (int them = 0; them < 9; ++them) {
          const int64_t main = (((int64_t)m * 14 + piece) * 9 + us) * 9 + them;
          const int pair = us * 9 + them;
          /* policy_king_distance_buckets (src/az.rs:841-859) */
          const int king = 89 - ((7 + them / 3) * 9 + (3 + them % 3));
          const int before = abs(from / 9 - king / 9) + abs(from % 9 - king % 9);
          const int after = abs(to / 9 - king / 9) + abs(to % 9 - king % 9);
          int approach = before - after;
          approach = (approach < -2 ? -2 : (approach > 2 ? 2 : approach)) + 2;
          const int distance = after < 5 ? after : 5;
          const int64_t f[5] = {(int64_t)m * 14 + piece, mp + (int64_t)m * 81 + pair, mp + mk + piece * 81 + pair,
                                mp + mk + pk + piece * 6 + distance, mp + mk + pk + dist + piece * 5 + approach};
          for (int k = 0; k < 5; ++k) folded[main] += t[20][f[k]];
        }
  }
  (void)main_size;
  scales[2] = az_quantize(folded, sparse_size, sparse_q);
  free(folded);
  for (int m = 0; m < moves; ++m) {
    const int from = d2s[m] / 90, to = d2s[m] % 90;
    for (int piece = 0; piece < 14; ++piece) {
      int32_t md = 0, cap = 0;
      for (int j = 0; j < rank; ++j) {
        const int32_t w = move_q[m * rank + j];
        const int32_t tq = feature_q[(piece * 90 + to) * rank + j], fq = feature_q[(piece * 90 + from) * rank + j];
        md += (tq - fq) * w;
        cap += tq * w;
      }
      moved_delta[m * 14 + piece] = md;
      capture[m * 14 + piece] = cap;
    }
  }
  int threat_active = 0, tactical_active = 0;
  for (int i = 0; i < 3 * 128 && !threat_active; ++i) threat_active = t[11][i] != 0.f;
  for (int i = 0; i < 16 * 128 && !threat_active; ++i) threat_active = t[12][i] != 0.f;
  for (int64_t i = 0; i < 934976 && !tactical_active; ++i) tactical_active = t[21][i] != 0.f;
  scales[3] = az_quantize(t[10], 57702LL * 64, threat_q);
  flags[0] = threat_active;
  flags[1] = tactical_active;
  return 0;
}

/* Saturating int16 row add (add_quantized_policy_row, src/az.rs:2439-2451). */
static void az_policy_row(int16_t* acc, const int8_t* q, int row, int sign) {
  for (int j = 0; j < 32; ++j) {
    int v = (int)acc[j] + sign * (int)q[row * 32 + j];
    acc[j] = (int16_t)(v < -32768 ? -32768 : (v > 32767 ? 32767 : v));
  }
}

static void az_policy_piece(int16_t* acc, const int8_t* q, const int rows[6], int sign) {
  for (int k = 0; k < 6; ++k) az_policy_row(acc, q, rows[k], sign);
}

/* quantized_policy_accumulator (src/az.rs:2344-2365): bias row 1545, then
 * every item's 6 rows, per item.  Returns 2 if an item was skipped. */
int oracle_az_policy_refresh(const int8_t* feature_q, const uint32_t* items, const uint32_t* offsets,
                             int64_t n_lists, int16_t* acc) {
  int status = 0;
  for (int64_t l = 0; l < n_lists; ++l) {
    int16_t* a = acc + l * 32;
    memset(a, 0, 64);
    az_policy_row(a, feature_q, 1545, 1);
    for (uint32_t i = offsets[l]; i < offsets[l + 1]; ++i) {
      int r[6];
      if (!az_rows(items[i], r)) { status = 2; continue; }
      az_policy_piece(a, feature_q, r, 1);
    }
  }
  return status;
}

/* apply_quantized_policy_transition (src/az.rs:2367-2409). */
int oracle_az_policy_transition(const int8_t* feature_q, const int16_t* parent, const uint32_t* delta,
                                const uint8_t* refresh, const uint32_t* items, const uint32_t* offsets,
                                int64_t n_lists, int16_t* child) {
  int status = 0;
  for (int64_t l = 0; l < n_lists; ++l) {
    if (refresh[l] & 1) {
      status |= oracle_az_policy_refresh(feature_q, items, offsets + l, 1, child + l * 32);
      continue;
    }
    int16_t* c = child + l * 32;
    memcpy(c, parent + l * 32, 64);
    for (int q = 0; q < 3; ++q) {
      const uint32_t it = delta[3 * l + q];
      if (it == 0xffffffffu) continue;
      int r[6];
      if (!az_rows(it, r)) { status = 2; continue; }
      az_policy_piece(c, feature_q, r, q < 2 ? -1 : 1);
    }
  }
  return status;
}

/* ---- C5: AlphaZero policy/value ResNet (workload specification) -------- */
/* Conventions (the specification leaves them open; the CUDA path follows
 * them): planes [B][15][10][9] (14 piece planes + side to move); stem conv
 * 3x3 15->128, pad 1, + bias, ReLU; 10 blocks h = ReLU(conv1(x) + b1),
 * x = ReLU(conv2(h) + b2 + x); policy head p = ReLU(conv1x1(x, 128->2) + b)
 * flattened channel-major (c * 90 + square) -> FC 180 -> 2086 logits ->
 * softmax; value head v = ReLU(conv1x1(x, 128->1) + b) -> FC 90 -> 256 + ReLU
 * -> FC 256 -> 1 -> tanh.  Weights are bf16 values (BN folded into conv
 * weights and biases); every trunk activation is rounded to bf16 after its
 * layer (the stored dtype), sums are fp32; the heads run in fp32 on the bf16
 * trunk output.  Conv weights OIHW: w[o][c][kh][kw]. */
#define RN_C 128
#define RN_SQ 90
#define RN_MOVES 2086

static void rn_conv3(const float* in, int cin, const float* w, const float* b, const float* resid, float* out) {
  for (int o = 0; o < RN_C; ++o)
    for (int p = 0; p < RN_SQ; ++p) {
      const int r = p / 9, f = p % 9;
      float s = 0.f;
      for (int c = 0; c < cin; ++c)
        for (int kh = 0; kh < 3; ++kh) {
          const int rr = r + kh - 1;
          if (rr < 0 || rr > 9) continue;
          for (int kw = 0; kw < 3; ++kw) {
            const int ff = f + kw - 1;
            if (ff < 0 || ff > 8) continue;
            s += in[c * RN_SQ + rr * 9 + ff] * w[((o * cin + c) * 3 + kh) * 3 + kw];
          }
        }
      s += b[o];
      if (resid) s += resid[o * RN_SQ + p];
      out[o * RN_SQ + p] = bf16_round(s > 0.f ? s : 0.f);
    }
}

void oracle_rn_forward(const float* stem_w, const float* stem_b, const float* block_w, const float* block_b,
                       const float* pcw, const float* pcb, const float* pfw, const float* pfb, const float* vcw,
                       const float* vcb, const float* v1w, const float* v1b, const float* v2w, const float* v2b,
                       const float* planes, int64_t batch, float* logits, float* probs, float* value_pre,
                       float* value, float* trunk) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t bi = 0; bi < batch; ++bi) {
    float* x = (float*)malloc(sizeof(float) * RN_C * RN_SQ);
    float* h = (float*)malloc(sizeof(float) * RN_C * RN_SQ);
    float* y = (float*)malloc(sizeof(float) * RN_C * RN_SQ);
    rn_conv3(planes + bi * 15 * RN_SQ, 15, stem_w, stem_b, NULL, x);
    for (int blk = 0; blk < 10; ++blk) {
      const float* w1 = block_w + (size_t)(2 * blk) * RN_C * RN_C * 9;
      const float* w2 = block_w + (size_t)(2 * blk + 1) * RN_C * RN_C * 9;
      rn_conv3(x, RN_C, w1, block_b + (2 * blk) * RN_C, NULL, h);
      rn_conv3(h, RN_C, w2, block_b + (2 * blk + 1) * RN_C, x, y);
      float* t = x;
      x = y;
      y = t;
    }
    if (trunk) memcpy(trunk + bi * RN_C * RN_SQ, x, sizeof(float) * RN_C * RN_SQ);
    float pc[2 * RN_SQ], vc[RN_SQ], hid[256];
    for (int o = 0; o < 2; ++o)
      for (int p = 0; p < RN_SQ; ++p) {
        float s = 0.f;
        for (int c = 0; c < RN_C; ++c) s += x[c * RN_SQ + p] * pcw[o * RN_C + c];
        s += pcb[o];
        pc[o * RN_SQ + p] = s > 0.f ? s : 0.f;
      }
    for (int p = 0; p < RN_SQ; ++p) {
      float s = 0.f;
      for (int c = 0; c < RN_C; ++c) s += x[c * RN_SQ + p] * vcw[c];
      s += vcb[0];
      vc[p] = s > 0.f ? s : 0.f;
    }
    float* lg = logits + bi * RN_MOVES;
    float mx = -INFINITY;
    for (int j = 0; j < RN_MOVES; ++j) {
      float s = 0.f;
      for (int k = 0; k < 2 * RN_SQ; ++k) s += pc[k] * pfw[j * 2 * RN_SQ + k];
      lg[j] = s + pfb[j];
      if (lg[j] > mx) mx = lg[j];
    }
    double sum = 0.0;
    for (int j = 0; j < RN_MOVES; ++j) sum += exp((double)(lg[j] - mx));
    for (int j = 0; j < RN_MOVES; ++j) probs[bi * RN_MOVES + j] = (float)(exp((double)(lg[j] - mx)) / sum);
    for (int i = 0; i < 256; ++i) {
      float s = 0.f;
      for (int p = 0; p < RN_SQ; ++p) s += vc[p] * v1w[i * RN_SQ + p];
      s += v1b[i];
      hid[i] = s > 0.f ? s : 0.f;
    }
    float s = 0.f;
    for (int i = 0; i < 256; ++i) s += hid[i] * v2w[i];
    s += v2b[0];
    value_pre[bi] = s;
    value[bi] = tanhf(s);
    free(x);
    free(h);
    free(y);
  }
}

/* ---- AZ-NNUE threat features and logits (reference-native) -------------- */
/* threat_reachable_square (src/az.rs:663-697), canonical squares. */
static int az_reach(int piece, int sq) {
  const int r = sq / 9, f = sq % 9, own = piece < 7;
  switch (piece % 7) {
    case 0: return f >= 3 && f <= 5 && (own ? r >= 7 : r <= 2);
    case 1:
      if (own) return (r == 7 && (f == 3 || f == 5)) || (r == 8 && f == 4) || (r == 9 && (f == 3 || f == 5));
      return (r == 0 && (f == 3 || f == 5)) || (r == 1 && f == 4) || (r == 2 && (f == 3 || f == 5));
    case 2:
      if (own)
        return (r == 5 && (f == 2 || f == 6)) || (r == 7 && (f == 0 || f == 4 || f == 8)) || (r == 9 && (f == 2 || f == 6));
      return (r == 0 && (f == 2 || f == 6)) || (r == 2 && (f == 0 || f == 4 || f == 8)) || (r == 4 && (f == 2 || f == 6));
    case 6:
      if (own) return r <= 4 || ((r == 5 || r == 6) && f % 2 == 0);
      return r >= 5 || ((r == 3 || r == 4) && f % 2 == 0);
    default: return 1;
  }
}

static uint32_t* az_rel = NULL; /* [14*90*90] */
static uint8_t az_att[90][14];
static uint32_t az_vocab = 0;

/* threat_relation_map + threat_attacked_offsets (src/az.rs:577-716). */
static void az_threat_init(void) {
  if (az_rel) return;
  uint32_t* rel = (uint32_t*)malloc(sizeof(uint32_t) * 14 * 90 * 90);
  for (int i = 0; i < 14 * 90 * 90; ++i) rel[i] = 0xffffffffu;
  uint32_t next = 0;
  for (int a = 0; a < 14; ++a) {
    const int own = a < 7, kind = a % 7;
    for (int src = 0; src < 90; ++src) {
      if (!az_reach(a, src)) continue;
      const int r = src / 9, f = src % 9;
      int tg[18], n = 0;
      if (kind == 4 || kind == 5) {
        for (int t = 0; t < 90; ++t)
          if (t != src && (t / 9 == r || t % 9 == f)) tg[n++] = t;
      } else {
        int st[8][2], ns = 0;
#define AZ_ST(x, y) (st[ns][0] = (x), st[ns][1] = (y), ++ns)
        if (kind == 0) { AZ_ST(0, -1); AZ_ST(0, 1); AZ_ST(-1, 0); AZ_ST(1, 0); }
        else if (kind == 1) { AZ_ST(-1, -1); AZ_ST(1, -1); AZ_ST(-1, 1); AZ_ST(1, 1); }
        else if (kind == 2) { AZ_ST(-2, -2); AZ_ST(2, -2); AZ_ST(-2, 2); AZ_ST(2, 2); }
        else if (kind == 3) { AZ_ST(-1, -2); AZ_ST(1, -2); AZ_ST(-1, 2); AZ_ST(1, 2); AZ_ST(-2, -1); AZ_ST(-2, 1); AZ_ST(2, -1); AZ_ST(2, 1); }
        else if (own && r <= 4) { AZ_ST(0, -1); AZ_ST(-1, 0); AZ_ST(1, 0); }
        else if (!own && r >= 5) { AZ_ST(0, 1); AZ_ST(-1, 0); AZ_ST(1, 0); }
        else if (own) { AZ_ST(0, -1); }
        else { AZ_ST(0, 1); }
#undef AZ_ST
        for (int i = 0; i < ns; ++i) {
          const int tf = f + st[i][0], tr = r + st[i][1];
          if (tf < 0 || tf > 8 || tr < 0 || tr > 9) continue;
          if ((kind == 0 || kind == 1) && (tf < 3 || tf > 5 || (own ? tr < 7 : tr > 2))) continue;
          if (kind == 2 && (own ? tr < 5 : tr > 4)) continue;
          tg[n++] = tr * 9 + tf;
        }
      }
      for (int i = 0; i < n; ++i) {
        rel[(a * 90 + src) * 90 + tg[i]] = next;
        for (int p = 0; p < 14; ++p) next += (uint32_t)az_reach(p, tg[i]);
      }
    }
  }
  for (int sq = 0; sq < 90; ++sq) {
    int k = 0;
    for (int p = 0; p < 14; ++p) az_att[sq][p] = az_reach(p, sq) ? (uint8_t)k++ : 255;
  }
  az_vocab = next;
  az_rel = rel;
}

int oracle_az_threat_vocab(void) {
  az_threat_init();
  return (int)az_vocab;
}

static void az_threat_push(int persp, int src, int attacker, int tgt, int attacked, uint32_t* out, int* n) {
  const int ai = ((attacker > 0 ? 0 : 1) == persp ? 0 : 7) + (attacker > 0 ? attacker : -attacker) - 1;
  const int vi = ((attacked > 0 ? 0 : 1) == persp ? 0 : 7) + (attacked > 0 ? attacked : -attacked) - 1;
  const int cs = persp == 0 ? src : 89 - src, ct = persp == 0 ? tgt : 89 - tgt;
  const uint32_t base = az_rel[(ai * 90 + cs) * 90 + ct];
  if (base == 0xffffffffu || az_att[ct][vi] == 255) return;
  if (*n < 256) out[(*n)++] = base + az_att[ct][vi];
}

/* visit_occupied_attacks (src/xiangqi/mod.rs:286-389) + value_threat_index
 * (src/az.rs:718-742).  Returns the feature count. */
int oracle_az_threat_features(const int8_t* b, int persp, uint32_t* out) {
  az_threat_init();
  int n = 0;
#define IN(x, y) ((x) >= 0 && (x) < 9 && (y) >= 0 && (y) < 10)
#define HIT(x, y) do { if (IN(x, y) && b[(y) * 9 + (x)]) az_threat_push(persp, s, v, (y) * 9 + (x), b[(y) * 9 + (x)], out, &n); } while (0)
  for (int s = 0; s < 90; ++s) {
    const int v = b[s];
    if (!v) continue;
    const int kind = (v > 0 ? v : -v) - 1, red = v > 0, f = s % 9, r = s / 9;
    if (kind == 0 || kind == 1) {
      static const int o[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
      static const int d[4][2] = {{-1, -1}, {-1, 1}, {1, -1}, {1, 1}};
      for (int i = 0; i < 4; ++i) {
        const int tf = f + (kind ? d[i][0] : o[i][0]), tr = r + (kind ? d[i][1] : o[i][1]);
        if (IN(tf, tr) && tf >= 3 && tf <= 5 && (red ? tr >= 7 : tr <= 2)) HIT(tf, tr);
      }
    } else if (kind == 2) {
      static const int e[4][2] = {{-2, -2}, {-2, 2}, {2, -2}, {2, 2}};
      for (int i = 0; i < 4; ++i) {
        const int tf = f + e[i][0], tr = r + e[i][1];
        if (IN(tf, tr) && (red ? tr >= 5 : tr <= 4) && !b[(r + e[i][1] / 2) * 9 + f + e[i][0] / 2]) HIT(tf, tr);
      }
    } else if (kind == 3) {
      static const int h[8][4] = {{0, -1, -1, -2}, {0, -1, 1, -2}, {0, 1, -1, 2}, {0, 1, 1, 2},
                                  {-1, 0, -2, -1}, {-1, 0, -2, 1}, {1, 0, 2, -1}, {1, 0, 2, 1}};
      for (int i = 0; i < 8; ++i)
        if (IN(f + h[i][2], r + h[i][3]) && IN(f + h[i][0], r + h[i][1]) && !b[(r + h[i][1]) * 9 + f + h[i][0]])
          HIT(f + h[i][2], r + h[i][3]);
    } else if (kind == 4 || kind == 5) {
      static const int o[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
      for (int i = 0; i < 4; ++i) {
        int tf = f + o[i][0], tr = r + o[i][1], occ = 0;
        while (IN(tf, tr)) {
          if (b[tr * 9 + tf]) {
            ++occ;
            if (kind == 4 || occ == 2) {
              az_threat_push(persp, s, v, tr * 9 + tf, b[tr * 9 + tf], out, &n);
              break;
            }
          }
          tf += o[i][0];
          tr += o[i][1];
        }
      }
    } else {
      HIT(f, r + (red ? -1 : 1));
      if (red ? r <= 4 : r >= 5) {
        HIT(f - 1, r);
        HIT(f + 1, r);
      }
    }
  }
#undef HIT
#undef IN
  return n;
}

/* value_threat_logits activation and output (src/az.rs:2103-2119). */
int oracle_az_threat_logits(const int8_t* table, float scale, const float* out_w, const uint32_t* features,
                            const uint32_t* offsets, int64_t n, float* logits, float* act_out) {
  int status = 0;
  for (int64_t p = 0; p < n; ++p) {
    int16_t acc[64];
    memset(acc, 0, sizeof(acc));
    for (uint32_t i = offsets[p]; i < offsets[p + 1]; ++i) {
      if (features[i] >= 57702u) { status = 2; continue; }
      for (int j = 0; j < 64; ++j) acc[j] = (int16_t)(uint16_t)((uint16_t)acc[j] + (uint16_t)(int16_t)table[(size_t)features[i] * 64 + j]);
    }
    float act[128];
    for (int j = 0; j < 64; ++j) {
      float v = (float)acc[j] * scale;
      v = v < 0.f ? 0.f : (v > 1.f ? 1.f : v);
      act[j] = v;
      act[64 + j] = v * v;
    }
    for (int o = 0; o < 3; ++o) logits[p * 3 + o] = az_dot(act, out_w + o * 128, 128);
    if (act_out) memcpy(act_out + p * 128, act, sizeof(act));
  }
  return status;
}

/* ---- AZ-NNUE policy logits (reference-native) --------------------------- */
static int az_gen(const int8_t* b, int color) {
  int g = -1;
  for (int sq = 0; sq < 90; ++sq)
    if (b[sq] == (color == 0 ? 1 : -1)) g = sq;
  return g;
}

/* attacked_squares_mask (src/xiangqi/mod.rs:391-484) as flags. */
static void az_attacked(const int8_t* b, int by, uint8_t* m) {
  memset(m, 0, 90);
#define INB(x, y) ((x) >= 0 && (x) < 9 && (y) >= 0 && (y) < 10)
  const int eg = az_gen(b, 1 - by);
  for (int s = 0; s < 90; ++s) {
    const int v = b[s];
    if (!v || (v > 0 ? 0 : 1) != by) continue;
    const int k = (v > 0 ? v : -v) - 1, f = s % 9, r = s / 9;
    if (k == 0 || k == 1) {
      for (int df = -1; df <= 1; ++df)
        for (int dr = -1; dr <= 1; ++dr) {
          const int ortho = (df == 0) != (dr == 0), diag = df != 0 && dr != 0;
          if (!(k == 0 ? ortho : diag)) continue;
          const int tf = f + df, tr = r + dr;
          if (INB(tf, tr) && tf >= 3 && tf <= 5 && (by == 0 ? tr >= 7 : tr <= 2)) m[tr * 9 + tf] = 1;
        }
      if (k == 0 && eg >= 0 && eg % 9 == f) {
        int clear = 1;
        const int lo = r < eg / 9 ? r : eg / 9, hi = r < eg / 9 ? eg / 9 : r;
        for (int rr = lo + 1; rr < hi; ++rr) clear &= b[rr * 9 + f] == 0;
        if (clear) m[eg] = 1;
      }
    } else if (k == 2) {
      for (int df = -2; df <= 2; df += 4)
        for (int dr = -2; dr <= 2; dr += 4) {
          const int tf = f + df, tr = r + dr;
          if (INB(tf, tr) && (by == 0 ? tr >= 5 : tr <= 4) && !b[(r + dr / 2) * 9 + f + df / 2]) m[tr * 9 + tf] = 1;
        }
    } else if (k == 3) {
      static const int h[8][4] = {{0, -1, -1, -2}, {0, -1, 1, -2}, {0, 1, -1, 2}, {0, 1, 1, 2},
                                  {-1, 0, -2, -1}, {-1, 0, -2, 1}, {1, 0, 2, -1}, {1, 0, 2, 1}};
      for (int i = 0; i < 8; ++i)
        if (INB(f + h[i][2], r + h[i][3]) && !b[(r + h[i][1]) * 9 + f + h[i][0]]) m[(r + h[i][3]) * 9 + f + h[i][2]] = 1;
    } else if (k == 4 || k == 5) {
      static const int o[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
      for (int i = 0; i < 4; ++i) {
        int tf = f + o[i][0], tr = r + o[i][1], seen = 0;
        for (; INB(tf, tr); tf += o[i][0], tr += o[i][1]) {
          const int occ = b[tr * 9 + tf] != 0;
          if (k == 4) {
            m[tr * 9 + tf] = 1;
            if (occ) break;
          } else {
            if (seen) m[tr * 9 + tf] = 1;
            if (occ) {
              if (seen) break;
              seen = 1;
            }
          }
        }
      }
    } else {
      const int fwd = by == 0 ? -1 : 1;
      if (INB(f, r + fwd)) m[(r + fwd) * 9 + f] = 1;
      if (by == 0 ? r <= 4 : r >= 5) {
        if (INB(f - 1, r)) m[r * 9 + f - 1] = 1;
        if (INB(f + 1, r)) m[r * 9 + f + 1] = 1;
      }
    }
  }
}

/* gives_check_after_move_fast (src/xiangqi/mod.rs:763-1012). */
static int az_vocc(const int8_t* b, int from, int to, int sq) { return sq == from ? 0 : (sq == to ? b[from] : b[sq]); }
static int az_between(const int8_t* b, int from, int to, int a, int c) {
  int n = 0;
  if (a % 9 == c % 9) {
    for (int r = (a < c ? a : c) / 9 + 1; r < (a < c ? c : a) / 9; ++r) n += az_vocc(b, from, to, r * 9 + a % 9) != 0;
    return n;
  }
  if (a / 9 == c / 9) {
    const int lo = a % 9 < c % 9 ? a % 9 : c % 9, hi = a % 9 < c % 9 ? c % 9 : a % 9;
    for (int f = lo + 1; f < hi; ++f) n += az_vocc(b, from, to, (a / 9) * 9 + f) != 0;
    return n;
  }
  return 1000;
}

static int az_gives_check(const int8_t* b, int side, int from, int to) {
  const int g = az_gen(b, 1 - side);
  if (g < 0 || !b[from]) return 0;
  const int mv = b[from], color = mv > 0 ? 0 : 1, kind = (mv > 0 ? mv : -mv) - 1;
  const int pf = to % 9, pr = to / 9, gf = g % 9, gr = g / 9, df = gf - pf, dr = gr - pr;
  const int adf = df < 0 ? -df : df, adr = dr < 0 ? -dr : dr;
  int hit = 0;
  if (kind == 0) {
    const int og = az_vocc(b, from, to, g);
    hit = (adf + adr == 1 && gf >= 3 && gf <= 5 && (color == 0 ? gr >= 7 : gr <= 2)) ||
          (pf == gf && og && (og > 0 ? og : -og) == 1 && (og > 0 ? 0 : 1) != color && az_between(b, from, to, to, g) == 0);
  } else if (kind == 1) {
    hit = adf == 1 && adr == 1 && gf >= 3 && gf <= 5 && (color == 0 ? gr >= 7 : gr <= 2);
  } else if (kind == 2) {
    hit = adf == 2 && adr == 2 && (color == 0 ? gr >= 5 : gr <= 4) && !az_vocc(b, from, to, ((pr + gr) / 2) * 9 + (pf + gf) / 2);
  } else if (kind == 3) {
    static const int h[8][4] = {{0, -1, -1, -2}, {0, -1, 1, -2}, {0, 1, -1, 2}, {0, 1, 1, 2},
                                {-1, 0, -2, -1}, {-1, 0, -2, 1}, {1, 0, 2, -1}, {1, 0, 2, 1}};
    for (int i = 0; i < 8; ++i)
      if (df == h[i][2] && dr == h[i][3]) {
        hit = !az_vocc(b, from, to, (pr + h[i][1]) * 9 + pf + h[i][0]);
        break;
      }
  } else if (kind == 4) {
    hit = (pf == gf || pr == gr) && az_between(b, from, to, to, g) == 0;
  } else if (kind == 5) {
    hit = (pf == gf || pr == gr) && az_between(b, from, to, to, g) == 1;
  } else {
    hit = (gf == pf && gr == pr + (color == 0 ? -1 : 1)) || ((color == 0 ? gr <= 4 : gr >= 5) && gr == pr && adf == 1);
  }
  if (hit) return 1;
  static const int o[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};
  for (int i = 0; i < 4; ++i) {
    const int odf = o[i][0], odr = o[i][1];
    const int on_from = odr == 0 ? (from / 9 == gr && (from % 9 - gf) * odf > 0) : (from % 9 == gf && (from / 9 - gr) * odr > 0);
    const int on_to = odr == 0 ? (to / 9 == gr && (to % 9 - gf) * odf > 0) : (to % 9 == gf && (to / 9 - gr) * odr > 0);
    if (!on_from && !on_to) continue;
    int screen = 0;
    for (int nf = gf + odf, nr = gr + odr; INB(nf, nr); nf += odf, nr += odr) {
      const int p = az_vocc(b, from, to, nr * 9 + nf);
      if (!p) continue;
      const int pc = p > 0 ? 0 : 1, pk = (p > 0 ? p : -p) - 1;
      if (!screen) {
        if (pc == side && (pk == 4 || (pk == 0 && odf == 0))) return 1;
        screen = 1;
      } else if (pc == side && pk == 5) {
        return 1;
      } else {
        break;
      }
    }
  }
  static const int h[8][4] = {{0, -1, -1, -2}, {0, -1, 1, -2}, {0, 1, -1, 2}, {0, 1, 1, 2},
                              {-1, 0, -2, -1}, {-1, 0, -2, 1}, {1, 0, 2, -1}, {1, 0, 2, 1}};
  for (int i = 0; i < 8; ++i) {
    const int of = gf - h[i][2], orr = gr - h[i][3];
    if (!INB(of, orr) || !INB(of + h[i][0], orr + h[i][1])) continue;
    const int p = az_vocc(b, from, to, orr * 9 + of);
    if ((orr + h[i][1]) * 9 + of + h[i][0] == from && p == (side == 0 ? 4 : -4)) return 1;
  }
  static const int e[4][4] = {{1, 1, 2, 2}, {1, -1, 2, -2}, {-1, 1, -2, 2}, {-1, -1, -2, -2}};
  for (int i = 0; i < 4; ++i) {
    const int of = gf - e[i][2], orr = gr - e[i][3];
    if (!INB(of, orr) || !INB(of + e[i][0], orr + e[i][1])) continue;
    const int p = az_vocc(b, from, to, orr * 9 + of);
    if ((orr + e[i][1]) * 9 + of + e[i][0] == from && p == (side == 0 ? 3 : -3) && (side == 0 ? gr >= 5 : gr <= 4)) return 1;
  }
#undef INB
  return 0;
}

/* The per-move records of cnnue_az_policy_moves, restated. */
int oracle_az_policy_moves(const int8_t* b, int side, const uint8_t* moves, int n, uint32_t* info) {
  uint16_t d2s[2086], s2d[8100];
  oracle_az_dense_moves(d2s);
  for (int i = 0; i < 8100; ++i) s2d[i] = 0xffff;
  for (int i = 0; i < 2086; ++i) s2d[d2s[i]] = (uint16_t)i;
  uint8_t opp[90], own[90];
  az_attacked(b, 1 - side, opp);
  az_attacked(b, side, own);
  uint32_t items[90];
  const int cnt = oracle_az_features(b, side, items);
  const uint32_t us = cnt ? (items[0] >> 11) & 15 : 4, them = cnt ? (items[0] >> 15) & 15 : 4;
  for (int i = 0; i < n; ++i) {
    const int from = moves[2 * i], to = moves[2 * i + 1];
    const int cf = side == 0 ? from : 89 - from, ct = side == 0 ? to : 89 - to;
    const int v = b[from], c = b[to];
    const uint32_t dense = s2d[cf * 90 + ct] == 0xffff ? 0xfffu : s2d[cf * 90 + ct];
    const uint32_t moved = (uint32_t)(((v > 0 ? 0 : 1) == side ? 0 : 7) + (v > 0 ? v : -v) - 1);
    const uint32_t cap = c ? (uint32_t)(((c > 0 ? 0 : 1) == side ? 0 : 7) + (c > 0 ? c : -c) - 1) : 15u;
    const uint32_t sig = opp[from] | opp[to] << 1 | own[from] << 2 | own[to] << 3 | (c != 0) << 4 |
                         (uint32_t)az_gives_check(b, side, from, to) << 5;
    info[2 * i] = dense | moved << 12 | cap << 16 | sig << 20;
    info[2 * i + 1] = (uint32_t)cf | (uint32_t)ct << 7 | us << 14 | them << 18;
  }
  return 0;
}

/* evaluate_prepared_hidden_with_context (src/az.rs:1766-1887) per move.
 * t = the 22 tensors; q = the oracle's quantised tables (feature, move,
 * sparse, moved delta, capture); x [n][h] normalised hidden; act [n][128]
 * threat activations or NULL; pacc [n][32]. */
int oracle_az_policy_logits(const float* const* t, int h, const int8_t* move_q, const int8_t* sparse_q,
                            const int32_t* mdelta, const int32_t* mcap, const float* scales, int tactical_active,
                            const float* x, const float* act, const int16_t* pacc, const uint32_t* info,
                            const uint32_t* offsets, int64_t n, float* logits) {
  float ps[1260];
  const int cs = h < 32 ? h : 32;
  for (int f = 0; f < 1260; ++f) ps[f] = az_dot(t[0] + (int64_t)f * h, t[14], cs);
  for (int64_t p = 0; p < n; ++p) {
    float ctx[16];
    for (int c = 0; c < 16; ++c) {
      ctx[c] = az_dot(x + p * h, t[15] + (int64_t)c * h, h);
      if (act) ctx[c] += az_dot(act + p * 128, t[12] + c * 128, 128);
    }
    for (uint32_t j = offsets[p]; j < offsets[p + 1]; ++j) {
      const uint32_t w0 = info[2 * j], w1 = info[2 * j + 1];
      const uint32_t dense = w0 & 0xfff, moved = (w0 >> 12) & 15, cap = (w0 >> 16) & 15, sig = (w0 >> 20) & 63;
      const uint32_t cf = w1 & 127, ct = (w1 >> 7) & 127, us = (w1 >> 14) & 15, them = (w1 >> 18) & 15;
      float psl = ps[moved * 90 + ct] - ps[moved * 90 + cf];
      psl = psl - (cap < 14 ? ps[cap * 90 + ct] : 0.f);
      const float cdot = az_dot(ctx, t[16] + dense * 16, 16);
      int32_t v = 0;
      for (int k = 0; k < 32; ++k) v += (int32_t)pacc[p * 32 + k] * (int32_t)move_q[dense * 32 + k];
      v += mdelta[dense * 14 + moved];
      if (cap < 14) v -= mcap[dense * 14 + cap];
      const float accl = (float)v * scales[0] * scales[1];
      const int64_t main = (((int64_t)dense * 14 + moved) * 9 + us) * 9 + them;
      const int64_t capi = 2086LL * 14 * 81 + dense * 15 + (cap < 14 ? cap : 14);
      const float sparse = (float)((int32_t)sparse_q[main] + (int32_t)sparse_q[capi]) * scales[2];
      float tactical = 0.f;
      if (tactical_active) {
        const int64_t exact = ((int64_t)dense * 7 + moved) * 64 + sig, factor = 2086LL * 7 * 64 + moved * 64 + sig;
        tactical = t[21][exact] + t[21][factor];
      }
      logits[j] = t[13][dense] + psl + cdot + accl + sparse + tactical;
    }
  }
  return 0;
}
