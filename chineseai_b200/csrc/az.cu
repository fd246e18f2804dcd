// az.cu - device side of the reference-native AZ-NNUE evaluator: the trunk
// accumulator refresh, its incremental transition, and the value head.
//
// The trunk of one perspective is a sum of fp32 rows of five tables, which the
// model keeps concatenated as one [1545][H] table (input 0, piece 1260, rank
// 1274, file 1284, king-piece 1293; the feature-pool layout of
// src/az/fused_feature_pool.rs:12-19).  Refresh and transition run one warp per
// item list; lane l owns the columns of chunks l, l+32, ... (a chunk is a
// float4 when H is a multiple of 4, else one float), so each column is summed
// by one thread in exactly the reference's row order, one IEEE add or
// subtract per row, which makes the accumulators bit-identical to the CPU
// ones.  Row loads of several items are issued before their adds so a warp
// keeps up to 20 row loads in flight; the table (H = 128: 791 KB) stays in L2.
//
// The value head runs one warp per 4 positions: x = ReLU(acc + rule rows),
// RMSNorm, then lane k computes value units k, k+32, k+64 for all 4 positions
// from the transposed head weights [H][96] held in shared memory, and the 3
// logits are warp sums.
#include <cfloat>
#include <cstring>

#include "az_weights.h"
#include "common.cuh"

struct cnnue_az_model {
  int device = 0;
  int64_t hidden = 0;
  void* blob = nullptr;
  float* trunk = nullptr;   // [1545][H]
  float* bias = nullptr;    // [H]
  float* rule = nullptr;    // [7][H]
  float* head_t = nullptr;  // value_head_hidden transposed, [H][96]
  float* head_b = nullptr;  // [96]
  float* head_o = nullptr;  // [3][96]
  int8_t* policy_q = nullptr;  // quantised policy feature rows [1546][32]
  int8_t* threat_q = nullptr;  // quantised threat embedding [57702][64]
  float* threat_out = nullptr; // value_threat_output [3][128]
  float threat_scale = 1.f;
  // policy head (evaluate_prepared_hidden_with_context, src/az.rs:1766-1887)
  float* ps_scores = nullptr;      // [1260] piece-square consequence scores
  float* move_bias = nullptr;      // [2086]
  float* move_context = nullptr;   // [2086][16]
  float* context_hidden = nullptr; // [16][H]
  float* threat_context = nullptr; // [16][128]
  int8_t* move_q = nullptr;        // [2086][32]
  int32_t* moved_delta = nullptr;  // [2086][14]
  int32_t* capture = nullptr;      // [2086][14]
  int8_t* sparse_q = nullptr;      // [2396815]
  float* tactical = nullptr;       // [934976]
  float feature_scale = 1.f, move_scale = 1.f, sparse_scale = 1.f;
  int threat_active = 0, tactical_active = 0;
  void* policy_blob = nullptr;
};

namespace cnnue {
namespace {

constexpr int kRows = CNNUE_AZ_TRUNK_ROWS;
constexpr int kHead = CNNUE_AZ_VALUE_HEAD;
constexpr int kListWarps = 8;  // warps per CTA of the refresh / transition kernels
constexpr int kValuePos = 4;   // positions per warp in the value head
constexpr unsigned kFull = 0xffffffffu;

// Row indices of an item: input, piece, rank, file, king(us), king(them).
// Returns false (rows all 0) for a feature >= 1260 or a bucket > 8.
__device__ __forceinline__ bool item_rows(uint32_t item, uint32_t r[6]) {
  const uint32_t feature = item & 0x7ffu, us = (item >> 11) & 0xfu, them = (item >> 15) & 0xfu;
  const bool ok = feature < (uint32_t)CNNUE_AZ_INPUT && us <= 8u && them <= 8u && (item >> 19) == 0u;
  const uint32_t f = ok ? feature : 0u;
  const uint32_t piece = f / 90u, sq = f - piece * 90u;
  r[0] = f;
  r[1] = 1260u + piece;
  r[2] = 1274u + sq / 9u;
  r[3] = 1284u + sq % 9u;
  r[4] = 1293u + (ok ? us : 0u) * 14u + piece;
  r[5] = 1293u + (9u + (ok ? them : 0u)) * 14u + piece;
  return ok;
}

// Columns of one lane: K chunks of VW floats.
template <int VW, int K>
struct Cols {
  float v[K][VW];
};

template <int VW, int K>
__device__ __forceinline__ void load_cols(const float* __restrict__ row, int chunks, int lane, Cols<VW, K>& c) {
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int ch = lane + 32 * k;
    if (ch < chunks) {
      if constexpr (VW == 4) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(row) + ch);
        c.v[k][0] = x.x;
        c.v[k][1] = x.y;
        c.v[k][2] = x.z;
        c.v[k][3] = x.w;
      } else {
        c.v[k][0] = __ldg(row + ch);
      }
    } else {
#pragma unroll
      for (int e = 0; e < VW; ++e) c.v[k][e] = 0.f;
    }
  }
}

template <int VW, int K>
__device__ __forceinline__ void store_cols(float* __restrict__ row, int chunks, int lane, const Cols<VW, K>& c) {
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int ch = lane + 32 * k;
    if (ch < chunks) {
      if constexpr (VW == 4) {
        reinterpret_cast<float4*>(row)[ch] = make_float4(c.v[k][0], c.v[k][1], c.v[k][2], c.v[k][3]);
      } else {
        row[ch] = c.v[k][0];
      }
    }
  }
}

template <int kSign>
__device__ __forceinline__ void add_pair_rn(float& a0, float& a1, float b0, float b1) {
  if constexpr (kSign > 0)
    fadd2_rn(a0, a1, b0, b1);
  else
    fsub2_rn(a0, a1, b0, b1);
}

// a += w (kSign > 0) or a -= w, one rounding per element (packed in pairs
// of columns for 4-wide chunks: half the add instructions).
template <int kSign, int VW, int K>
__device__ __forceinline__ void accumulate(Cols<VW, K>& a, const Cols<VW, K>& w) {
#pragma unroll
  for (int k = 0; k < K; ++k) {
    if constexpr (VW == 4) {
      add_pair_rn<kSign>(a.v[k][0], a.v[k][1], w.v[k][0], w.v[k][1]);
      add_pair_rn<kSign>(a.v[k][2], a.v[k][3], w.v[k][2], w.v[k][3]);
    } else {
#pragma unroll
      for (int e = 0; e < VW; ++e)
        a.v[k][e] = kSign > 0 ? __fadd_rn(a.v[k][e], w.v[k][e]) : __fsub_rn(a.v[k][e], w.v[k][e]);
    }
  }
}

// acc += the rows of the items [beg, end) in the reference's refresh order:
// the input row of every item, then for every item its five structural rows.
// Returns CNNUE_STATUS_BAD_INDEX if an item was skipped.
template <int VW, int K>
__device__ uint32_t add_list(const float* __restrict__ trunk, int H, int chunks, const uint32_t* __restrict__ items,
                             uint32_t beg, uint32_t end, int lane, Cols<VW, K>& a) {
  // Rows loaded ahead of their adds, about 32-40 registers of row data.
  constexpr int kRowRegs = VW * K;
  constexpr int kIn = 32 / kRowRegs > 0 ? 32 / kRowRegs : 1;            // input rows
  constexpr int kSt = 40 / (5 * kRowRegs) > 0 ? 40 / (5 * kRowRegs) : 1;  // items of 5 structural rows
  uint32_t bad = 0;
  for (int pass = 0; pass < 2; ++pass) {
    for (uint32_t base = beg; base < end; base += 32) {
      const uint32_t mine = base + lane < end ? items[base + lane] : 0u;
      uint32_t r[6];
      const bool ok = item_rows(mine, r);
      if (base + lane < end && !ok) bad = CNNUE_STATUS_BAD_INDEX;
      const uint32_t ok_mask = __ballot_sync(kFull, ok);
      const int cnt = (int)min(32u, end - base);
      if (pass == 0) {
        for (int j0 = 0; j0 < cnt; j0 += kIn) {
          Cols<VW, K> w[kIn];
#pragma unroll
          for (int b = 0; b < kIn; ++b) {
            const uint32_t row = __shfl_sync(kFull, r[0], (j0 + b) & 31);
            if (j0 + b < cnt) load_cols(trunk + (size_t)row * H, chunks, lane, w[b]);
          }
#pragma unroll
          for (int b = 0; b < kIn; ++b)
            if (j0 + b < cnt && ((ok_mask >> (j0 + b)) & 1u)) accumulate<1>(a, w[b]);
        }
      } else {
        for (int j0 = 0; j0 < cnt; j0 += kSt) {
          Cols<VW, K> w[kSt][5];
#pragma unroll
          for (int b = 0; b < kSt; ++b) {
#pragma unroll
            for (int s = 0; s < 5; ++s) {
              const uint32_t row = __shfl_sync(kFull, r[s + 1], (j0 + b) & 31);
              if (j0 + b < cnt) load_cols(trunk + (size_t)row * H, chunks, lane, w[b][s]);
            }
          }
#pragma unroll
          for (int b = 0; b < kSt; ++b)
            if (j0 + b < cnt && ((ok_mask >> (j0 + b)) & 1u))
#pragma unroll
              for (int s = 0; s < 5; ++s) accumulate<1>(a, w[b][s]);
        }
      }
    }
  }
  return bad;
}

// a -= 6 rows (kSign < 0) or a += 6 rows of one item, in the order input,
// piece, rank, file, king(us), king(them).
template <int kSign, int VW, int K>
__device__ __forceinline__ uint32_t apply_item(const float* __restrict__ trunk, int H, int chunks, uint32_t item,
                                               int lane, Cols<VW, K>& a) {
  if (item == CNNUE_AZ_NO_ITEM) return 0u;
  uint32_t r[6];
  if (!item_rows(item, r)) return CNNUE_STATUS_BAD_INDEX;
  Cols<VW, K> w[6];
#pragma unroll
  for (int s = 0; s < 6; ++s) load_cols(trunk + (size_t)r[s] * H, chunks, lane, w[s]);
#pragma unroll
  for (int s = 0; s < 6; ++s) accumulate<kSign>(a, w[s]);
  return 0u;
}

struct ListArgs {
  const float* trunk;
  const float* bias;
  int H;
  int chunks;
  const uint32_t* items;
  uint32_t n_items;
  const uint32_t* offsets;
  int64_t n_lists;
  // transition only
  const float* parent;
  const uint32_t* delta;
  const uint8_t* refresh;
  float* out;
  WorkspaceHeader* hdr;
};

// One warp per list.  kTransition: parent +- delta rows unless refresh[l].
template <bool kTransition, int VW, int K>
__global__ void __launch_bounds__(kListWarps * 32) az_list_kernel(ListArgs p) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * kListWarps;
  uint32_t status = 0;
  for (int64_t l = (int64_t)blockIdx.x * kListWarps + (threadIdx.x >> 5); l < p.n_lists; l += warps) {
    Cols<VW, K> a;
    const bool do_refresh = !kTransition || (p.refresh[l] & 1u);
    if (do_refresh) {
      load_cols(p.bias, p.chunks, lane, a);
      if (p.offsets == nullptr) {
        status |= CNNUE_STATUS_BAD_OFFSETS;
      } else {
        const uint32_t beg = p.offsets[l], end = p.offsets[l + 1];
        if (beg <= end && end <= p.n_items)
          status |= add_list(p.trunk, p.H, p.chunks, p.items, beg, end, lane, a);
        else
          status |= CNNUE_STATUS_BAD_OFFSETS;
      }
    } else {
      load_cols(p.parent + (size_t)l * p.H, p.chunks, lane, a);
      const uint32_t from = p.delta[3 * l], captured = p.delta[3 * l + 1], to = p.delta[3 * l + 2];
      status |= apply_item<-1>(p.trunk, p.H, p.chunks, from, lane, a);
      status |= apply_item<-1>(p.trunk, p.H, p.chunks, captured, lane, a);
      status |= apply_item<1>(p.trunk, p.H, p.chunks, to, lane, a);
    }
    store_cols(p.out + (size_t)l * p.H, p.chunks, lane, a);
  }
  status = __reduce_or_sync(kFull, status);
  if (lane == 0 && status) atomicOr(&p.hdr->status, status);
}

template <bool kTransition>
int launch_list(const ListArgs& a, cudaStream_t s) {
  const bool vec = a.H % 4 == 0;
  const int chunks = vec ? a.H / 4 : a.H;
  const int k = (chunks + 31) / 32;
  ListArgs p = a;
  p.chunks = chunks;
  const int64_t want = (a.n_lists + kListWarps - 1) / kListWarps;
  const unsigned blocks = (unsigned)(want < 148 * 32 ? want : 148 * 32);
  const dim3 block(kListWarps * 32);
  if (vec) {
    if (k <= 1) az_list_kernel<kTransition, 4, 1><<<blocks, block, 0, s>>>(p);
    else if (k <= 2) az_list_kernel<kTransition, 4, 2><<<blocks, block, 0, s>>>(p);
    else az_list_kernel<kTransition, 4, 4><<<blocks, block, 0, s>>>(p);
  } else {  // H < 128 (checked at model creation)
    if (k <= 1) az_list_kernel<kTransition, 1, 1><<<blocks, block, 0, s>>>(p);
    else if (k <= 2) az_list_kernel<kTransition, 1, 2><<<blocks, block, 0, s>>>(p);
    else az_list_kernel<kTransition, 1, 4><<<blocks, block, 0, s>>>(p);
  }
  return check_launch_error(kTransition ? "az_list_kernel<transition>" : "az_list_kernel<refresh>");
}

// ---- value head ------------------------------------------------------------
struct ValueArgs {
  const float* head_t;  // [H][96]
  const float* head_b;  // [96]
  const float* head_o;  // [3][96]
  const float* rule_rows;  // [7][H]
  int H;
  const float* acc;
  const uint8_t* side;
  const float* rule;
  const float* threat;
  int64_t n;
  float* wdl;
  float* q;
  float* x_out;  // optional [n][H]: the normalised hidden the policy head reads
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// Dynamic shared memory: head_t [H][96], head_o [3][96], head_b [96], then
// per warp x [kValuePos][H].
__global__ void __launch_bounds__(256) az_value_kernel(ValueArgs p) {
  extern __shared__ float sm[];
  const int H = p.H, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  float* w_t = sm;
  float* w_o = w_t + (size_t)H * kHead;
  float* w_b = w_o + 3 * kHead;
  float* xs = w_b + kHead + (size_t)warp * kValuePos * H;
  for (int i = threadIdx.x; i < H * kHead; i += blockDim.x) w_t[i] = p.head_t[i];
  for (int i = threadIdx.x; i < 3 * kHead; i += blockDim.x) w_o[i] = p.head_o[i];
  for (int i = threadIdx.x; i < kHead; i += blockDim.x) w_b[i] = p.head_b[i];
  __syncthreads();

  const int64_t groups = (p.n + kValuePos - 1) / kValuePos;
  for (int64_t g = (int64_t)blockIdx.x * nwarps + warp; g < groups; g += (int64_t)gridDim.x * nwarps) {
    // 1. x = ReLU(acc + rule context), then RMSNorm.
#pragma unroll
    for (int i = 0; i < kValuePos; ++i) {
      const int64_t pos = g * kValuePos + i;
      float* x = xs + i * H;
      if (pos >= p.n) {
        for (int c = lane; c < H; c += 32) x[c] = 0.f;
        continue;
      }
      const float* src = p.acc + (p.side ? ((size_t)pos * 2 + (p.side[pos] ? 1 : 0)) : (size_t)pos) * H;
      float rule[CNNUE_AZ_RULE_CONTEXT];
#pragma unroll
      for (int k = 0; k < CNNUE_AZ_RULE_CONTEXT; ++k) rule[k] = p.rule ? p.rule[pos * CNNUE_AZ_RULE_CONTEXT + k] : 0.f;
      float ss = 0.f;
      for (int c = lane; c < H; c += 32) {
        float v = src[c];
#pragma unroll
        for (int k = 0; k < CNNUE_AZ_RULE_CONTEXT; ++k)
          if (rule[k] != 0.f) v = __fadd_rn(v, __fmul_rn(rule[k], p.rule_rows[(size_t)k * H + c]));
        v = fmaxf(v, 0.f);
        ss = fmaf(v, v, ss);
        x[c] = v;
      }
      ss = warp_sum(ss);
      const float inv = 1.0f / sqrtf(ss / (float)H + 1e-6f);
      for (int c = lane; c < H; c += 32) {
        x[c] *= inv;
        if (p.x_out) p.x_out[(size_t)pos * H + c] = x[c];
      }
    }
    __syncwarp();
    // 2. value units k, k+32, k+64 of the 4 positions.
    float d[kValuePos][3];
#pragma unroll
    for (int i = 0; i < kValuePos; ++i) d[i][0] = d[i][1] = d[i][2] = 0.f;
    for (int j = 0; j < H; ++j) {
      const float w0 = w_t[j * kHead + lane], w1 = w_t[j * kHead + lane + 32], w2 = w_t[j * kHead + lane + 64];
#pragma unroll
      for (int i = 0; i < kValuePos; ++i) {
        const float xv = xs[i * H + j];
        d[i][0] = fmaf(xv, w0, d[i][0]);
        d[i][1] = fmaf(xv, w1, d[i][1]);
        d[i][2] = fmaf(xv, w2, d[i][2]);
      }
    }
    // 3. logits, softmax, q.
    float logit[kValuePos][3];
#pragma unroll
    for (int i = 0; i < kValuePos; ++i) {
      const float v0 = fmaxf(w_b[lane] + d[i][0], 0.f), v1 = fmaxf(w_b[lane + 32] + d[i][1], 0.f),
                  v2 = fmaxf(w_b[lane + 64] + d[i][2], 0.f);
#pragma unroll
      for (int o = 0; o < 3; ++o)
        logit[i][o] = warp_sum(v0 * w_o[o * kHead + lane] + v1 * w_o[o * kHead + lane + 32] +
                               v2 * w_o[o * kHead + lane + 64]);
    }
#pragma unroll
    for (int i = 0; i < kValuePos; ++i) {
      const int64_t pos = g * kValuePos + i;
      if (lane == i && pos < p.n) {
        float l[3];
#pragma unroll
        for (int o = 0; o < 3; ++o) l[o] = logit[i][o] + (p.threat ? p.threat[pos * 3 + o] : 0.f);
        const float m = fmaxf(fmaxf(fmaxf(-INFINITY, l[0]), l[1]), l[2]);
        const float e0 = expf(l[0] - m), e1 = expf(l[1] - m), e2 = expf(l[2] - m);
        const float sum = fmaxf(e0 + e1 + e2, FLT_MIN);
        const float p0 = e0 / sum, p1 = e1 / sum, p2 = e2 / sum;
        p.wdl[pos * 3 + 0] = p0;
        p.wdl[pos * 3 + 1] = p1;
        p.wdl[pos * 3 + 2] = p2;
        p.q[pos] = p0 - p2;
      }
    }
    __syncwarp();
  }
}

size_t value_smem_bytes(int64_t H, int warps) {
  return sizeof(float) * ((size_t)H * kHead + 4 * kHead + (size_t)warps * kValuePos * H);
}

constexpr size_t kMaxSmem = 227 * 1024;

int value_warps(int64_t H) {
  int w = 8;
  while (w > 1 && value_smem_bytes(H, w) > kMaxSmem) w >>= 1;
  return w;
}

__global__ void transpose_head_kernel(const float* __restrict__ w, int H, float* __restrict__ wt) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < (int64_t)H * kHead) {
    const int64_t k = i / H, j = i - k * H;  // w[k][j] -> wt[j][k]
    wt[j * kHead + k] = w[i];
  }
}

// ---- int16 policy accumulator ----------------------------------------------
// 4 lists per warp, 8 lanes per list; lane s of a list owns ranks 4s..4s+3 as
// two words of int16 pairs.  The int8 table is widened into shared memory as
// [1546][16] words, so one row add is one 8-byte shared load and two
// saturating pair adds (__vaddss2 / __vsubss2).
constexpr int kPolicyWarps = 8;
constexpr size_t kPolicySmem = (size_t)CNNUE_AZ_POLICY_ROWS * CNNUE_AZ_POLICY_RANK * 2;

struct PolicyArgs {
  const int8_t* q;
  const uint32_t* items;
  uint32_t n_items;
  const uint32_t* offsets;
  int64_t n_lists;
  const int16_t* parent;
  const uint32_t* delta;
  const uint8_t* refresh;
  int16_t* out;
  WorkspaceHeader* hdr;
};

__device__ __forceinline__ uint32_t widen2(uint32_t b) {  // int8 bytes 0,1 -> int16 pair
  return (uint32_t)(uint16_t)(int16_t)(int8_t)(b & 0xffu) | ((uint32_t)(uint16_t)(int16_t)(int8_t)((b >> 8) & 0xffu) << 16);
}

template <int kSign>
__device__ __forceinline__ void policy_row(const uint2* __restrict__ tab, uint32_t row, int sub, uint32_t& a0, uint32_t& a1) {
  const uint2 w = tab[row * 8 + sub];
  if (kSign > 0) {
    a0 = __vaddss2(a0, w.x);
    a1 = __vaddss2(a1, w.y);
  } else {
    a0 = __vsubss2(a0, w.x);
    a1 = __vsubss2(a1, w.y);
  }
}

template <int kSign>
__device__ __forceinline__ void policy_item(const uint2* __restrict__ tab, const uint32_t r[6], int sub, uint32_t& a0,
                                            uint32_t& a1) {
#pragma unroll
  for (int k = 0; k < 6; ++k) policy_row<kSign>(tab, r[k], sub, a0, a1);
}

template <bool kTransition>
__global__ void __launch_bounds__(kPolicyWarps * 32) az_policy_kernel(PolicyArgs p) {
  extern __shared__ uint2 ptab[];  // [1546][8] uint2 = [1546][32] int16
  const uint32_t* q32 = reinterpret_cast<const uint32_t*>(p.q);
  uint32_t* t32 = reinterpret_cast<uint32_t*>(ptab);
  for (int i = threadIdx.x; i < CNNUE_AZ_POLICY_ROWS * CNNUE_AZ_POLICY_RANK / 4; i += blockDim.x) {
    const uint32_t v = __ldg(q32 + i);
    t32[2 * i] = widen2(v);
    t32[2 * i + 1] = widen2(v >> 16);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, group = lane >> 3, sub = lane & 7;
  const unsigned gmask = 0xffu << (8 * group);
  uint32_t status = 0;
  const int64_t stride = (int64_t)gridDim.x * kPolicyWarps * 4;
  for (int64_t base = ((int64_t)blockIdx.x * kPolicyWarps + (threadIdx.x >> 5)) * 4; base < p.n_lists; base += stride) {
    const int64_t l = base + group;
    if (l < p.n_lists) {
      uint32_t a0 = 0, a1 = 0;
      const bool do_refresh = !kTransition || (p.refresh[l] & 1u);
      if (do_refresh) {
        policy_row<1>(ptab, CNNUE_AZ_POLICY_ROWS - 1, sub, a0, a1);  // bias row
        uint32_t beg = 0, end = 0;
        if (p.offsets == nullptr) {
          status |= CNNUE_STATUS_BAD_OFFSETS;
        } else {
          beg = p.offsets[l];
          end = p.offsets[l + 1];
          if (!(beg <= end && end <= p.n_items)) {
            status |= CNNUE_STATUS_BAD_OFFSETS;
            beg = end = 0;
          }
        }
        for (uint32_t b = beg; b < end; b += 8) {
          const uint32_t mine = b + sub < end ? p.items[b + sub] : 0u;
          const uint32_t cnt = min(8u, end - b);
          for (uint32_t k = 0; k < cnt; ++k) {
            const uint32_t it = __shfl_sync(gmask, mine, (int)k, 8);
            uint32_t r[6];
            if (item_rows(it, r)) policy_item<1>(ptab, r, sub, a0, a1);
            else status |= CNNUE_STATUS_BAD_INDEX;
          }
        }
      } else {
        const uint2 par = reinterpret_cast<const uint2*>(p.parent + l * CNNUE_AZ_POLICY_RANK)[sub];
        a0 = par.x;
        a1 = par.y;
#pragma unroll
        for (int d = 0; d < 3; ++d) {
          const uint32_t it = p.delta[3 * l + d];
          if (it == CNNUE_AZ_NO_ITEM) continue;
          uint32_t r[6];
          if (!item_rows(it, r)) {
            status |= CNNUE_STATUS_BAD_INDEX;
            continue;
          }
          if (d < 2) policy_item<-1>(ptab, r, sub, a0, a1);
          else policy_item<1>(ptab, r, sub, a0, a1);
        }
      }
      reinterpret_cast<uint2*>(p.out + l * CNNUE_AZ_POLICY_RANK)[sub] = make_uint2(a0, a1);
    }
  }
  status = __reduce_or_sync(kFull, status);
  if (lane == 0 && status) atomicOr(&p.hdr->status, status);
}

template <bool kTransition>
int launch_policy(const PolicyArgs& a, cudaStream_t s) {
  const int64_t want = (a.n_lists + 4 * kPolicyWarps - 1) / (4 * kPolicyWarps);
  const unsigned blocks = (unsigned)(want < 148 * 2 ? want : 148 * 2);
  az_policy_kernel<kTransition><<<blocks, kPolicyWarps * 32, kPolicySmem, s>>>(a);
  return check_launch_error(kTransition ? "az_policy_kernel<transition>" : "az_policy_kernel<refresh>");
}

// ---- threat logits (value_threat_logits, src/az.rs:2078-2120) -------------
// One warp per position: lane l owns threat ranks 2l, 2l+1 as one word of an
// int16 pair; each feature row (64 int8) is widened and added with wrapping
// (__vadd2, as the reference's epi16 adds), which makes the sum independent
// of the feature order.  Then act = clamp(acc * scale, 0, 1) and act^2 go to
// shared memory and lanes 0-2 form the three logits with the reference's
// x86-64 AVX2/FMA dot-product order (four 8-lane fused accumulators over
// 32-element chunks, lanes combined (a0 + a1) + (a2 + a3), then summed).
constexpr int kThreatWarps = 8;

__global__ void __launch_bounds__(kThreatWarps * 32) az_threat_kernel(
    const int8_t* __restrict__ table, float scale, const float* __restrict__ out_w,
    const uint32_t* __restrict__ features, uint32_t n_features, const uint32_t* __restrict__ offsets, int64_t n,
    float* __restrict__ logits, float* __restrict__ act_out, WorkspaceHeader* hdr) {
  __shared__ float act[kThreatWarps][2 * CNNUE_AZ_THREAT_RANK];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t status = 0;
  for (int64_t p = (int64_t)blockIdx.x * kThreatWarps + warp; p < n; p += (int64_t)gridDim.x * kThreatWarps) {
    const uint32_t beg = offsets[p], end = offsets[p + 1];
    uint32_t acc = 0;
    if (beg <= end && end <= n_features) {
      for (uint32_t i = beg; i < end; ++i) {
        const uint32_t f = features[i];
        if (f >= (uint32_t)CNNUE_AZ_THREAT_VOCAB) {
          status |= CNNUE_STATUS_BAD_INDEX;
          continue;
        }
        const uint16_t two = __ldg(reinterpret_cast<const uint16_t*>(table + (size_t)f * CNNUE_AZ_THREAT_RANK) + lane);
        acc = __vadd2(acc, widen2(two));
      }
    } else {
      status |= CNNUE_STATUS_BAD_OFFSETS;
    }
    const float x0 = fminf(fmaxf(__fmul_rn((float)(int16_t)(acc & 0xffffu), scale), 0.f), 1.f);
    const float x1 = fminf(fmaxf(__fmul_rn((float)(int16_t)(acc >> 16), scale), 0.f), 1.f);
    float* a = act[warp];
    a[2 * lane] = x0;
    a[2 * lane + 1] = x1;
    a[CNNUE_AZ_THREAT_RANK + 2 * lane] = __fmul_rn(x0, x0);
    a[CNNUE_AZ_THREAT_RANK + 2 * lane + 1] = __fmul_rn(x1, x1);
    __syncwarp();
    if (act_out) {
      float* o = act_out + (size_t)p * 2 * CNNUE_AZ_THREAT_RANK;
      for (int i = lane; i < 2 * CNNUE_AZ_THREAT_RANK; i += 32) o[i] = a[i];
    }
    if (lane < 3) {
      const float* w = out_w + lane * 2 * CNNUE_AZ_THREAT_RANK;
      float part[4][8];
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int k = 0; k < 8; ++k) part[q][k] = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int k = 0; k < 8; ++k) part[q][k] = fmaf(a[c * 32 + q * 8 + k], __ldg(w + c * 32 + q * 8 + k), part[q][k]);
      float sum = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) sum = __fadd_rn(sum, __fadd_rn(__fadd_rn(part[0][k], part[1][k]), __fadd_rn(part[2][k], part[3][k])));
      logits[p * 3 + lane] = sum;
    }
    __syncwarp();
  }
  status = __reduce_or_sync(kFull, status);
  if (lane == 0 && status) atomicOr(&hdr->status, status);
}

// ---- policy logits (evaluate_prepared_hidden_with_context) -----------------
// One warp per position.  Lanes 0-15 form the 16 context values (normalised
// hidden . policy_context_hidden[c], + threat activation .
// policy_threat_context[c] when the threat branch is active); then each lane
// takes moves j = lane, lane + 32, ... and sums the six terms in the
// reference's order: move bias, piece-square consequence, context . move
// context, quantised accumulator, folded sparse table, tactical table.
constexpr int kPolicyLogitWarps = 8;
constexpr int64_t kSparseMain = (int64_t)CNNUE_AZ_DENSE_MOVES * 14 * 81;
constexpr int64_t kTacticalExact = (int64_t)CNNUE_AZ_DENSE_MOVES * 7 * 64;

struct PolicyLogitArgs {
  const float* x;          // [n][H] normalised hidden
  const float* threat_act; // [n][128] or null
  const int16_t* pacc;     // [n][32] or [n][2][32] with side
  const uint8_t* side;
  const uint32_t* info;    // [moves][2]
  uint32_t n_moves;
  const uint32_t* offsets; // [n+1]
  int64_t n;
  int H;
  float* logits;
  WorkspaceHeader* hdr;
  // model tables
  const float* ps;
  const float* bias;
  const float* mctx;
  const float* pch;
  const float* ptc;
  const int8_t* mq;
  const int32_t* mdelta;
  const int32_t* mcap;
  const int8_t* sq;
  const float* tac;
  float fscale, mscale, sscale;
  int tactical_active;
};

__global__ void __launch_bounds__(kPolicyLogitWarps * 32) az_policy_logits_kernel(PolicyLogitArgs a) {
  __shared__ float ctx[kPolicyLogitWarps][16];
  __shared__ int16_t pacc[kPolicyLogitWarps][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t status = 0;
  for (int64_t p = (int64_t)blockIdx.x * kPolicyLogitWarps + warp; p < a.n; p += (int64_t)gridDim.x * kPolicyLogitWarps) {
    if (lane < 16) {
      const float* x = a.x + (size_t)p * a.H;
      const float* w = a.pch + (size_t)lane * a.H;
      float c = 0.f;
      for (int j = 0; j < a.H; ++j) c = fmaf(__ldg(x + j), __ldg(w + j), c);
      if (a.threat_act) {
        const float* t = a.threat_act + (size_t)p * 2 * CNNUE_AZ_THREAT_RANK;
        const float* tw = a.ptc + lane * 2 * CNNUE_AZ_THREAT_RANK;
        float d = 0.f;
        for (int j = 0; j < 2 * CNNUE_AZ_THREAT_RANK; ++j) d = fmaf(__ldg(t + j), __ldg(tw + j), d);
        c += d;
      }
      ctx[warp][lane] = c;
    }
    const int16_t* prow = a.pacc + (a.side ? ((size_t)p * 2 + (a.side[p] ? 1 : 0)) : (size_t)p) * 32;
    pacc[warp][lane] = prow[lane];
    __syncwarp();
    const uint32_t beg = a.offsets[p], end = a.offsets[p + 1];
    if (!(beg <= end && end <= a.n_moves)) {
      status |= CNNUE_STATUS_BAD_OFFSETS;
    } else {
      for (uint32_t j = beg + lane; j < end; j += 32) {
        const uint32_t w0 = a.info[2 * j], w1 = a.info[2 * j + 1];
        const uint32_t dense = w0 & 0xfffu, moved = (w0 >> 12) & 15u, cap = (w0 >> 16) & 15u, sig = (w0 >> 20) & 63u;
        const uint32_t cf = w1 & 127u, ct = (w1 >> 7) & 127u, us = (w1 >> 14) & 15u, them = (w1 >> 18) & 15u;
        if (dense >= (uint32_t)CNNUE_AZ_DENSE_MOVES || moved >= 14u || (cap >= 14u && cap != 15u) || cf >= 90u ||
            ct >= 90u || us > 8u || them > 8u) {
          status |= CNNUE_STATUS_BAD_INDEX;
          a.logits[j] = 0.f;
          continue;
        }
        // piece-square consequence: scores[to] - scores[from] - scores[captured]
        float ps = __fsub_rn(__ldg(a.ps + moved * 90 + ct), __ldg(a.ps + moved * 90 + cf));
        ps = __fsub_rn(ps, cap < 14u ? __ldg(a.ps + cap * 90 + ct) : 0.f);
        // context . move_context[dense]: dot_product's scalar path (16 < 64)
        const float* mc = a.mctx + dense * 16;
        float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k) s4[k] = __fadd_rn(s4[k], __fmul_rn(ctx[warp][4 * c + k], __ldg(mc + 4 * c + k)));
        const float cdot = __fadd_rn(__fadd_rn(s4[0], s4[1]), __fadd_rn(s4[2], s4[3]));
        // quantised accumulator . move row (exact integers)
        int32_t v = 0;
        const int8_t* mrow = a.mq + dense * 32;
#pragma unroll
        for (int k = 0; k < 32; ++k) v += (int32_t)pacc[warp][k] * (int32_t)__ldg(mrow + k);
        v += __ldg(a.mdelta + dense * 14 + moved);
        if (cap < 14u) v -= __ldg(a.mcap + dense * 14 + cap);
        const float accl = __fmul_rn(__fmul_rn((float)v, a.fscale), a.mscale);
        // folded sparse table
        const int64_t main = (((int64_t)dense * 14 + moved) * 9 + us) * 9 + them;
        const int64_t capi = kSparseMain + (int64_t)dense * 15 + (cap < 14u ? cap : 14u);
        const float sparse = __fmul_rn((float)((int32_t)__ldg(a.sq + main) + (int32_t)__ldg(a.sq + capi)), a.sscale);
        float tactical = 0.f;
        if (a.tactical_active && moved < 7u) {
          const int64_t exact = ((int64_t)dense * 7 + moved) * 64 + sig;
          const int64_t factor = kTacticalExact + (int64_t)moved * 64 + sig;
          tactical = __fadd_rn(__ldg(a.tac + exact), __ldg(a.tac + factor));
        }
        float logit = __fadd_rn(__ldg(a.bias + dense), ps);
        logit = __fadd_rn(logit, cdot);
        logit = __fadd_rn(logit, accl);
        logit = __fadd_rn(logit, sparse);
        logit = __fadd_rn(logit, tactical);
        a.logits[j] = logit;
      }
    }
    __syncwarp();
  }
  status = __reduce_or_sync(kFull, status);
  if (lane == 0 && status) atomicOr(&a.hdr->status, status);
}

// Device copy of the policy-head tables (one allocation).
int upload_policy(const cnnue_az_weights& w, cnnue_az_model* m) {
  using namespace cnnue::az;
  const int64_t H = w.hidden;
  const int D = CNNUE_AZ_DENSE_MOVES;
  if (w.ps_scores.size() != (size_t)CNNUE_AZ_INPUT || w.q8[1].size() != (size_t)D * 32 ||
      w.q8[2].size() != (size_t)2396815 || w.q32[0].size() != (size_t)D * 14 || w.q32[1].size() != (size_t)D * 14)
    return set_error(CNNUE_ERR_INVALID_ARG, "weights have no quantised policy tables (run cnnue_az_quantize)");
  struct Part {
    const void* src;
    size_t bytes;
    void** dst;
  };
  Part parts[] = {
      {w.ps_scores.data(), w.ps_scores.size() * 4, (void**)&m->ps_scores},
      {w.t[13].data(), w.t[13].size() * 4, (void**)&m->move_bias},
      {w.t[16].data(), w.t[16].size() * 4, (void**)&m->move_context},
      {w.t[15].data(), w.t[15].size() * 4, (void**)&m->context_hidden},
      {w.t[12].data(), w.t[12].size() * 4, (void**)&m->threat_context},
      {w.q8[1].data(), w.q8[1].size(), (void**)&m->move_q},
      {w.q32[0].data(), w.q32[0].size() * 4, (void**)&m->moved_delta},
      {w.q32[1].data(), w.q32[1].size() * 4, (void**)&m->capture},
      {w.q8[2].data(), w.q8[2].size(), (void**)&m->sparse_q},
      {w.t[21].data(), w.t[21].size() * 4, (void**)&m->tactical},
  };
  if (w.t[15].size() != (size_t)16 * H) return set_error(CNNUE_ERR_INVALID_ARG, "policy_context_hidden size");
  size_t total = 0;
  for (const Part& p : parts) total += align_up(p.bytes, 256);
  cudaError_t e = cudaMalloc(&m->policy_blob, total);
  if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(az policy tables)");
  char* p = (char*)m->policy_blob;
  for (const Part& part : parts) {
    *part.dst = p;
    if ((e = cudaMemcpy(p, part.src, part.bytes, cudaMemcpyHostToDevice)) != cudaSuccess)
      return cuda_error(e, "az policy table upload");
    p += align_up(part.bytes, 256);
  }
  m->feature_scale = w.scale[0];
  m->move_scale = w.scale[1];
  m->sparse_scale = w.scale[2];
  m->threat_active = w.value_threat_active;
  m->tactical_active = w.policy_tactical_active;
  return CNNUE_OK;
}

// The float4 column path needs 16-byte aligned accumulator rows.
int check_rows_aligned(int64_t H, const void* a, const char* what) {
  if (H % 4 == 0 && ((uintptr_t)a & 15u) != 0)
    return set_error(CNNUE_ERR_INVALID_ARG, "%s must be 16-byte aligned when hidden %% 4 == 0", what);
  return CNNUE_OK;
}

}  // namespace
}  // namespace cnnue

using namespace cnnue;

extern "C" {

size_t cnnue_az_workspace_bytes(void) { return sizeof(WorkspaceHeader); }

int cnnue_az_model_create(const cnnue_az_weights* w, int device, cnnue_az_model** out) {
  if (!w || !out) return set_error(CNNUE_ERR_INVALID_ARG, "null weights or out");
  *out = nullptr;
  const int64_t H = w->hidden;
  if (H <= 0 || H > CNNUE_AZ_MAX_HIDDEN || (H >= 128 && H % 4 != 0))
    return set_error(CNNUE_ERR_INVALID_ARG, "hidden %lld: the device model takes 1..127 or multiples of 4 up to %d",
                     (long long)H, CNNUE_AZ_MAX_HIDDEN);
  if (value_smem_bytes(H, value_warps(H)) > kMaxSmem)
    return set_error(CNNUE_ERR_INVALID_ARG, "hidden %lld: value head does not fit in shared memory", (long long)H);
  DeviceGuard guard(device);
  if (guard.status) return guard.status;
  const size_t trunk = align_up(sizeof(float) * kRows * H, 256), vecH = align_up(sizeof(float) * H, 256),
               rule = align_up(sizeof(float) * 7 * H, 256), head = align_up(sizeof(float) * kHead * H, 256),
               small = align_up(sizeof(float) * kHead, 256), out3 = align_up(sizeof(float) * 3 * kHead, 256);
  const size_t staging = align_up(sizeof(float) * kHead * H, 256);
  const size_t policy = align_up((size_t)CNNUE_AZ_POLICY_ROWS * CNNUE_AZ_POLICY_RANK, 256);
  const size_t threat = align_up((size_t)CNNUE_AZ_THREAT_VOCAB * CNNUE_AZ_THREAT_RANK, 256);
  const size_t threat_out = align_up(sizeof(float) * 3 * 2 * CNNUE_AZ_THREAT_RANK, 256);
  if (w->q8[3].size() != (size_t)CNNUE_AZ_THREAT_VOCAB * CNNUE_AZ_THREAT_RANK)
    return set_error(CNNUE_ERR_INVALID_ARG, "weights have no quantised threat table (run cnnue_az_quantize)");
  if (w->q8[0].size() != (size_t)CNNUE_AZ_POLICY_ROWS * CNNUE_AZ_POLICY_RANK)
    return set_error(CNNUE_ERR_INVALID_ARG, "weights have no quantised policy table (run cnnue_az_quantize)");
  auto* m = new (std::nothrow) cnnue_az_model;
  if (!m) return set_error(CNNUE_ERR_INVALID_ARG, "out of host memory");
  m->device = device;
  m->hidden = H;
  cudaError_t e =
      cudaMalloc(&m->blob, trunk + vecH + rule + head + small + out3 + policy + threat + threat_out + staging);
  if (e != cudaSuccess) {
    delete m;
    return cuda_error(e, "cudaMalloc(az model)");
  }
  char* p = (char*)m->blob;
  m->trunk = (float*)p;
  m->bias = (float*)(p += trunk);
  m->rule = (float*)(p += vecH);
  m->head_t = (float*)(p += rule);
  m->head_b = (float*)(p += head);
  m->head_o = (float*)(p += small);
  m->policy_q = (int8_t*)(p += out3);
  m->threat_q = (int8_t*)(p += policy);
  m->threat_out = (float*)(p += threat);
  m->threat_scale = w->scale[3];
  float* stage = (float*)(p += threat_out);
  using namespace cnnue::az;
  const int tables[5] = {kInputHidden, kInputPiece, kInputRank, kInputFile, kInputKingPiece};
  const int rows[5] = {1260, 14, 10, 9, 252};
  size_t row = 0;
  int st = CNNUE_OK;
  auto copy = [&](void* dst, const std::vector<float>& src, size_t n, const char* what) {
    if (st) return;
    if (src.size() != n) {
      st = set_error(CNNUE_ERR_INVALID_ARG, "tensor %s has %zu elements, expected %zu", what, src.size(), n);
      return;
    }
    const cudaError_t ce = cudaMemcpy(dst, src.data(), n * sizeof(float), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) st = cuda_error(ce, what);
  };
  for (int t = 0; t < 5; ++t) {
    copy(m->trunk + row * H, w->t[tables[t]], (size_t)rows[t] * H, "trunk table");
    row += rows[t];
  }
  copy(m->bias, w->t[kHiddenBias], (size_t)H, "hidden_bias");
  copy(m->rule, w->t[kRuleContext], (size_t)7 * H, "rule_context_hidden");
  copy(stage, w->t[kValueHeadHidden], (size_t)kHead * H, "value_head_hidden");
  copy(m->head_b, w->t[kValueHeadBias], kHead, "value_head_bias");
  copy(m->head_o, w->t[kValueHeadOutput], 3 * kHead, "value_head_output");
  if (!st) {
    const cudaError_t ce = cudaMemcpy(m->policy_q, w->q8[0].data(), w->q8[0].size(), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) st = cuda_error(ce, "policy table");
  }
  if (!st) {
    const cudaError_t ce = cudaMemcpy(m->threat_q, w->q8[3].data(), w->q8[3].size(), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) st = cuda_error(ce, "threat table");
  }
  copy(m->threat_out, w->t[11], 3 * 2 * CNNUE_AZ_THREAT_RANK, "value_threat_output");
  if (!st) st = upload_policy(*w, m);
  if (!st) {
    const int64_t n = (int64_t)kHead * H;
    transpose_head_kernel<<<(unsigned)((n + 255) / 256), 256>>>(stage, (int)H, m->head_t);
    st = check_launch_error("transpose_head_kernel");
  }
  if (!st) {
    // The largest opt-in size, so models of different hidden sizes coexist.
    const cudaError_t ce =
        cudaFuncSetAttribute(az_value_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
    if (ce != cudaSuccess) st = cuda_error(ce, "cudaFuncSetAttribute(az_value_kernel)");
  }
  for (int k = 0; k < 2 && !st; ++k) {
    const cudaError_t ce = cudaFuncSetAttribute(k ? az_policy_kernel<true> : az_policy_kernel<false>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPolicySmem);
    if (ce != cudaSuccess) st = cuda_error(ce, "cudaFuncSetAttribute(az_policy_kernel)");
  }
  if (!st) {
    const cudaError_t ce = cudaDeviceSynchronize();
    if (ce != cudaSuccess) st = cuda_error(ce, "az model upload");
  }
  if (st) {
    cudaFree(m->blob);
    if (m->policy_blob) cudaFree(m->policy_blob);
    delete m;
    return st;
  }
  *out = m;
  return CNNUE_OK;
}

int cnnue_az_model_device(const cnnue_az_model* m) { return m ? m->device : -1; }

int cnnue_az_model_destroy(cnnue_az_model* m) {
  if (!m) return CNNUE_OK;
  DeviceGuard guard(m->device);
  if (m->policy_blob) cudaFree(m->policy_blob);
  if (m->blob) cudaFree(m->blob);
  delete m;
  return guard.status;
}

int cnnue_az_refresh(const cnnue_az_model* m, const uint32_t* d_items, uint32_t n_items, const uint32_t* d_offsets,
                     int64_t n_lists, float* d_acc, void* ws, size_t ws_bytes, void* stream) {
  if (!m || !ws || (n_lists > 0 && (!d_offsets || !d_acc || (n_items > 0 && !d_items))) || n_lists < 0)
    return set_error(CNNUE_ERR_INVALID_ARG, "null model, workspace, offsets, items or acc, or n_lists < 0");
  if (ws_bytes < sizeof(WorkspaceHeader))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu bytes < %zu", ws_bytes, sizeof(WorkspaceHeader));
  if (int st = check_rows_aligned(m->hidden, d_acc, "d_acc")) return st;
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  CNNUE_CUDA_TRY(cudaMemsetAsync(ws, 0, sizeof(WorkspaceHeader), s));
  if (n_lists == 0) return CNNUE_OK;
  ListArgs a{};
  a.trunk = m->trunk;
  a.bias = m->bias;
  a.H = (int)m->hidden;
  a.items = d_items;
  a.n_items = n_items;
  a.offsets = d_offsets;
  a.n_lists = n_lists;
  a.out = d_acc;
  a.hdr = (WorkspaceHeader*)ws;
  return launch_list<false>(a, s);
}

int cnnue_az_transition(const cnnue_az_model* m, const float* d_parent, const uint32_t* d_delta,
                        const uint8_t* d_refresh, const uint32_t* d_items, uint32_t n_items,
                        const uint32_t* d_offsets, int64_t n_lists, float* d_child, void* ws, size_t ws_bytes,
                        void* stream) {
  if (!m || !ws || n_lists < 0 || (n_lists > 0 && (!d_parent || !d_delta || !d_refresh || !d_child)) ||
      (n_items > 0 && !d_items))
    return set_error(CNNUE_ERR_INVALID_ARG, "null model, workspace, parent, delta, refresh, child or items");
  if (ws_bytes < sizeof(WorkspaceHeader))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu bytes < %zu", ws_bytes, sizeof(WorkspaceHeader));
  if (int st = check_rows_aligned(m->hidden, d_parent, "d_parent")) return st;
  if (int st = check_rows_aligned(m->hidden, d_child, "d_child")) return st;
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  CNNUE_CUDA_TRY(cudaMemsetAsync(ws, 0, sizeof(WorkspaceHeader), s));
  if (n_lists == 0) return CNNUE_OK;
  ListArgs a{};
  a.trunk = m->trunk;
  a.bias = m->bias;
  a.H = (int)m->hidden;
  a.items = d_items;
  a.n_items = n_items;
  a.offsets = d_offsets;  // NULL: a list with the refresh flag is flagged bad offsets
  a.n_lists = n_lists;
  a.parent = d_parent;
  a.delta = d_delta;
  a.refresh = d_refresh;
  a.out = d_child;
  a.hdr = (WorkspaceHeader*)ws;
  return launch_list<true>(a, s);
}

int cnnue_az_value(const cnnue_az_model* m, const float* d_acc, const uint8_t* d_side, const float* d_rule,
                   const float* d_threat, int64_t n, float* d_wdl, float* d_q, void* stream) {
  if (!m || n < 0 || (n > 0 && (!d_acc || !d_wdl || !d_q)))
    return set_error(CNNUE_ERR_INVALID_ARG, "null model, acc, wdl or q, or n < 0");
  if (n == 0) return CNNUE_OK;
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  ValueArgs a{};
  a.head_t = m->head_t;
  a.head_b = m->head_b;
  a.head_o = m->head_o;
  a.rule_rows = m->rule;
  a.H = (int)m->hidden;
  a.acc = d_acc;
  a.side = d_side;
  a.rule = d_rule;
  a.threat = d_threat;
  a.n = n;
  a.wdl = d_wdl;
  a.q = d_q;
  const int warps = value_warps(m->hidden);
  const size_t smem = value_smem_bytes(m->hidden, warps);
  const int64_t groups = (n + kValuePos - 1) / kValuePos;
  const int64_t want = (groups + warps - 1) / warps;
  int per_sm = (int)(kMaxSmem / smem);
  per_sm = per_sm < 1 ? 1 : (per_sm > 4 ? 4 : per_sm);
  const unsigned blocks = (unsigned)(want < 148 * per_sm ? want : 148 * per_sm);
  az_value_kernel<<<blocks, warps * 32, smem, (cudaStream_t)stream>>>(a);
  return check_launch_error("az_value_kernel");
}

int cnnue_az_policy_refresh(const cnnue_az_model* m, const uint32_t* d_items, uint32_t n_items,
                            const uint32_t* d_offsets, int64_t n_lists, int16_t* d_acc, void* ws, size_t ws_bytes,
                            void* stream) {
  if (!m || !ws || n_lists < 0 || (n_lists > 0 && (!d_offsets || !d_acc || (n_items > 0 && !d_items))))
    return set_error(CNNUE_ERR_INVALID_ARG, "null model, workspace, offsets, items or acc, or n_lists < 0");
  if (ws_bytes < sizeof(WorkspaceHeader))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu bytes < %zu", ws_bytes, sizeof(WorkspaceHeader));
  if ((uintptr_t)d_acc & 7u) return set_error(CNNUE_ERR_INVALID_ARG, "d_acc must be 8-byte aligned");
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  CNNUE_CUDA_TRY(cudaMemsetAsync(ws, 0, sizeof(WorkspaceHeader), s));
  if (n_lists == 0) return CNNUE_OK;
  PolicyArgs a{};
  a.q = m->policy_q;
  a.items = d_items;
  a.n_items = n_items;
  a.offsets = d_offsets;
  a.n_lists = n_lists;
  a.out = d_acc;
  a.hdr = (WorkspaceHeader*)ws;
  return launch_policy<false>(a, s);
}

int cnnue_az_policy_transition(const cnnue_az_model* m, const int16_t* d_parent, const uint32_t* d_delta,
                               const uint8_t* d_refresh, const uint32_t* d_items, uint32_t n_items,
                               const uint32_t* d_offsets, int64_t n_lists, int16_t* d_child, void* ws,
                               size_t ws_bytes, void* stream) {
  if (!m || !ws || n_lists < 0 || (n_lists > 0 && (!d_parent || !d_delta || !d_refresh || !d_child)) ||
      (n_items > 0 && !d_items))
    return set_error(CNNUE_ERR_INVALID_ARG, "null model, workspace, parent, delta, refresh, child or items");
  if (ws_bytes < sizeof(WorkspaceHeader))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu bytes < %zu", ws_bytes, sizeof(WorkspaceHeader));
  if (((uintptr_t)d_parent | (uintptr_t)d_child) & 7u)
    return set_error(CNNUE_ERR_INVALID_ARG, "d_parent and d_child must be 8-byte aligned");
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  CNNUE_CUDA_TRY(cudaMemsetAsync(ws, 0, sizeof(WorkspaceHeader), s));
  if (n_lists == 0) return CNNUE_OK;
  PolicyArgs a{};
  a.q = m->policy_q;
  a.items = d_items;
  a.n_items = n_items;
  a.offsets = d_offsets;
  a.n_lists = n_lists;
  a.parent = d_parent;
  a.delta = d_delta;
  a.refresh = d_refresh;
  a.out = d_child;
  a.hdr = (WorkspaceHeader*)ws;
  return launch_policy<true>(a, s);
}

int cnnue_az_threat_logits(const cnnue_az_model* m, const uint32_t* d_features, uint32_t n_features,
                           const uint32_t* d_offsets, int64_t n, float* d_logits, void* ws, size_t ws_bytes,
                           void* stream) {
  if (!m || !ws || n < 0 || (n > 0 && (!d_offsets || !d_logits)) || (n_features > 0 && !d_features))
    return set_error(CNNUE_ERR_INVALID_ARG, "null model, workspace, offsets, features or logits, or n < 0");
  if (ws_bytes < sizeof(WorkspaceHeader))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu bytes < %zu", ws_bytes, sizeof(WorkspaceHeader));
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  CNNUE_CUDA_TRY(cudaMemsetAsync(ws, 0, sizeof(WorkspaceHeader), s));
  if (n == 0) return CNNUE_OK;
  const int64_t want = (n + kThreatWarps - 1) / kThreatWarps;
  const unsigned blocks = (unsigned)(want < 148 * 16 ? want : 148 * 16);
  az_threat_kernel<<<blocks, kThreatWarps * 32, 0, s>>>(m->threat_q, m->threat_scale, m->threat_out, d_features,
                                                        n_features, d_offsets, n, d_logits, nullptr,
                                                        (WorkspaceHeader*)ws);
  return check_launch_error("az_threat_kernel");
}

size_t cnnue_az_evaluate_workspace_bytes(const cnnue_az_model* m, int64_t n) {
  if (!m || n < 0) return 0;
  return sizeof(WorkspaceHeader) + align_up((size_t)n * m->hidden * 4, 256) + align_up((size_t)n * 3 * 4, 256) +
         align_up((size_t)n * 2 * CNNUE_AZ_THREAT_RANK * 4, 256);
}

int cnnue_az_evaluate(const cnnue_az_model* m, const float* d_acc, const uint8_t* d_side, const float* d_rule,
                      const uint32_t* d_threat_features, uint32_t n_threat_features, const uint32_t* d_threat_offsets,
                      const int16_t* d_policy_acc, const uint32_t* d_move_info, uint32_t n_moves,
                      const uint32_t* d_move_offsets, int64_t n, float* d_wdl, float* d_q, float* d_logits, void* ws,
                      size_t ws_bytes, void* stream) {
  if (!m || !ws || n < 0 || (n > 0 && (!d_acc || !d_wdl || !d_q)))
    return set_error(CNNUE_ERR_INVALID_ARG, "null model, workspace, acc, wdl or q, or n < 0");
  if (d_move_info && (!d_move_offsets || !d_logits || !d_policy_acc))
    return set_error(CNNUE_ERR_INVALID_ARG, "moves need offsets, logits and the policy accumulators");
  if (d_threat_features && !d_threat_offsets) return set_error(CNNUE_ERR_INVALID_ARG, "threat features need offsets");
  if (ws_bytes < cnnue_az_evaluate_workspace_bytes(m, n))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu < %zu bytes", ws_bytes, cnnue_az_evaluate_workspace_bytes(m, n));
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  CNNUE_CUDA_TRY(cudaMemsetAsync(ws, 0, sizeof(WorkspaceHeader), s));
  if (n == 0) return CNNUE_OK;
  char* p = (char*)ws + sizeof(WorkspaceHeader);
  float* x = (float*)p;
  p += align_up((size_t)n * m->hidden * 4, 256);
  float* tlogits = (float*)p;
  p += align_up((size_t)n * 3 * 4, 256);
  float* tact = (float*)p;
  WorkspaceHeader* hdr = (WorkspaceHeader*)ws;
  // 1. threat branch, when the model has one (value_threat_active)
  const bool threat = d_threat_offsets != nullptr && m->threat_active;
  if (threat) {
    const int64_t want = (n + kThreatWarps - 1) / kThreatWarps;
    const unsigned blocks = (unsigned)(want < 148 * 16 ? want : 148 * 16);
    az_threat_kernel<<<blocks, kThreatWarps * 32, 0, s>>>(m->threat_q, m->threat_scale, m->threat_out,
                                                          d_threat_features, n_threat_features, d_threat_offsets, n,
                                                          tlogits, tact, hdr);
    if (int st = check_launch_error("az_threat_kernel")) return st;
  }
  // 2. value head, keeping the normalised hidden for the policy head
  {
    ValueArgs a{};
    a.head_t = m->head_t;
    a.head_b = m->head_b;
    a.head_o = m->head_o;
    a.rule_rows = m->rule;
    a.H = (int)m->hidden;
    a.acc = d_acc;
    a.side = d_side;
    a.rule = d_rule;
    a.threat = threat ? tlogits : nullptr;
    a.n = n;
    a.wdl = d_wdl;
    a.q = d_q;
    a.x_out = x;
    const int warps = value_warps(m->hidden);
    const size_t smem = value_smem_bytes(m->hidden, warps);
    const int64_t groups = (n + kValuePos - 1) / kValuePos;
    const int64_t want = (groups + warps - 1) / warps;
    int per_sm = (int)(kMaxSmem / smem);
    per_sm = per_sm < 1 ? 1 : (per_sm > 4 ? 4 : per_sm);
    const unsigned blocks = (unsigned)(want < 148 * per_sm ? want : 148 * per_sm);
    az_value_kernel<<<blocks, warps * 32, smem, s>>>(a);
    if (int st = check_launch_error("az_value_kernel")) return st;
  }
  // 3. policy logits of the listed moves
  if (d_move_info) {
    PolicyLogitArgs a{};
    a.x = x;
    a.threat_act = threat ? tact : nullptr;
    a.pacc = d_policy_acc;
    a.side = d_side;
    a.info = d_move_info;
    a.n_moves = n_moves;
    a.offsets = d_move_offsets;
    a.n = n;
    a.H = (int)m->hidden;
    a.logits = d_logits;
    a.hdr = hdr;
    a.ps = m->ps_scores;
    a.bias = m->move_bias;
    a.mctx = m->move_context;
    a.pch = m->context_hidden;
    a.ptc = m->threat_context;
    a.mq = m->move_q;
    a.mdelta = m->moved_delta;
    a.mcap = m->capture;
    a.sq = m->sparse_q;
    a.tac = m->tactical;
    a.fscale = m->feature_scale;
    a.mscale = m->move_scale;
    a.sscale = m->sparse_scale;
    a.tactical_active = m->tactical_active;
    const int64_t want = (n + kPolicyLogitWarps - 1) / kPolicyLogitWarps;
    const unsigned blocks = (unsigned)(want < 148 * 16 ? want : 148 * 16);
    az_policy_logits_kernel<<<blocks, kPolicyLogitWarps * 32, 0, s>>>(a);
    if (int st = check_launch_error("az_policy_logits_kernel")) return st;
  }
  return CNNUE_OK;
}

}  // extern "C"
