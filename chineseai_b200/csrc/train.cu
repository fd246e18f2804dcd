// train.cu - one data-parallel training step of the HalfKA network (the
// fp32-master / bf16-activation form of the quantised evaluator) on sm_100a.
//
// Per rank and step:
//   1. bucket sort of the positions (shared with the evaluators);
//   2. t_gather_kernel: FT gather from the bf16 shadow of the FT weights,
//      fp32 sums in index order from the bias, activation a stored as bf16
//      [n][2][1024] (128 threads per position, 16-byte row loads);
//   3. t_head_kernel: per position (bucket order, 128 threads): pairwise pack
//      x = bf16(clamp(a_j) clamp(a_j+512)), stack 1024->16->32->1 in fp32,
//      loss (sigmoid(s/400) - t)^2 and the whole backward of the head: the
//      per-position head vectors (h1, dh1, h2, dh2, ds) and da [n][2][1024]
//      fp32 (the FT output gradient, through pack and clamp);
//   4. t_w1grad_kernel / t_smallgrad_kernel: bucketed stack gradients
//      (per bucket, positions summed in bucket order - deterministic);
//   5. the FT gradient by the segmented reduction of segreduce.cuh: every
//      entry of an active list contributes its list's da row to its feature's
//      gradient row, and every list contributes to row 11340 (the FT bias),
//      so one pass yields [11340 + 1][1024] = the FT weight and bias
//      gradients, without atomics;
//   6. the loss mean (one CTA).
// The gradient all-reduce across ranks happens on the host (NCCL) and
// cnnue_t_adam applies Adam to the flat parameters and refreshes the shadow.
#include <algorithm>

#include <cuda_bf16.h>

#include "common.cuh"
#include "segreduce.cuh"

namespace cnnue {
namespace tr {

constexpr int kF = CNNUE_T_FEATURES;
constexpr int kCols = 1024;
constexpr int kNB = 16;
constexpr unsigned kFull = 0xffffffffu;

// Flat parameter layout (fp32), see cnnue.h.
constexpr int64_t kOffFt = 0;
constexpr int64_t kOffFtBias = (int64_t)kF * kCols;
constexpr int64_t kOffW1 = kOffFtBias + kCols;
constexpr int64_t kOffB1 = kOffW1 + kNB * 16 * kCols;
constexpr int64_t kOffW2 = kOffB1 + kNB * 16;
constexpr int64_t kOffB2 = kOffW2 + kNB * 32 * 16;
constexpr int64_t kOffW3 = kOffB2 + kNB * 32;
constexpr int64_t kOffB3 = kOffW3 + kNB * 32;
constexpr int64_t kParams = kOffB3 + kNB;
static_assert(kParams == CNNUE_T_PARAMS, "parameter count");
static_assert(kOffW1 == CNNUE_T_SHADOW, "shadow covers the FT weights and bias");

// Per-position head record: h1[16] dh1[16] h2[32] dh2[32] ds (padded to 128)
constexpr int kHead = 128;
constexpr int kHH1 = 0, kHDH1 = 16, kHH2 = 32, kHDH2 = 64, kHDS = 96;

struct Ws {
  WorkspaceView sort;  // bucket sort (header = status word)
  __nv_bfloat16* a;    // [n][2][1024]
  float* da;           // [2n][1024]
  float* head;         // [n][kHead] per-position head vectors
  float* loss;         // [n]
  uint32_t* list_of;   // [n_idx] list id of each index entry
  void* seg;           // segmented-reduction workspace
};

inline size_t seg_bytes(int64_t n, uint32_t n_idx) {
  return seg::bwd_bytes((int64_t)n_idx + 2 * n, 1, kF + 1, kCols);
}

inline size_t ws_bytes(int64_t n, uint32_t n_idx) {
  size_t b = align_up(bucket_workspace_bytes(n), 256);
  b += align_up((size_t)n * 2 * kCols * 2, 256);
  b += align_up((size_t)n * 2 * kCols * 4, 256);
  b += align_up((size_t)n * kHead * 4, 256);
  b += align_up((size_t)n * 4, 256);
  b += align_up((size_t)std::max<uint32_t>(n_idx, 1) * 4, 256);
  b += align_up(seg_bytes(n, n_idx), 256);
  return b;
}

inline Ws carve(void* ws, int64_t n, uint32_t n_idx) {
  Ws w;
  char* p = (char*)ws;
  w.sort = carve_workspace(p, n);
  p += align_up(bucket_workspace_bytes(n), 256);
  w.a = (__nv_bfloat16*)p;
  p += align_up((size_t)n * 2 * kCols * 2, 256);
  w.da = (float*)p;
  p += align_up((size_t)n * 2 * kCols * 4, 256);
  w.head = (float*)p;
  p += align_up((size_t)n * kHead * 4, 256);
  w.loss = (float*)p;
  p += align_up((size_t)n * 4, 256);
  w.list_of = (uint32_t*)p;
  p += align_up((size_t)std::max<uint32_t>(n_idx, 1) * 4, 256);
  w.seg = p;
  return w;
}

__device__ __forceinline__ float clamp01(float v) { return fminf(fmaxf(v, 0.f), 1.f); }
__device__ __forceinline__ float dclamp01(float z) { return (z > 0.f && z < 1.f) ? 1.f : 0.f; }

__device__ __forceinline__ void unpack8(const uint4& v, float f[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float f[8]) {
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

// ---------------------------------------------------------------------------
// 2. FT gather: 128 threads per position; thread (p, c) owns columns
//    [8c, 8c+8) and [512+8c, 512+8c+8) of perspective p.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) t_gather_kernel(const __nv_bfloat16* __restrict__ shadow,
                                                       const uint16_t* __restrict__ idx,
                                                       uint32_t n_idx,
                                                       const uint32_t* __restrict__ offsets,
                                                       int64_t n, __nv_bfloat16* __restrict__ a,
                                                       uint32_t* status) {
  const int g = threadIdx.x >> 7, t = threadIdx.x & 127, lane = t & 31;
  const int persp = t >> 6, c = t & 63;
  const int64_t groups = (int64_t)gridDim.x * 2;
  const char* base = (const char*)shadow + c * 16;
  const char* bias = (const char*)(shadow + (int64_t)kF * kCols) + c * 16;
  float blo[8], bhi[8];
  unpack8(__ldg((const uint4*)bias), blo);
  unpack8(__ldg((const uint4*)(bias + kCols)), bhi);
  for (int64_t pos = (int64_t)blockIdx.x * 2 + g; pos < n; pos += groups) {
    const int64_t ps = 2 * pos + persp;
    const uint32_t ob = min(offsets[ps], n_idx);
    const uint32_t oe = min(max(offsets[ps + 1], ob), n_idx);
    float lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      lo[i] = blo[i];
      hi[i] = bhi[i];
    }
    for (uint32_t b0 = ob; b0 < oe; b0 += 32) {
      const int cnt = (int)min(32u, oe - b0);
      uint32_t my = lane < cnt ? (uint32_t)idx[b0 + lane] : 0u;
      const bool bad = lane < cnt && my >= (uint32_t)kF;
      if (__any_sync(kFull, bad) && bad) atomicOr(status, CNNUE_STATUS_BAD_INDEX);
      if (bad) my = kF;  // marks the entry to skip below
      for (int r0 = 0; r0 < cnt; r0 += 4) {
        uint4 vl[4], vh[4];
        bool ok[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t f = __shfl_sync(kFull, my, (r0 + u) & 31);
          ok[u] = r0 + u < cnt && f < (uint32_t)kF;
          if (ok[u]) {
            const char* row = base + (size_t)f * kCols * 2;
            vl[u] = ldg_stream16(row);
            vh[u] = ldg_stream16(row + kCols);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (!ok[u]) continue;
          float fl[8], fh[8];
          unpack8(vl[u], fl);
          unpack8(vh[u], fh);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            lo[i] += fl[i];
            hi[i] += fh[i];
          }
        }
      }
    }
    char* out = (char*)(a + ps * kCols) + c * 16;
    *(uint4*)out = pack8(lo);
    *(uint4*)(out + kCols) = pack8(hi);
  }
}

// ---------------------------------------------------------------------------
// 3. Head forward + backward, 128 threads per position in bucket order.
//    Thread t owns x[8t, 8t+8): perspective p = t >> 6, pair columns
//    j = 8(t&63) .. +8 and j + 512 of a_p.
// ---------------------------------------------------------------------------
struct HeadArgs {
  const float* params;
  const __nv_bfloat16* a;
  const float* target;
  const uint32_t* perm;
  const uint8_t* sorted_bucket;
  int64_t n;
  float inv_n;
  float* da;
  float* head;
  float* loss;
};

__global__ void __launch_bounds__(128) t_head_kernel(const HeadArgs A) {
  __shared__ float red[4][16];
  __shared__ float h1s[16], dh1s[16];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int persp = t >> 6, c = t & 63;
  const float* W1 = A.params + kOffW1;
  const float* B1 = A.params + kOffB1;
  const float* W2 = A.params + kOffW2;
  const float* B2 = A.params + kOffB2;
  const float* W3 = A.params + kOffW3;
  const float* B3 = A.params + kOffB3;
  for (int64_t i = blockIdx.x; i < A.n; i += gridDim.x) {
    const uint32_t pos = A.perm[i];
    const int bk = A.sorted_bucket[i];
    const char* ap = (const char*)(A.a + (2 * (int64_t)pos + persp) * kCols) + c * 16;
    float alo[8], ahi[8], x[8];
    unpack8(*(const uint4*)ap, alo);
    unpack8(*(const uint4*)(ap + kCols), ahi);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      x[q] = __bfloat162float(__float2bfloat16_rn(clamp01(alo[q]) * clamp01(ahi[q])));
    const float* w1p = W1 + (size_t)bk * 16 * kCols + 8 * t;
    float v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float4 wa = __ldg((const float4*)(w1p + (size_t)k * kCols));
      const float4 wb = __ldg((const float4*)(w1p + (size_t)k * kCols + 4));
      v[k] = wa.x * x[0] + wa.y * x[1] + wa.z * x[2] + wa.w * x[3] + wb.x * x[4] + wb.y * x[5] +
             wb.z * x[6] + wb.w * x[7];
    }
    // reduce-scatter: lane l ends with the warp total of output l >> 1
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const bool up = lane & 16;
      const float send = up ? v[j] : v[j + 8];
      const float keep = up ? v[j + 8] : v[j];
      v[j] = keep + __shfl_xor_sync(kFull, send, 16);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool up = lane & 8;
      const float send = up ? v[j] : v[j + 4];
      const float keep = up ? v[j + 4] : v[j];
      v[j] = keep + __shfl_xor_sync(kFull, send, 8);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const bool up = lane & 4;
      const float send = up ? v[j] : v[j + 2];
      const float keep = up ? v[j + 2] : v[j];
      v[j] = keep + __shfl_xor_sync(kFull, send, 4);
    }
    {
      const bool up = lane & 2;
      const float send = up ? v[0] : v[1];
      const float keep = up ? v[1] : v[0];
      v[0] = keep + __shfl_xor_sync(kFull, send, 2);
    }
    v[0] += __shfl_xor_sync(kFull, v[0], 1);
    if ((lane & 1) == 0) red[warp][lane >> 1] = v[0];
    __syncthreads();
    if (warp == 0) {
      float z1 = 0.f, h1 = 0.f;
      if (lane < 16) {
        z1 = B1[bk * 16 + lane] + red[0][lane] + red[1][lane] + red[2][lane] + red[3][lane];
        h1 = clamp01(z1);
        h1s[lane] = h1;
      }
      __syncwarp();
      float z2 = B2[bk * 32 + lane];
#pragma unroll
      for (int k = 0; k < 16; ++k) z2 += W2[(bk * 32 + lane) * 16 + k] * h1s[k];
      const float h2 = clamp01(z2);
      float s = W3[bk * 32 + lane] * h2;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
      s += B3[bk];
      const float sg = 1.f / (1.f + __expf(-s / 400.f));
      const float d = sg - A.target[pos];
      const float ds = 2.f * d * sg * (1.f - sg) / 400.f * A.inv_n;
      const float dh2 = ds * W3[bk * 32 + lane] * dclamp01(z2);
      float dh1 = 0.f;
#pragma unroll
      for (int m = 0; m < 32; ++m) {
        const float dm = __shfl_sync(kFull, dh2, m);
        if (lane < 16) dh1 += W2[(bk * 32 + m) * 16 + lane] * dm;
      }
      float* hrec = A.head + (size_t)pos * kHead;
      if (lane < 16) {
        dh1 *= dclamp01(z1);
        dh1s[lane] = dh1;
        hrec[kHH1 + lane] = h1;
        hrec[kHDH1 + lane] = dh1;
      }
      hrec[kHH2 + lane] = h2;
      hrec[kHDH2 + lane] = dh2;
      if (lane == 0) {
        hrec[kHDS] = ds;
        A.loss[pos] = d * d;
      }
    }
    __syncthreads();
    // dx for this thread's 8 inputs, then da through the pack and the clamps
    float dx[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) dx[q] = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float4 wa = __ldg((const float4*)(w1p + (size_t)k * kCols));
      const float4 wb = __ldg((const float4*)(w1p + (size_t)k * kCols + 4));
      const float gk = dh1s[k];
      dx[0] += wa.x * gk;
      dx[1] += wa.y * gk;
      dx[2] += wa.z * gk;
      dx[3] += wa.w * gk;
      dx[4] += wb.x * gk;
      dx[5] += wb.y * gk;
      dx[6] += wb.z * gk;
      dx[7] += wb.w * gk;
    }
    float dlo[8], dhi[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      dlo[q] = dx[q] * clamp01(ahi[q]) * dclamp01(alo[q]);
      dhi[q] = dx[q] * clamp01(alo[q]) * dclamp01(ahi[q]);
    }
    float* dp = A.da + (2 * (int64_t)pos + persp) * kCols + 8 * c;
    *(float4*)dp = make_float4(dlo[0], dlo[1], dlo[2], dlo[3]);
    *(float4*)(dp + 4) = make_float4(dlo[4], dlo[5], dlo[6], dlo[7]);
    *(float4*)(dp + 512) = make_float4(dhi[0], dhi[1], dhi[2], dhi[3]);
    *(float4*)(dp + 516) = make_float4(dhi[4], dhi[5], dhi[6], dhi[7]);
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// 4a. dW1[b][k][i] = sum over positions of bucket b (bucket order) of
//     dh1[k] x[i]; one CTA per (bucket, 128-column tile), thread = column.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) t_w1grad_kernel(const __nv_bfloat16* __restrict__ a,
                                                       const float* __restrict__ head,
                                                       const uint32_t* __restrict__ perm,
                                                       const WorkspaceHeader* hdr, float* grads) {
  const int bk = blockIdx.y;
  const int i = blockIdx.x * 128 + threadIdx.x;  // x index 0..1023
  const int persp = i >> 9, j = i & 511;
  uint32_t start = 0;
  for (int b = 0; b < bk; ++b) start += hdr->counts[b];
  const uint32_t cnt = hdr->counts[bk];
  __shared__ float dh1s[32][16];
  float acc[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) acc[k] = 0.f;
  __shared__ uint32_t poss[32];
  for (uint32_t c0 = 0; c0 < cnt; c0 += 32) {
    const uint32_t m = min(32u, cnt - c0);
    __syncthreads();
    if (threadIdx.x < m) poss[threadIdx.x] = perm[start + c0 + threadIdx.x];
    for (uint32_t e = threadIdx.x; e < m * 16; e += 128) {
      const uint32_t pos = perm[start + c0 + e / 16];
      dh1s[e / 16][e % 16] = head[(size_t)pos * kHead + kHDH1 + e % 16];
    }
    __syncthreads();
    // all 2 x m activation loads of this thread are independent: issue them first
    __nv_bfloat16 lo[32], hi[32];
#pragma unroll
    for (uint32_t q = 0; q < 32; ++q) {
      if (q < m) {
        const __nv_bfloat16* ap = a + (2 * (int64_t)poss[q] + persp) * kCols;
        lo[q] = ap[j];
        hi[q] = ap[j + 512];
      }
    }
#pragma unroll
    for (uint32_t q = 0; q < 32; ++q) {
      if (q < m) {
        const float x = __bfloat162float(__float2bfloat16_rn(clamp01(__bfloat162float(lo[q])) *
                                                             clamp01(__bfloat162float(hi[q]))));
#pragma unroll
        for (int k = 0; k < 16; ++k) acc[k] += dh1s[q][k] * x;
      }
    }
  }
  float* g = grads + kOffW1 + (size_t)bk * 16 * kCols + i;
#pragma unroll
  for (int k = 0; k < 16; ++k) g[(size_t)k * kCols] = acc[k];
}

// 4b. dW2, dW3, db1, db2, db3: one CTA per bucket, 512 threads; the head
//     records of 64 positions at a time are staged in shared memory with
//     coalesced loads, then summed in bucket order.
__global__ void __launch_bounds__(512) t_smallgrad_kernel(const float* __restrict__ head,
                                                          const uint32_t* __restrict__ perm,
                                                          const WorkspaceHeader* hdr, float* grads) {
  constexpr int kChunk = 64;
  constexpr int kRec = 97;  // h1, dh1, h2, dh2, ds
  __shared__ float rec[kChunk][kRec];
  const int bk = blockIdx.x, t = threadIdx.x;
  uint32_t start = 0;
  for (int b = 0; b < bk; ++b) start += hdr->counts[b];
  const uint32_t cnt = hdr->counts[bk];
  const int m = t >> 4, k = t & 15;  // dW2[m][k]
  float w2 = 0.f, w3 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
  for (uint32_t c0 = 0; c0 < cnt; c0 += kChunk) {
    const uint32_t nq = min((uint32_t)kChunk, cnt - c0);
    __syncthreads();
    for (uint32_t e = t; e < nq * kRec; e += 512) {
      const uint32_t q = e / kRec, f = e % kRec;
      rec[q][f] = head[(size_t)perm[start + c0 + q] * kHead + f];
    }
    __syncthreads();
    for (uint32_t q = 0; q < nq; ++q) {
      const float* h = rec[q];
      w2 += h[kHDH2 + m] * h[kHH1 + k];
      if (t < 32) {
        w3 += h[kHDS] * h[kHH2 + t];
        b2 += h[kHDH2 + t];
      }
      if (t < 16) b1 += h[kHDH1 + t];
      if (t == 0) b3 += h[kHDS];
    }
  }
  grads[kOffW2 + (size_t)bk * 512 + t] = w2;
  if (t < 32) {
    grads[kOffW3 + bk * 32 + t] = w3;
    grads[kOffB2 + bk * 32 + t] = b2;
  }
  if (t < 16) grads[kOffB1 + bk * 16 + t] = b1;
  if (t == 0) grads[kOffB3 + bk] = b3;
}

// list id of every index entry
__global__ void t_list_of_kernel(const uint32_t* __restrict__ offsets, uint32_t n_idx,
                                 int64_t n_lists, uint32_t* __restrict__ list_of) {
  const int64_t l = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (l >= n_lists) return;
  const uint32_t b = min(offsets[l], n_idx), e = min(max(offsets[l + 1], b), n_idx);
  for (uint32_t i = b; i < e; ++i) list_of[i] = (uint32_t)l;
}

// Contributions of the FT backward: index entry e (< n_idx) adds list
// list_of[e]'s da row to row idx[e]; entry n_idx + l adds list l's da row to
// row kF (the bias).
struct FtDecoder {
  static constexpr int kSlots = 1;
  int64_t n_rows;  // kF + 1
  const uint16_t* idx;
  const uint32_t* list_of;
  uint32_t n_idx;
  __device__ __forceinline__ uint32_t src(int64_t e) const {
    return e < (int64_t)n_idx ? list_of[e] : (uint32_t)(e - n_idx);
  }
  __device__ __forceinline__ int decode(int64_t e, uint32_t rows[1]) const {
    if (e >= (int64_t)n_idx) {
      rows[0] = kF;
      return 1;
    }
    const uint32_t f = idx[e];
    rows[0] = f;
    return f < (uint32_t)kF ? 1 : -1;
  }
};

// 6. mean loss (one CTA, fixed order)
__global__ void t_loss_kernel(const float* __restrict__ loss, int64_t n, float* out) {
  __shared__ float part[32];
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += loss[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += part[w];
    *out = tot / (float)n;
  }
}

// Adam over the flat parameters; the first `shadow_count` parameters also
// refresh their bf16 shadow.
__global__ void t_adam_kernel(float* __restrict__ w, float* __restrict__ m, float* __restrict__ v,
                              const float* __restrict__ g, int64_t count, __nv_bfloat16* shadow,
                              int64_t shadow_count, float grad_scale, float lr, float beta1,
                              float beta2, float eps, float c1, float c2) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride) {
    const float gi = g[i] * grad_scale;
    const float mi = beta1 * m[i] + (1.f - beta1) * gi;
    const float vi = beta2 * v[i] + (1.f - beta2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    const float wi = w[i] - lr * (mi / c1) / (sqrtf(vi / c2) + eps);
    w[i] = wi;
    if (i < shadow_count) shadow[i] = __float2bfloat16_rn(wi);
  }
}

__global__ void t_shadow_kernel(const float* __restrict__ w, int64_t count, __nv_bfloat16* shadow) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride)
    shadow[i] = __float2bfloat16_rn(w[i]);
}

}  // namespace tr
}  // namespace cnnue

using namespace cnnue;
using namespace cnnue::tr;

extern "C" {

size_t cnnue_t_param_count(void) { return (size_t)kParams; }

size_t cnnue_t_workspace_bytes(int64_t n_positions, uint32_t n_indices) {
  if (n_positions <= 0) return 0;
  return ws_bytes(n_positions, n_indices);
}

int cnnue_t_make_shadow(const float* d_params, uint16_t* d_shadow, void* stream) {
  if (!d_params || !d_shadow) return set_error(CNNUE_ERR_INVALID_ARG, "null buffer");
  t_shadow_kernel<<<1184, 256, 0, (cudaStream_t)stream>>>(d_params, kOffW1, (__nv_bfloat16*)d_shadow);
  return check_launch_error("t_shadow_kernel");
}

int cnnue_t_forward_backward(const float* d_params, const uint16_t* d_shadow,
                             const uint16_t* d_indices, uint32_t n_indices,
                             const uint32_t* d_offsets, int64_t n, const float* d_target,
                             float* d_grads, float* d_loss, void* d_ws, size_t ws_size,
                             void* stream) {
  if (n <= 0 || n > (int64_t)INT32_MAX) return set_error(CNNUE_ERR_INVALID_ARG, "bad n_positions");
  if (!d_params || !d_shadow || !d_offsets || !d_target || !d_grads || !d_loss || !d_ws ||
      (n_indices && !d_indices))
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer");
  if (((uintptr_t)d_params | (uintptr_t)d_shadow | (uintptr_t)d_grads) & 15u)
    return set_error(CNNUE_ERR_INVALID_ARG, "params, shadow and grads must be 16-byte aligned");
  if (ws_size < ws_bytes(n, n_indices))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu < %zu", ws_size, ws_bytes(n, n_indices));
  cudaStream_t s = (cudaStream_t)stream;
  Ws w = carve(d_ws, n, n_indices);
  int st = launch_bucket_sort(d_offsets, n_indices, nullptr, n, 1, kNB, d_ws, s);
  if (st) return st;
  uint32_t* status = &w.sort.hdr->status;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  t_gather_kernel<<<sms * 4, 256, 0, s>>>((const __nv_bfloat16*)d_shadow, d_indices, n_indices,
                                          d_offsets, n, w.a, status);
  if ((st = check_launch_error("t_gather_kernel"))) return st;
  HeadArgs h{d_params, w.a, d_target, w.sort.perm, w.sort.sorted_bucket, n, 1.f / (float)n,
             w.da, w.head, w.loss};
  t_head_kernel<<<(unsigned)std::min<int64_t>(n, (int64_t)sms * 16), 128, 0, s>>>(h);
  if ((st = check_launch_error("t_head_kernel"))) return st;
  t_w1grad_kernel<<<dim3(8, kNB), 128, 0, s>>>(w.a, w.head, w.sort.perm, w.sort.hdr, d_grads);
  if ((st = check_launch_error("t_w1grad_kernel"))) return st;
  t_smallgrad_kernel<<<kNB, 512, 0, s>>>(w.head, w.sort.perm, w.sort.hdr, d_grads);
  if ((st = check_launch_error("t_smallgrad_kernel"))) return st;
  t_list_of_kernel<<<(unsigned)((2 * n + 255) / 256), 256, 0, s>>>(d_offsets, n_indices, 2 * n,
                                                                  w.list_of);
  if ((st = check_launch_error("t_list_of_kernel"))) return st;
  FtDecoder dec{kF + 1, d_indices, w.list_of, n_indices};
  st = seg::launch_bwd((int64_t)n_indices + 2 * n, w.da, kCols, dec, d_grads + kOffFt, w.seg, s);
  if (st) return st;
  t_loss_kernel<<<1, 1024, 0, s>>>(w.loss, n, d_loss);
  return check_launch_error("t_loss_kernel");
}

int cnnue_t_adam(float* d_params, float* d_m, float* d_v, const float* d_grads, uint16_t* d_shadow,
                 float grad_scale, float lr, float beta1, float beta2, float eps, int step,
                 void* stream) {
  if (!d_params || !d_m || !d_v || !d_grads || !d_shadow)
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer");
  if (step < 1) return set_error(CNNUE_ERR_INVALID_ARG, "step must be >= 1");
  const float c1 = 1.f - powf(beta1, (float)step);
  const float c2 = 1.f - powf(beta2, (float)step);
  t_adam_kernel<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(d_params, d_m, d_v, d_grads, kParams,
                                                            (__nv_bfloat16*)d_shadow, kOffW1,
                                                            grad_scale, lr, beta1, beta2, eps, c1, c2);
  return check_launch_error("t_adam_kernel");
}

}  // extern "C"
