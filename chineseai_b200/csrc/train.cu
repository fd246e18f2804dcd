// train.cu - one data-parallel training step of the HalfKA network (the
// fp32-master / bf16-activation form of the quantised evaluator) on sm_100a.
//
// Per rank and step:
//   1. bucket sort of the positions (shared with the evaluators);
//   2. t_gather_kernel: FT gather from the bf16 shadow of the FT weights,
//      fp32 sums in index order from the bias, activation a stored as bf16
//      [n][2][1024] (128 threads per position, 16-byte row loads);
//   3. the head over bucket tiles (128 positions of one bucket in sorted
//      order): t_head_tc_kernel forms the pairwise pack x = bf16(clamp(a_j)
//      clamp(a_j+512)) into shared memory and computes L1 = x . W1^T on the
//      tensor cores (tcgen05 kind::f16, W1 as bf16 hi + lo halves, fp32
//      accumulator in TMEM), then per position the rest of the stack, the
//      loss and its backward to dh1, and per tile the partial gradients of
//      W2, W3 and the biases; t_dx_kernel forms dx = dh1 . W1 and da [n][2]
//      [1024] fp32 (the FT output gradient, through pack and clamp);
//      t_w1part_kernel the tile's partial dW1 = dh1^T x;
//   4. ordered per-bucket sums of the tile partials (deterministic);
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

#include <mutex>

#include "common.cuh"
#include "pipeline.cuh"
#include "segreduce.cuh"
#include "tcgen05.cuh"

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

// Per-position head record staged by the head kernel: h1[16] dh1[16] h2[32]
// dh2[32] ds
constexpr int kRec = 97;
constexpr int kHH1 = 0, kHDH1 = 16, kHH2 = 32, kHDH2 = 64, kHDS = 96;

// Head tiles: 128 sorted positions of one bucket.
constexpr int kTile = 128;
constexpr int kSmallPart = 608;
constexpr int kRowSplit = 4;     // the SIMT tile kernels split a tile's rows over this many CTAs  // per tile: dW2 512, dW3 32, db2 32, db1 16, db3 1 (padded)
inline int64_t max_tiles(int64_t n) { return (n + kTile - 1) / kTile + kNB; }
// W1 as the tensor-core B operand: per bucket and 64-column K chunk, the
// bf16 hi and lo halves of its 16 rows (128B-swizzled K-major, 2 KB each).
constexpr int kW1Chunks = kCols / 64;
constexpr size_t kW1TileBytes = 16 * 128;
constexpr size_t kW1Tiles = (size_t)kNB * kW1Chunks * 2 * kW1TileBytes;

struct Ws {
  WorkspaceView sort;  // bucket sort (header = status word)
  __nv_bfloat16* a;    // [n][2][1024]
  float* da;           // [2n][1024]
  float* dh1;          // [n][16] in sorted order
  float* small_part;   // [tiles][kSmallPart]
  float* w1_part;      // [tiles][16][1024]
  uint8_t* w1_tiles;   // kW1Tiles bytes
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
  b += align_up((size_t)n * 16 * 4, 256);
  b += align_up((size_t)max_tiles(n) * kSmallPart * 4, 256);
  b += align_up((size_t)max_tiles(n) * kRowSplit * 16 * kCols * 4, 256);
  b += align_up(kW1Tiles, 1024) + 1024;
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
  w.dh1 = (float*)p;
  p += align_up((size_t)n * 16 * 4, 256);
  w.small_part = (float*)p;
  p += align_up((size_t)max_tiles(n) * kSmallPart * 4, 256);
  w.w1_part = (float*)p;
  p += align_up((size_t)max_tiles(n) * kRowSplit * 16 * kCols * 4, 256);
  w.w1_tiles = (uint8_t*)(((uintptr_t)p + 1023) & ~(uintptr_t)1023);
  p += align_up(kW1Tiles, 1024) + 1024;
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
// 3. Head over bucket tiles.
// ---------------------------------------------------------------------------
// Byte offset of (row, kbyte) in a 128B-swizzled K-major tile of 128-byte rows.
__host__ __device__ constexpr uint32_t sw128(int row, int kbyte) {
  return (uint32_t)(row * 128 + ((((kbyte >> 4) ^ row) & 7) << 4) + (kbyte & 15));
}

// W1 (fp32 master) -> the tensor-core B tiles: w = hi + lo with hi = bf16(w),
// lo = bf16(w - hi), so x . hi + x . lo carries w to ~2^-17 relative.
__global__ void t_w1tiles_kernel(const float* __restrict__ params, uint8_t* __restrict__ tiles) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;  // bucket * 16K + k * 1024 + i
  if (e >= kNB * 16 * kCols) return;
  const int b = e / (16 * kCols), k = (e / kCols) % 16, i = e % kCols;
  const float w = params[kOffW1 + e];
  const __nv_bfloat16 hi = __float2bfloat16_rn(w);
  const __nv_bfloat16 lo = __float2bfloat16_rn(w - __bfloat162float(hi));
  const int c = i / 64;
  uint8_t* t = tiles + ((size_t)(b * kW1Chunks + c) * 2) * kW1TileBytes;
  const uint32_t off = sw128(k, 2 * (i % 64));
  *reinterpret_cast<__nv_bfloat16*>(t + off) = hi;
  *reinterpret_cast<__nv_bfloat16*>(t + kW1TileBytes + off) = lo;
}

constexpr int kHStages = 4;
constexpr int kHThreads = 192;  // warps 0-3: x rows + epilogue (row = lane), 4: W1 loads + TMEM, 5: MMA

struct HeadTcSmem {
  alignas(1024) uint8_t a[kHStages][kTile * 128];  // x chunk: 128 rows x 64 bf16
  alignas(1024) uint8_t b[kHStages][2][kW1TileBytes];
  uint64_t a_full[kHStages];  // 128 arrivals: the chunk's x rows are written
  uint64_t b_full[kHStages];  // the chunk's W1 tiles landed
  uint64_t empty[kHStages];   // the chunk's MMAs completed
  uint64_t accum, drain;
  alignas(16) float w2[32][16];
  float b1[16], b2[32], w3[32];
  float b3;
  uint32_t tmem_base;
  int bucket, start, count;
  uint32_t first_tile;
  int abort;
};
static_assert(sizeof(float) * kTile * kRec <= sizeof(((HeadTcSmem*)0)->a), "records fit the x ring");

struct HeadTcArgs {
  const float* params;
  const __nv_bfloat16* a;
  const float* target;
  const uint32_t* perm;
  const WorkspaceHeader* hdr;
  const uint8_t* w1_tiles;
  int64_t n;
  float inv_n;
  float* dh1;         // [n][16] sorted order
  float* loss;        // [n]
  float* small_part;  // [tiles][kSmallPart]
  uint32_t* status;
};

__device__ __forceinline__ uint4 pack_x8(const uint4& lo, const uint4& hi) {
  float fl[8], fh[8], x[8];
  unpack8(lo, fl);
  unpack8(hi, fh);
#pragma unroll
  for (int q = 0; q < 8; ++q) x[q] = clamp01(fl[q]) * clamp01(fh[q]);
  return pack8(x);
}

__global__ void __launch_bounds__(kHThreads) t_head_tc_kernel(const HeadTcArgs A) {
  extern __shared__ uint8_t smem_raw[];
  HeadTcSmem& sm = *reinterpret_cast<HeadTcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    int b = -1, st = 0, cnt = 0;
    uint32_t ft = 0;
    if (!bucket_tile(A.hdr, kNB, kTile, blockIdx.x, &b, &st, &cnt, &ft)) b = -1;
    sm.bucket = b;
    sm.start = st;
    sm.count = cnt;
    sm.first_tile = ft;
    for (int s = 0; s < kHStages; ++s) {
      pipe::mbar_init(&sm.a_full[s], kTile);
      pipe::mbar_init(&sm.b_full[s], 1);
      pipe::mbar_init(&sm.empty[s], 1);
    }
    pipe::mbar_init(&sm.accum, 1);
    pipe::mbar_init(&sm.drain, 1);
    sm.abort = 0;
    pipe::mbar_init_fence();
  }
  __syncthreads();
  const int bk = sm.bucket;
  if (bk < 0) return;  // past the last tile (uniform; no TMEM held yet)
  if (warp == 4) {
    tc::tmem_alloc(pipe::smem_addr(&sm.tmem_base), 32);
    tc::tmem_relinquish();
  }
  for (int e = tid; e < 32 * 16; e += kHThreads) sm.w2[e / 16][e % 16] = A.params[kOffW2 + (size_t)bk * 512 + e];
  if (tid < 32) {
    sm.b2[tid] = A.params[kOffB2 + bk * 32 + tid];
    sm.w3[tid] = A.params[kOffW3 + bk * 32 + tid];
  }
  if (tid < 16) sm.b1[tid] = A.params[kOffB1 + bk * 16 + tid];
  if (tid == 0) sm.b3 = A.params[kOffB3 + bk];
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  const int start = sm.start, count = sm.count;

  if (warp < 4) {
    // ---- x rows: row r of the tile is sorted slot start + r
    const int r = tid;
    const bool valid = r < count;
    const uint32_t pos = valid ? A.perm[start + r] : 0u;
    for (int c = 0; c < kW1Chunks; ++c) {
      const int s = c % kHStages, u = c / kHStages;
      if (u > 0) pipe::mbar_wait_sleep(&sm.empty[s], (u - 1) & 1, &sm.abort, A.status);
      const int p = c >> 3, j0 = (c & 7) * 64;
      uint8_t* row = sm.a[s] + r * 128;
      if (valid) {
        const uint4* lo = (const uint4*)(A.a + (2 * (int64_t)pos + p) * kCols + j0);
        const uint4* hi = lo + 512 / 8;
        uint4 vl[8], vh[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          vl[q] = __ldg(lo + q);
          vh[q] = __ldg(hi + q);
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) *(uint4*)(row + (((q ^ r) & 7) << 4)) = pack_x8(vl[q], vh[q]);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) *(uint4*)(row + (q << 4)) = make_uint4(0, 0, 0, 0);
      }
      pipe::fence_proxy_async_smem();
      pipe::mbar_arrive(&sm.a_full[s]);
    }
    // ---- epilogue: TMEM lane = row
    const bool ok = pipe::mbar_wait_sleep(&sm.accum, 0, &sm.abort, A.status);
    tc::fence_after_sync();
    uint32_t v[16];
    __syncwarp();
    tc::tmem_ld16(tmem + ((uint32_t)(32 * warp) << 16), v);
    tc::wait_ld();
    // The rows' records go to shared memory over the x ring (idle: every MMA
    // has completed, and with it every x write).  The stack runs row-wise
    // with the L2 rows read from shared memory one at a time, so the
    // compiler keeps only h1 and dh1 in registers.
    float* rec = reinterpret_cast<float*>(&sm.a[0][0]);
    float* my = rec + (size_t)r * kRec;
    const bool live = ok && valid;
    float h1[16], dh1[16];
    uint32_t mask1 = 0, mask2 = 0;  // clamp derivatives (bit k: z strictly inside (0, 1))
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float z = sm.b1[k] + __uint_as_float(v[k]);
      h1[k] = live ? clamp01(z) : 0.f;
      mask1 |= (dclamp01(z) != 0.f ? 1u : 0u) << k;
      my[kHH1 + k] = h1[k];
    }
    float sc = sm.b3;
#pragma unroll 1
    for (int m = 0; m < 32; ++m) {
      const float4* wr = reinterpret_cast<const float4*>(&sm.w2[m][0]);
      float z = sm.b2[m];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 w = wr[q];
        z += w.x * h1[4 * q];
        z += w.y * h1[4 * q + 1];
        z += w.z * h1[4 * q + 2];
        z += w.w * h1[4 * q + 3];
      }
      const float h2 = live ? clamp01(z) : 0.f;
      mask2 |= (dclamp01(z) != 0.f ? 1u : 0u) << m;
      sc += sm.w3[m] * h2;
      my[kHH2 + m] = h2;
    }
    float ds = 0.f;
    if (live) {
      const float sg = 1.f / (1.f + __expf(-sc / 400.f));
      const float d = sg - A.target[pos];
      ds = 2.f * d * sg * (1.f - sg) / 400.f * A.inv_n;
      A.loss[pos] = d * d;
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) dh1[k] = 0.f;
#pragma unroll 1
    for (int m = 0; m < 32; ++m) {
      const float dh2 = (mask2 >> m) & 1u ? ds * sm.w3[m] : 0.f;
      my[kHDH2 + m] = dh2;
      const float4* wr = reinterpret_cast<const float4*>(&sm.w2[m][0]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 w = wr[q];
        dh1[4 * q] += w.x * dh2;
        dh1[4 * q + 1] += w.y * dh2;
        dh1[4 * q + 2] += w.z * dh2;
        dh1[4 * q + 3] += w.w * dh2;
      }
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      dh1[k] = (mask1 >> k) & 1u ? dh1[k] : 0.f;
      my[kHDH1 + k] = dh1[k];
    }
    my[kHDS] = ds;
    if (live) {
      float4* o = (float4*)(A.dh1 + (size_t)(start + r) * 16);
#pragma unroll
      for (int q = 0; q < 4; ++q) o[q] = make_float4(dh1[4 * q], dh1[4 * q + 1], dh1[4 * q + 2], dh1[4 * q + 3]);
    }
    // ---- per-tile partial gradients of the small stack tensors: the
    //      records summed over the tile's rows in order
    named_bar_sync(1, kTile);
    float* part = A.small_part + (size_t)blockIdx.x * kSmallPart;
    for (int e = tid; e < 593; e += kTile) {
      float acc = 0.f;
      if (e < 512) {
        const int m = e / 16, k = e % 16;
        for (int q = 0; q < count; ++q) acc += rec[q * kRec + kHDH2 + m] * rec[q * kRec + kHH1 + k];
      } else if (e < 544) {
        const int m = e - 512;
        for (int q = 0; q < count; ++q) acc += rec[q * kRec + kHDS] * rec[q * kRec + kHH2 + m];
      } else if (e < 576) {
        const int m = e - 544;
        for (int q = 0; q < count; ++q) acc += rec[q * kRec + kHDH2 + m];
      } else if (e < 592) {
        const int k = e - 576;
        for (int q = 0; q < count; ++q) acc += rec[q * kRec + kHDH1 + k];
      } else {
        for (int q = 0; q < count; ++q) acc += rec[q * kRec + kHDS];
      }
      part[e] = acc;
    }
  } else if (warp == 4) {
    // ---- W1 tiles of the bucket, chunk by chunk
    if (lane == 0) {
      int issued = 0;
      for (int c = 0; c < kW1Chunks; ++c) {
        const int s = c % kHStages, u = c / kHStages;
        if (u > 0 && !pipe::mbar_wait_sleep(&sm.empty[s], (u - 1) & 1, &sm.abort, A.status)) break;
        pipe::mbar_arrive_expect_tx(&sm.b_full[s], 2 * kW1TileBytes);
        pipe::bulk_copy_g2s(&sm.b[s][0][0], A.w1_tiles + ((size_t)(bk * kW1Chunks + c) * 2) * kW1TileBytes,
                            2 * kW1TileBytes, &sm.b_full[s]);
        ++issued;
      }
      if (sm.abort)
        for (int c = max(0, issued - kHStages); c < issued; ++c)
          pipe::mbar_wait_drain(&sm.b_full[c % kHStages], (c / kHStages) & 1, A.status);
    }
    __syncwarp();
  } else {
    // ---- MMA issuer: per chunk 4 K steps x (hi, lo)
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(kTile, 16);
      for (int c = 0; c < kW1Chunks; ++c) {
        const int s = c % kHStages, u = c / kHStages;
        if (!pipe::mbar_wait_sleep(&sm.a_full[s], u & 1, &sm.abort, A.status)) break;
        if (!pipe::mbar_wait_sleep(&sm.b_full[s], u & 1, &sm.abort, A.status)) break;
        tc::fence_after_sync();
        const uint32_t a0 = pipe::smem_addr(sm.a[s]);
        const uint32_t bh = pipe::smem_addr(sm.b[s][0]), bl = pipe::smem_addr(sm.b[s][1]);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = tc::smem_desc(a0 + kk * 32, 0, 1024, tc::kSwizzle128B);
          tc::mma_bf16(tmem, ad, tc::smem_desc(bh + kk * 32, 0, 1024, tc::kSwizzle128B), idesc,
                       (c | kk) != 0 ? 1u : 0u);
          tc::mma_bf16(tmem, ad, tc::smem_desc(bl + kk * 32, 0, 1024, tc::kSwizzle128B), idesc, 1u);
        }
        tc::commit(pipe::smem_addr(&sm.empty[s]));
      }
      tc::commit(pipe::smem_addr(&sm.accum));
      tc::commit(pipe::smem_addr(&sm.drain));
      pipe::mbar_wait_drain(&sm.drain, 0, A.status);
    }
    __syncwarp();
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 4) tc::tmem_dealloc(tmem, 32);
}

// dx = dh1 . W1 and da through the pack and the clamps, per bucket tile,
// with the tile's rows split over kRowSplit CTAs (blockIdx.y): thread t owns
// x columns [4t, 4t+4) (perspective t / 128, pair columns j and j + 512 with
// j = 4 (t % 128)), holds its 16 x 4 W1 entries in registers and walks its
// rows (coalesced 8-byte reads of a, 16-byte writes of da).
constexpr int kColThreads = 256;

__global__ void __launch_bounds__(kColThreads) t_dx_kernel(const float* __restrict__ params,
                                                           const __nv_bfloat16* __restrict__ a,
                                                           const float* __restrict__ dh1,
                                                           const uint32_t* __restrict__ perm,
                                                           const WorkspaceHeader* hdr, float* __restrict__ da) {
  constexpr int kRows = kTile / kRowSplit;
  __shared__ float d_s[kRows][16];
  int bk, start, count;
  uint32_t ft;
  if (!bucket_tile(hdr, kNB, kTile, blockIdx.x, &bk, &start, &count, &ft)) return;
  const int r0 = blockIdx.y * kRows, r1 = min(count, r0 + kRows);
  if (r0 >= r1) return;
  const int t = threadIdx.x, p = t >> 7, j = 4 * (t & 127);
  for (int e = t; e < (r1 - r0) * 16; e += kColThreads) d_s[e / 16][e % 16] = dh1[(size_t)(start + r0) * 16 + e];
  float w[16][4];
  const float* w1 = params + kOffW1 + (size_t)bk * 16 * kCols + 4 * t;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float4 x0 = __ldg((const float4*)(w1 + (size_t)k * kCols));
    w[k][0] = x0.x; w[k][1] = x0.y; w[k][2] = x0.z; w[k][3] = x0.w;
  }
  __syncthreads();
  for (int r = r0; r < r1; ++r) {
    const uint32_t pos = perm[start + r];
    const __nv_bfloat16* ap = a + (2 * (int64_t)pos + p) * kCols + j;
    const uint2 vl = *(const uint2*)ap, vh = *(const uint2*)(ap + 512);
    const float2 l0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vl.x));
    const float2 l1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vl.y));
    const float2 h0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vh.x));
    const float2 h1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vh.y));
    const float alo[4] = {l0.x, l0.y, l1.x, l1.y}, ahi[4] = {h0.x, h0.y, h1.x, h1.y};
    float dx[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float g = d_s[r - r0][k];
#pragma unroll
      for (int q = 0; q < 4; ++q) dx[q] += w[k][q] * g;
    }
    float dlo[4], dhi[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      dlo[q] = dx[q] * clamp01(ahi[q]) * dclamp01(alo[q]);
      dhi[q] = dx[q] * clamp01(alo[q]) * dclamp01(ahi[q]);
    }
    float* dp = da + (2 * (int64_t)pos + p) * kCols + j;
    *(float4*)dp = make_float4(dlo[0], dlo[1], dlo[2], dlo[3]);
    *(float4*)(dp + 512) = make_float4(dhi[0], dhi[1], dhi[2], dhi[3]);
  }
}

// Partial dW1[k][i] = sum over a quarter of a tile's rows (in order) of
// dh1[k] x[i]; thread t owns columns [4t, 4t+4); partial index = tile *
// kRowSplit + blockIdx.y.
__global__ void __launch_bounds__(kColThreads) t_w1part_kernel(const __nv_bfloat16* __restrict__ a,
                                                               const float* __restrict__ dh1,
                                                               const uint32_t* __restrict__ perm,
                                                               const WorkspaceHeader* hdr,
                                                               float* __restrict__ w1_part) {
  constexpr int kRows = kTile / kRowSplit;
  __shared__ float d_s[kRows][16];
  int bk, start, count;
  uint32_t ft;
  if (!bucket_tile(hdr, kNB, kTile, blockIdx.x, &bk, &start, &count, &ft)) return;
  const int r0 = blockIdx.y * kRows, r1 = min(count, r0 + kRows);
  const int t = threadIdx.x, p = t >> 7, j = 4 * (t & 127);
  for (int e = t; e < max(r1 - r0, 0) * 16; e += kColThreads) d_s[e / 16][e % 16] = dh1[(size_t)(start + r0) * 16 + e];
  __syncthreads();
  float acc[16][4];
#pragma unroll
  for (int k = 0; k < 16; ++k)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[k][q] = 0.f;
  for (int r = r0; r < r1; ++r) {
    const uint32_t pos = perm[start + r];
    const __nv_bfloat16* ap = a + (2 * (int64_t)pos + p) * kCols + j;
    const uint2 vl = *(const uint2*)ap, vh = *(const uint2*)(ap + 512);
    const float2 l0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vl.x));
    const float2 l1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vl.y));
    const float2 h0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vh.x));
    const float2 h1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vh.y));
    const float alo[4] = {l0.x, l0.y, l1.x, l1.y}, ahi[4] = {h0.x, h0.y, h1.x, h1.y};
    float x[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) x[q] = __bfloat162float(__float2bfloat16_rn(clamp01(alo[q]) * clamp01(ahi[q])));
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float g = d_s[r - r0][k];
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[k][q] += g * x[q];
    }
  }
  float* out = w1_part + ((size_t)blockIdx.x * kRowSplit + blockIdx.y) * 16 * kCols + 4 * t;
#pragma unroll
  for (int k = 0; k < 16; ++k) *(float4*)(out + (size_t)k * kCols) = make_float4(acc[k][0], acc[k][1], acc[k][2], acc[k][3]);
}

// Ordered sums of the tile partials of each bucket: dW1 (one thread per
// (bucket, k, i)) and the small tensors (one CTA per bucket).
__device__ __forceinline__ void bucket_tiles(const WorkspaceHeader* hdr, int bk, uint32_t* first, uint32_t* n) {
  uint32_t f = 0;
  for (int b = 0; b < bk; ++b) f += (hdr->counts[b] + kTile - 1) / kTile;
  *first = f;
  *n = (hdr->counts[bk] + kTile - 1) / kTile;
}

__global__ void t_w1sum_kernel(const float* __restrict__ w1_part, const WorkspaceHeader* hdr, float* grads) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;  // bucket * 16K + k * 1024 + i
  if (e >= kNB * 16 * kCols) return;
  const int bk = e / (16 * kCols), ki = e % (16 * kCols);
  uint32_t first, nt;
  bucket_tiles(hdr, bk, &first, &nt);
  float acc = 0.f;
  for (uint32_t g = first * kRowSplit; g < (first + nt) * kRowSplit; ++g) acc += w1_part[(size_t)g * 16 * kCols + ki];
  grads[kOffW1 + e] = acc;
}

__global__ void t_smallsum_kernel(const float* __restrict__ small_part, const WorkspaceHeader* hdr, float* grads) {
  const int bk = blockIdx.x, e = threadIdx.x;
  if (e >= 593) return;
  uint32_t first, nt;
  bucket_tiles(hdr, bk, &first, &nt);
  float acc = 0.f;
  for (uint32_t g = 0; g < nt; ++g) acc += small_part[(size_t)(first + g) * kSmallPart + e];
  if (e < 512)
    grads[kOffW2 + (size_t)bk * 512 + e] = acc;
  else if (e < 544)
    grads[kOffW3 + bk * 32 + (e - 512)] = acc;
  else if (e < 576)
    grads[kOffB2 + bk * 32 + (e - 544)] = acc;
  else if (e < 592)
    grads[kOffB1 + bk * 16 + (e - 576)] = acc;
  else
    grads[kOffB3 + bk] = acc;
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
                              float beta2, float eps, float c1, float c2, const float* skip) {
  if (skip != nullptr && *skip != 0.f) return;  // some rank's batch was bad: no update anywhere
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

// The workspace status word as a float flag (0 = clean) for the gradient
// all-reduce, so every rank sees whether any rank's batch was bad.
__global__ void t_status_flag_kernel(const uint32_t* status, float* flag) { *flag = *status != 0u ? 1.f : 0.f; }

__global__ void t_shadow_kernel(const float* __restrict__ w, int64_t count, __nv_bfloat16* shadow) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride)
    shadow[i] = __float2bfloat16_rn(w[i]);
}

}  // namespace tr
}  // namespace cnnue

using namespace cnnue;
using namespace cnnue::tr;

namespace {
size_t head_tc_smem_bytes() { return sizeof(HeadTcSmem) + 1024; }
// Opt the head kernel in to its dynamic shared memory once per device.
int head_tc_setup() {
  static std::mutex mu;
  static bool done[64] = {};
  int dev = 0;
  CNNUE_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && !done[dev]) {
    CNNUE_CUDA_TRY(cudaFuncSetAttribute(t_head_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)head_tc_smem_bytes()));
    done[dev] = true;
  }
  return CNNUE_OK;
}
}  // namespace

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

namespace {

int check_fb_args(const float* d_params, const uint16_t* d_shadow, const uint16_t* d_indices, uint32_t n_indices,
                  const uint32_t* d_offsets, int64_t n, const float* d_target, const float* d_grads, void* d_ws,
                  size_t ws_size) {
  if (n <= 0 || n > (int64_t)INT32_MAX) return set_error(CNNUE_ERR_INVALID_ARG, "bad n_positions");
  if (!d_params || !d_shadow || !d_offsets || !d_target || !d_grads || !d_ws || (n_indices && !d_indices))
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer");
  if (((uintptr_t)d_params | (uintptr_t)d_shadow | (uintptr_t)d_grads) & 15u)
    return set_error(CNNUE_ERR_INVALID_ARG, "params, shadow and grads must be 16-byte aligned");
  if (ws_size < ws_bytes(n, n_indices))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu < %zu", ws_size, ws_bytes(n, n_indices));
  return CNNUE_OK;
}

}  // namespace

int cnnue_t_forward_backward_begin(const float* d_params, const uint16_t* d_shadow, const uint16_t* d_indices,
                                   uint32_t n_indices, const uint32_t* d_offsets, int64_t n, const float* d_target,
                                   float* d_grads, void* d_ws, size_t ws_size, void* stream) {
  int st = check_fb_args(d_params, d_shadow, d_indices, n_indices, d_offsets, n, d_target, d_grads, d_ws, ws_size);
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
  Ws w = carve(d_ws, n, n_indices);
  st = head_tc_setup();
  if (st) return st;
  st = launch_bucket_sort(d_offsets, n_indices, nullptr, n, 1, kNB, d_ws, s);
  if (st) return st;
  uint32_t* status = &w.sort.hdr->status;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  t_gather_kernel<<<sms * 4, 256, 0, s>>>((const __nv_bfloat16*)d_shadow, d_indices, n_indices,
                                          d_offsets, n, w.a, status);
  if ((st = check_launch_error("t_gather_kernel"))) return st;
  t_w1tiles_kernel<<<kNB * 16 * kCols / 256, 256, 0, s>>>(d_params, w.w1_tiles);
  if ((st = check_launch_error("t_w1tiles_kernel"))) return st;
  const unsigned tiles = (unsigned)max_tiles(n);
  HeadTcArgs h{d_params, w.a, d_target, w.sort.perm, w.sort.hdr, w.w1_tiles, n, 1.f / (float)n,
               w.dh1, w.loss, w.small_part, status};
  t_head_tc_kernel<<<tiles, kHThreads, head_tc_smem_bytes(), s>>>(h);
  if ((st = check_launch_error("t_head_tc_kernel"))) return st;
  t_dx_kernel<<<dim3(tiles, kRowSplit), kColThreads, 0, s>>>(d_params, w.a, w.dh1, w.sort.perm, w.sort.hdr, w.da);
  if ((st = check_launch_error("t_dx_kernel"))) return st;
  t_w1part_kernel<<<dim3(tiles, kRowSplit), kColThreads, 0, s>>>(w.a, w.dh1, w.sort.perm, w.sort.hdr, w.w1_part);
  if ((st = check_launch_error("t_w1part_kernel"))) return st;
  t_w1sum_kernel<<<kNB * 16 * kCols / 256, 256, 0, s>>>(w.w1_part, w.sort.hdr, d_grads);
  if ((st = check_launch_error("t_w1sum_kernel"))) return st;
  t_smallsum_kernel<<<kNB, 608, 0, s>>>(w.small_part, w.sort.hdr, d_grads);
  if ((st = check_launch_error("t_smallsum_kernel"))) return st;
  t_list_of_kernel<<<(unsigned)((2 * n + 255) / 256), 256, 0, s>>>(d_offsets, n_indices, 2 * n,
                                                                  w.list_of);
  if ((st = check_launch_error("t_list_of_kernel"))) return st;
  FtDecoder dec{kF + 1, d_indices, w.list_of, n_indices};
  return seg::launch_bwd_prepare((int64_t)n_indices + 2 * n, dec, w.seg, s);
}

int cnnue_t_ft_grad_rows(int64_t n, uint32_t n_indices, float* d_grads, void* d_ws, size_t ws_size,
                         int64_t row_begin, int64_t row_end, void* stream) {
  if (n <= 0 || !d_grads || !d_ws) return set_error(CNNUE_ERR_INVALID_ARG, "null buffer or bad n_positions");
  if (ws_size < ws_bytes(n, n_indices)) return set_error(CNNUE_ERR_WORKSPACE, "workspace too small");
  if (row_begin < 0 || row_end > kF + 1 || row_begin > row_end)
    return set_error(CNNUE_ERR_INVALID_ARG, "row range [%lld, %lld) outside [0, %d]", (long long)row_begin,
                     (long long)row_end, kF + 1);
  Ws w = carve(d_ws, n, n_indices);
  return seg::launch_bwd_rows((int64_t)n_indices + 2 * n, 1, w.da, kCols, kF + 1, d_grads + kOffFt, w.seg,
                              row_begin, row_end, (cudaStream_t)stream);
}

int cnnue_t_finish(int64_t n, uint32_t n_indices, float* d_loss, void* d_ws, size_t ws_size, float* d_flag,
                   void* stream) {
  if (n <= 0 || !d_loss || !d_ws) return set_error(CNNUE_ERR_INVALID_ARG, "null buffer or bad n_positions");
  if (ws_size < ws_bytes(n, n_indices)) return set_error(CNNUE_ERR_WORKSPACE, "workspace too small");
  cudaStream_t s = (cudaStream_t)stream;
  Ws w = carve(d_ws, n, n_indices);
  t_loss_kernel<<<1, 1024, 0, s>>>(w.loss, n, d_loss);
  int st = check_launch_error("t_loss_kernel");
  if (st || !d_flag) return st;
  t_status_flag_kernel<<<1, 1, 0, s>>>(&w.sort.hdr->status, d_flag);
  return check_launch_error("t_status_flag_kernel");
}

int cnnue_t_forward_backward(const float* d_params, const uint16_t* d_shadow,
                             const uint16_t* d_indices, uint32_t n_indices,
                             const uint32_t* d_offsets, int64_t n, const float* d_target,
                             float* d_grads, float* d_loss, void* d_ws, size_t ws_size,
                             void* stream) {
  if (!d_loss) return set_error(CNNUE_ERR_INVALID_ARG, "null loss");
  int st = cnnue_t_forward_backward_begin(d_params, d_shadow, d_indices, n_indices, d_offsets, n, d_target, d_grads,
                                          d_ws, ws_size, stream);
  if (st) return st;
  st = cnnue_t_ft_grad_rows(n, n_indices, d_grads, d_ws, ws_size, 0, kF + 1, stream);
  if (st) return st;
  return cnnue_t_finish(n, n_indices, d_loss, d_ws, ws_size, nullptr, stream);
}

int cnnue_t_adam(float* d_params, float* d_m, float* d_v, const float* d_grads, uint16_t* d_shadow,
                 float grad_scale, float lr, float beta1, float beta2, float eps, int step,
                 const float* d_skip, void* stream) {
  if (!d_params || !d_m || !d_v || !d_grads || !d_shadow)
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer");
  if (step < 1) return set_error(CNNUE_ERR_INVALID_ARG, "step must be >= 1");
  const float c1 = 1.f - powf(beta1, (float)step);
  const float c2 = 1.f - powf(beta2, (float)step);
  t_adam_kernel<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(d_params, d_m, d_v, d_grads, kParams,
                                                            (__nv_bfloat16*)d_shadow, kOffW1,
                                                            grad_scale, lr, beta1, beta2, eps, c1, c2, d_skip);
  return check_launch_error("t_adam_kernel");
}

int cnnue_t_adam_range(float* d_params, float* d_m, float* d_v, const float* d_grads, uint16_t* d_shadow,
                       int64_t begin, int64_t end, float grad_scale, float lr, float beta1, float beta2, float eps,
                       int step, const float* d_skip, void* stream) {
  if (!d_params || !d_m || !d_v || !d_grads || !d_shadow)
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer");
  if (step < 1) return set_error(CNNUE_ERR_INVALID_ARG, "step must be >= 1");
  if (begin < 0 || end > kParams || begin > end)
    return set_error(CNNUE_ERR_INVALID_ARG, "parameter range [%lld, %lld) outside [0, %lld)", (long long)begin,
                     (long long)end, (long long)kParams);
  if (begin == end) return CNNUE_OK;
  const float c1 = 1.f - powf(beta1, (float)step);
  const float c2 = 1.f - powf(beta2, (float)step);
  const int64_t shadow_end = std::min<int64_t>(end, kOffW1);
  t_adam_kernel<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(
      d_params + begin, d_m + begin, d_v + begin, d_grads + begin, end - begin,
      (__nv_bfloat16*)d_shadow + begin, std::max<int64_t>(0, shadow_end - begin), grad_scale, lr, beta1, beta2, eps,
      c1, c2, d_skip);
  return check_launch_error("t_adam_kernel");
}

}  // extern "C"
