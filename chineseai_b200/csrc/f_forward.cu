// f_forward.cu - fp32 HalfKA NNUE evaluation on sm_100a.
//
// One cooperative launch per batch (after the workspace header is cleared):
// f_fused_kernel, every CTA resident, in two phases split by a grid barrier.
//   Phase 1 (the FT gather): every warp takes (position, perspective) lists
//   from a global counter, one list at a time (the next one claimed while the
//   current one's rows are in flight), so long and short lists balance over
//   the whole GPU.  Lane l owns FT columns [4l, 4l + 4) and
//   [128 + 4l, 128 + 4l + 4): two 16-byte loads per 1 KB row, each load
//   instruction covering 512 contiguous bytes, six rows in flight.  Each
//   column is summed bias-first in index order with plain fp32 adds - the
//   order of the scalar evaluator - so the FT outputs are bit-identical to
//   it; the clipped values go to the workspace x [n][512] (perspective 0, then
//   1; 8 MB at 4096 positions, L2-resident until phase 2), and the warp that
//   gathered a position's perspective-0 list appends the position to its
//   bucket's list (bucket = min((max(n0, 1) - 1) >> 2, 7)).  Offsets and
//   indices are checked here.  While the lists run, each CTA bulk-copies its
//   bucket's 16x512 L1 weights into shared memory and prefetches its share of
//   the FT table into L2 (the table is cold after an L2 flush).
//   Phase 2 (the stacks): CTA c serves bucket c % 8, its share of that
//   bucket's list two positions per warp (each weight read from shared
//   memory serves both): L1 by lanes over 16 of the 512
//   inputs and a 16-way warp reduce-scatter, L2 by lanes over its 32 outputs,
//   L3 by a warp sum (a fixed order, within 1e-4 of the scalar one).  The
//   stack work per position does not depend on the bucket, so the phase is
//   balanced by equal shares.
// Scores do not depend on the order of the bucket lists (each position is
// evaluated on its own), so the result is deterministic.
#include <algorithm>

#include "common.cuh"
#include "pipeline.cuh"

namespace cnnue {
namespace f {

constexpr int kF = CNNUE_F_FEATURES;
constexpr int kCols = CNNUE_F_COLS;
constexpr int kRowBytes = kCols * 4;
constexpr int kNB = CNNUE_F_BUCKETS;
constexpr int kIn = 2 * kCols;
constexpr int kUnroll = 6;   // rows in flight per warp
constexpr int kWarps = 8;
constexpr int kMinBlocks = 3;  // CTAs per SM the register budget is set for
constexpr uint32_t kW1Bytes = 16 * kIn * 4;
constexpr unsigned kFull = 0xffffffffu;
static_assert(kCols == 256 && kIn == 512, "lane mapping assumes 256 columns per perspective");

struct DevWeights {
  const float* ft;
  const float* bias;
  const float* l1w;
  const float* l1b;
  const float* l2w;
  const float* l2b;
  const float* l3w;
  const float* l3b;
};

// Counters in the cleared workspace header.
struct Header {
  uint32_t status;
  uint32_t next_list;   // phase 1 work counter
  uint32_t arrived;     // grid barrier
  uint32_t pad0[29];
  uint32_t bucket_n[32];  // positions appended to each bucket's list
  uint32_t pad1[64];
};
static_assert(sizeof(Header) == sizeof(WorkspaceHeader), "the header is the common workspace header");

struct Args {
  DevWeights w;
  const uint16_t* idx;
  uint32_t n_idx;
  const uint32_t* offsets;
  float* x;          // [n][512] clipped FT outputs
  uint32_t* blist;   // [8][n] positions per bucket
  float* out;
  uint32_t n;        // positions, at most 2^31 - 1
  Header* hdr;
};

struct __align__(16) Smem {
  float w1[16 * kIn];  // bucket c % 8's L1 weights [16][512] (32 KB)
  float w2[32 * 16];   // L2 weights [32][16]
  float b1[16];
  float b2[32];
  float w3[32];
  uint64_t bar;        // completes when w1 has landed
  int abort;
  float b3;
};

__device__ __forceinline__ void add4(float4& a, const float4& b) {
  a.x += b.x;
  a.y += b.y;
  a.z += b.z;
  a.w += b.w;
}

__device__ __forceinline__ float clamp01(float v) { return fminf(fmaxf(v, 0.f), 1.f); }
__device__ __forceinline__ float4 clamp01(float4 v) {
  return make_float4(clamp01(v.x), clamp01(v.y), clamp01(v.z), clamp01(v.w));
}

__device__ __forceinline__ float dot4(const float4 w, const float4 x, float s) {
  s = fmaf(w.x, x.x, s);
  s = fmaf(w.y, x.y, s);
  s = fmaf(w.z, x.z, s);
  return fmaf(w.w, x.w, s);
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// All CTAs of the (cooperative, fully resident) grid meet here; a wait past
// the limit flags CNNUE_STATUS_TIMEOUT and lets the CTA go on.
__device__ __forceinline__ void grid_barrier(Header* h) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(&h->arrived, 1u);
    const unsigned long long t0 = pipe::globaltimer();
    while (ld_acquire(&h->arrived) < gridDim.x) {
      if (pipe::globaltimer() - t0 > pipe::kWaitLimitNs) {
        atomicOr(&h->status, CNNUE_STATUS_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
    __threadfence();
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kWarps * 32, kMinBlocks) f_fused_kernel(const Args a) {
  __shared__ Smem s;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.x % kNB;
  {
    const int t = threadIdx.x;
    if (t == 0) {
      s.abort = 0;
      pipe::mbar_init(&s.bar, 1);
      pipe::mbar_init_fence();
      pipe::mbar_arrive_expect_tx(&s.bar, kW1Bytes);
      pipe::bulk_copy_g2s(s.w1, a.w.l1w + (size_t)b * 16 * kIn, kW1Bytes, &s.bar);
      // this CTA's share of the FT table into L2 (16-byte granules)
      const uint64_t table = (uint64_t)kF * kRowBytes;
      const uint64_t share = ((table + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
      const uint64_t lo = share * blockIdx.x;
      if (lo < table) prefetch_l2((const char*)a.w.ft + lo, (uint32_t)min(share, table - lo));
    } else if (t >= 32 && t < 160) {
      ((float4*)s.w2)[t - 32] = __ldg((const float4*)(a.w.l2w + (size_t)b * 32 * 16) + (t - 32));
    } else if (t >= 160 && t < 176) {
      s.b1[t - 160] = __ldg(a.w.l1b + b * 16 + (t - 160));
    } else if (t >= 176 && t < 208) {
      s.b2[t - 176] = __ldg(a.w.l2b + b * 32 + (t - 176));
    } else if (t >= 208 && t < 240) {
      s.w3[t - 208] = __ldg(a.w.l3w + b * 32 + (t - 208));
    } else if (t == 240) {
      s.b3 = __ldg(a.w.l3b + b);
    }
  }
  // ---- phase 1: FT gather, one list per claim --------------------------------
  const uint32_t lists = 2 * a.n;
  const char* ft = (const char*)a.w.ft + lane * 16;
  uint32_t l = 0;
  if (lane == 0) l = atomicAdd(&a.hdr->next_list, 1u);
  l = __shfl_sync(kFull, l, 0);
  while (l < lists) {
    uint32_t next = 0;
    if (lane == 0) next = atomicAdd(&a.hdr->next_list, 1u);  // lands while this list runs
    const uint32_t o0 = a.offsets[l], o1 = a.offsets[l + 1];
    if (lane == 0 && !(o0 <= o1 && o1 <= a.n_idx)) atomicOr(&a.hdr->status, CNNUE_STATUS_BAD_OFFSETS);
    const uint32_t ob = min(o0, a.n_idx);
    const uint32_t oe = min(max(o1, ob), a.n_idx);
    float4 acc0 = __ldg((const float4*)(a.w.bias + 4 * lane));
    float4 acc1 = __ldg((const float4*)(a.w.bias + 128 + 4 * lane));
    for (uint32_t rb = ob; rb < oe; rb += 32) {
      const int cnt = (int)min(32u, oe - rb);
      uint32_t my = lane < cnt ? (uint32_t)a.idx[rb + lane] : 0u;
      if (lane < cnt && my >= (uint32_t)kF) {
        atomicOr(&a.hdr->status, CNNUE_STATUS_BAD_INDEX);
        my = 0xffffffffu;
      }
      for (int r0 = 0; r0 < cnt; r0 += kUnroll) {
        float4 v0[kUnroll], v1[kUnroll];
        bool ok[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const uint32_t f = __shfl_sync(kFull, my, (r0 + u) & 31);
          ok[u] = r0 + u < cnt && f != 0xffffffffu;
          if (ok[u]) {
            v0[u] = ldg_stream16f(ft + (size_t)f * kRowBytes);
            v1[u] = ldg_stream16f(ft + (size_t)f * kRowBytes + 512);
          }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          if (ok[u]) {
            add4(acc0, v0[u]);
            add4(acc1, v1[u]);
          }
      }
    }
    const uint32_t q = l >> 1;
    float* xo = a.x + (size_t)q * kIn + (l & 1) * kCols + 4 * lane;
    *(float4*)xo = clamp01(acc0);
    *(float4*)(xo + 128) = clamp01(acc1);
    if (!(l & 1) && lane == 0) {
      const uint32_t bk = min((max(oe - ob, 1u) - 1u) >> 2, (uint32_t)(kNB - 1));
      a.blist[(size_t)bk * a.n + atomicAdd(&a.hdr->bucket_n[bk], 1u)] = q;
    }
    l = __shfl_sync(kFull, next, 0);
  }
  grid_barrier(a.hdr);
  // ---- phase 2: bucket stacks --------------------------------------------------
  const uint32_t cnt = *(volatile uint32_t*)&a.hdr->bucket_n[b];
  const uint32_t ctas = gridDim.x / kNB, c = blockIdx.x / kNB;
  const uint32_t p_begin = (uint32_t)((uint64_t)cnt * c / ctas);
  const uint32_t p_end = (uint32_t)((uint64_t)cnt * (c + 1) / ctas);
  if (p_begin + 2 * warp < p_end) pipe::mbar_wait(&s.bar, 0, &s.abort, &a.hdr->status);
  const uint32_t* list = a.blist + (size_t)b * a.n;
  // two positions per warp, so that every weight load from shared memory
  // serves both (the phase is bound by shared-memory reads of the weights)
  for (uint32_t i = p_begin + 2 * warp; i < p_end; i += 2 * kWarps) {
    const bool two = i + 1 < p_end;
    const uint32_t qa = __ldcg(list + i);
    const uint32_t qb = two ? __ldcg(list + i + 1) : qa;
    // x was written in phase 1 by other CTAs: read through L2, not the
    // read-only path; lane l holds inputs 4l + 128k (k < 4)
    const float4* xpa = (const float4*)(a.x + (size_t)qa * kIn) + lane;
    const float4* xpb = (const float4*)(a.x + (size_t)qb * kIn) + lane;
    float4 xa[4], xb[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      xa[k] = __ldcg(xpa + 32 * k);
      xb[k] = __ldcg(xpb + 32 * k);
    }
    // the 16 sums of each position are reduced over the 32 lanes so that
    // output o ends on lanes 2o, 2o+1 (the first halving step taken as each
    // pair of outputs o, o + 8 is formed)
    const float* wp = s.w1 + 4 * lane;
    float va[8], vb[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float la = 0.f, ha = 0.f, lb = 0.f, hb = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 wl = *(const float4*)(wp + j * kIn + 128 * k);
        const float4 wh = *(const float4*)(wp + (j + 8) * kIn + 128 * k);
        la = dot4(wl, xa[k], la);
        ha = dot4(wh, xa[k], ha);
        lb = dot4(wl, xb[k], lb);
        hb = dot4(wh, xb[k], hb);
      }
      const bool up = lane & 16;
      va[j] = (up ? ha : la) + __shfl_xor_sync(kFull, up ? la : ha, 16);
      vb[j] = (up ? hb : lb) + __shfl_xor_sync(kFull, up ? lb : hb, 16);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool up = lane & 8;
      va[j] = (up ? va[j + 4] : va[j]) + __shfl_xor_sync(kFull, up ? va[j] : va[j + 4], 8);
      vb[j] = (up ? vb[j + 4] : vb[j]) + __shfl_xor_sync(kFull, up ? vb[j] : vb[j + 4], 8);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const bool up = lane & 4;
      va[j] = (up ? va[j + 2] : va[j]) + __shfl_xor_sync(kFull, up ? va[j] : va[j + 2], 4);
      vb[j] = (up ? vb[j + 2] : vb[j]) + __shfl_xor_sync(kFull, up ? vb[j] : vb[j + 2], 4);
    }
    {
      const bool up = lane & 2;
      va[0] = (up ? va[1] : va[0]) + __shfl_xor_sync(kFull, up ? va[0] : va[1], 2);
      vb[0] = (up ? vb[1] : vb[0]) + __shfl_xor_sync(kFull, up ? vb[0] : vb[1], 2);
    }
    va[0] += __shfl_xor_sync(kFull, va[0], 1);
    vb[0] += __shfl_xor_sync(kFull, vb[0], 1);
    const float b1 = s.b1[lane >> 1];
    const float ya = clamp01(b1 + va[0]), yb = clamp01(b1 + vb[0]);  // output lane >> 1
    const float4* w2r = (const float4*)(s.w2 + lane * 16);
    float sa = s.b2[lane], sb = sa;
#pragma unroll
    for (int qd = 0; qd < 4; ++qd) {
      const float4 w2 = w2r[qd];
      sa += w2.x * __shfl_sync(kFull, ya, 8 * qd) + w2.y * __shfl_sync(kFull, ya, 8 * qd + 2) +
            w2.z * __shfl_sync(kFull, ya, 8 * qd + 4) + w2.w * __shfl_sync(kFull, ya, 8 * qd + 6);
      sb += w2.x * __shfl_sync(kFull, yb, 8 * qd) + w2.y * __shfl_sync(kFull, yb, 8 * qd + 2) +
            w2.z * __shfl_sync(kFull, yb, 8 * qd + 4) + w2.w * __shfl_sync(kFull, yb, 8 * qd + 6);
    }
    const float w3 = s.w3[lane];
    float ta = w3 * clamp01(sa), tb = w3 * clamp01(sb);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ta += __shfl_xor_sync(kFull, ta, o);
      tb += __shfl_xor_sync(kFull, tb, o);
    }
    if (lane == 0) {
      a.out[qa] = s.b3 + ta;
      if (two) a.out[qb] = s.b3 + tb;
    }
  }
  // the w1 copy lands before the CTA ends (also when no warp waited for it)
  if (threadIdx.x == 0) pipe::mbar_wait_drain(&s.bar, 0, &a.hdr->status);
}

}  // namespace f
}  // namespace cnnue

using namespace cnnue;
using namespace cnnue::f;

struct cnnue_f_model {
  int device = 0;
  DevWeights w{};
  void* blob = nullptr;
  int sms = 148;
  int ctas_per_sm = 1;  // resident f_fused_kernel CTAs per SM (cooperative grid bound)
};

extern "C" {

int cnnue_f_model_create(const cnnue_f_weights* w, int device, cnnue_f_model** out) {
  if (!w || !out) return set_error(CNNUE_ERR_INVALID_ARG, "null weights or out");
  if (!w->ft_weight || !w->ft_bias || !w->l1_weight || !w->l1_bias || !w->l2_weight ||
      !w->l2_bias || !w->l3_weight || !w->l3_bias)
    return set_error(CNNUE_ERR_INVALID_ARG, "a weight pointer is null");
  *out = nullptr;
  int n_dev = 0;
  if (cudaGetDeviceCount(&n_dev) != cudaSuccess || n_dev == 0)
    return set_error(CNNUE_ERR_NO_DEVICE, "no CUDA device");
  if (device < 0 || device >= n_dev)
    return set_error(CNNUE_ERR_NO_DEVICE, "device %d out of range", device);
  DeviceGuard guard(device);
  if (guard.status) return guard.status;
  const size_t sizes[8] = {(size_t)kF * kCols * 4, kCols * 4, (size_t)kNB * 16 * kIn * 4,
                           kNB * 16 * 4, kNB * 32 * 16 * 4, kNB * 32 * 4, kNB * 32 * 4, kNB * 4};
  const void* srcs[8] = {w->ft_weight, w->ft_bias, w->l1_weight, w->l1_bias,
                         w->l2_weight, w->l2_bias, w->l3_weight, w->l3_bias};
  size_t offs[8], total = 0;
  for (int i = 0; i < 8; ++i) {
    offs[i] = total;
    total += align_up(sizes[i], 256);
  }
  auto* m = new cnnue_f_model();
  m->device = device;
  cudaError_t e = cudaMalloc(&m->blob, total);
  if (e != cudaSuccess) {
    delete m;
    return cuda_error(e, "cudaMalloc(weights)");
  }
  for (int i = 0; i < 8; ++i) {
    e = cudaMemcpy((char*)m->blob + offs[i], srcs[i], sizes[i], cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      cudaFree(m->blob);
      delete m;
      return cuda_error(e, "cudaMemcpy(weights)");
    }
  }
  const float** dst[8] = {&m->w.ft, &m->w.bias, &m->w.l1w, &m->w.l1b,
                          &m->w.l2w, &m->w.l2b, &m->w.l3w, &m->w.l3b};
  for (int i = 0; i < 8; ++i) *dst[i] = (const float*)((char*)m->blob + offs[i]);
  cudaDeviceGetAttribute(&m->sms, cudaDevAttrMultiProcessorCount, device);
  e = cudaFuncSetAttribute(f_fused_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&m->ctas_per_sm, f_fused_kernel, kWarps * 32, 0);
  if (e != cudaSuccess || m->ctas_per_sm < 1) {
    cudaFree(m->blob);
    delete m;
    return e != cudaSuccess ? cuda_error(e, "occupancy of f_fused_kernel")
                            : set_error(CNNUE_ERR_CUDA, "f_fused_kernel does not fit on an SM");
  }
  *out = m;
  return CNNUE_OK;
}

int cnnue_f_model_destroy(cnnue_f_model* m) {
  if (!m) return CNNUE_OK;
  DeviceGuard guard(m->device);
  if (m->blob) cudaFree(m->blob);
  delete m;
  return CNNUE_OK;
}

size_t cnnue_f_workspace_bytes(int64_t n_positions) {
  const size_t n = (size_t)std::max<int64_t>(n_positions, 1);
  return sizeof(WorkspaceHeader) + align_up(n * kIn * 4, 256) + align_up(n * kNB * 4, 256);
}

int cnnue_f_forward(const cnnue_f_model* m, const uint16_t* d_idx, uint32_t n_idx,
                    const uint32_t* d_offsets, int64_t n, float* d_out, void* ws, size_t ws_bytes,
                    void* stream) {
  if (!m) return set_error(CNNUE_ERR_INVALID_ARG, "model is null");
  if (n < 0 || n > (int64_t)INT32_MAX) return set_error(CNNUE_ERR_INVALID_ARG, "bad n_positions");
  if (n == 0) return CNNUE_OK;
  if (!d_offsets || !d_out || (n_idx && !d_idx) || !ws)
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer");
  if (ws_bytes < cnnue_f_workspace_bytes(n))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu < %zu", ws_bytes, cnnue_f_workspace_bytes(n));
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  CNNUE_CUDA_TRY(cudaMemsetAsync(ws, 0, sizeof(WorkspaceHeader), s));
  Args a{};
  a.w = m->w;
  a.idx = d_idx;
  a.n_idx = n_idx;
  a.offsets = d_offsets;
  a.x = (float*)((char*)ws + sizeof(WorkspaceHeader));
  a.blist = (uint32_t*)((char*)a.x + align_up((size_t)n * kIn * 4, 256));
  a.out = d_out;
  a.n = (uint32_t)n;
  a.hdr = (Header*)ws;
  // a multiple of 8 CTAs (every bucket the same number of phase-2 CTAs), all
  // resident: one warp per list at most
  const int64_t cap = (int64_t)m->sms * m->ctas_per_sm / kNB * kNB;
  const int64_t want = ((2 * n + kWarps - 1) / kWarps + kNB - 1) / kNB * kNB;
  const unsigned grid = (unsigned)std::max<int64_t>(kNB, std::min(cap, want));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, f_fused_kernel, a);
  if (e != cudaSuccess) return cuda_error(e, "cudaLaunchKernelEx(f_fused_kernel, cooperative)");
  return check_launch_error("f_fused_kernel");
}

}  // extern "C"
