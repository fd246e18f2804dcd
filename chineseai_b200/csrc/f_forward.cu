// f_forward.cu - fp32 HalfKA NNUE evaluation on sm_100a.
//
// Two launches per batch (after the status word is cleared; the second is a
// programmatic dependent launch that stages its weights during the first's tail):
//   1. f_gather_kernel (which also checks every list's offsets: monotone,
//      within the index array): one warp per (position, perspective) list, lane l
//      owning FT columns [4l, 4l + 4) and [128 + 4l, 128 + 4l + 4) (two
//      16-byte loads per 1 KB row, each load instruction covering 512
//      contiguous bytes, rows eight at a time in flight).  Each column is summed bias-first in
//      index order with plain fp32 adds - the order of the scalar evaluator -
//      so the FT output is bit-identical to it; the clipped values go to the
//      workspace as x [n][512] (perspective 0, then 1);
//   2. f_stack_kernel: CTA (bucket b, part j) keeps bucket b's 16x512 L1
//      weights in shared memory and evaluates the positions of bucket b
//      (bucket = min((max(n0, 1) - 1) >> 2, 7) from the perspective-0 count)
//      in its contiguous share (offsets read 32 positions at a time, the
//      bucket's positions picked by ballot), one warp per position: L1 by lanes over the 512
//      inputs and a 16-way warp reduce-scatter, L2 by lanes over its 32
//      outputs, L3 by a warp sum (a fixed order, within 1e-4 of the scalar
//      one).  No bucket sort: every part of every bucket scans the batch's
//      offsets (4 bytes x 2 per position).
#include <algorithm>

#include "common.cuh"

namespace cnnue {
namespace f {

constexpr int kF = CNNUE_F_FEATURES;
constexpr int kCols = CNNUE_F_COLS;
constexpr int kRowBytes = kCols * 4;
constexpr int kNB = CNNUE_F_BUCKETS;
constexpr int kIn = 2 * kCols;
constexpr int kUnroll = 8;
constexpr int kWarps = 8;  // warps per CTA in both kernels
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

struct Args {
  DevWeights w;
  const uint16_t* idx;
  uint32_t n_idx;
  const uint32_t* offsets;
  float* x;  // [n][512] clipped FT outputs (workspace)
  float* out;
  int64_t n;
  uint32_t* status;
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

__global__ void __launch_bounds__(kWarps * 32) f_gather_kernel(const Args a) {
  // the stack kernel may be scheduled now: it stages its weights, then waits
  // for this grid to complete before reading x
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * kWarps;
  const char* ft = (const char*)a.w.ft + lane * 16;
  const float4 bias0 = __ldg((const float4*)(a.w.bias + 4 * lane));
  const float4 bias1 = __ldg((const float4*)(a.w.bias + 128 + 4 * lane));
  for (int64_t l = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); l < 2 * a.n; l += warps) {
    const uint32_t o0 = a.offsets[l], o1 = a.offsets[l + 1];
    if (lane == 0 && !(o0 <= o1 && o1 <= a.n_idx)) atomicOr(a.status, CNNUE_STATUS_BAD_OFFSETS);
    const uint32_t ob = min(o0, a.n_idx);
    const uint32_t oe = min(max(o1, ob), a.n_idx);
    float4 acc0 = bias0, acc1 = bias1;
    for (uint32_t base = ob; base < oe; base += 32) {
      const int cnt = (int)min(32u, oe - base);
      uint32_t my = lane < cnt ? (uint32_t)a.idx[base + lane] : 0u;
      const bool bad = lane < cnt && my >= (uint32_t)kF;
      if (bad) {
        atomicOr(a.status, CNNUE_STATUS_BAD_INDEX);
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
    float* xo = a.x + (l >> 1) * kIn + (l & 1) * kCols + 4 * lane;
    *(float4*)xo = clamp01(acc0);
    *(float4*)(xo + 128) = clamp01(acc1);
  }
}

__global__ void __launch_bounds__(kWarps * 32) f_stack_kernel(const Args a) {
  __shared__ __align__(16) float w1s[16 * kIn];  // this CTA's bucket: 32 KB
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.x % kNB;
  const int part = blockIdx.x / kNB, parts = gridDim.x / kNB;
  const float4* w1g = (const float4*)(a.w.l1w + (size_t)b * 16 * kIn);
  for (int i = threadIdx.x; i < 16 * kIn / 4; i += kWarps * 32) ((float4*)w1s)[i] = __ldg(w1g + i);
  const float b1v = __ldg(a.w.l1b + b * 16 + (lane >> 1));
  float4 w2[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) w2[q] = __ldg((const float4*)(a.w.l2w + ((size_t)b * 32 + lane) * 16) + q);
  const float b2v = __ldg(a.w.l2b + b * 32 + lane), w3v = __ldg(a.w.l3w + b * 32 + lane), b3v = __ldg(a.w.l3b + b);
  __syncthreads();
  // launched as a programmatic dependent of f_gather_kernel: x is complete
  // (and visible) only after this wait
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // this warp's contiguous share of the batch, scanned 32 positions at a time
  const int64_t wid = (int64_t)part * kWarps + warp, nw = (int64_t)parts * kWarps;
  const int64_t p_begin = a.n * wid / nw, p_end = a.n * (wid + 1) / nw;
  for (int64_t c0 = p_begin; c0 < p_end; c0 += 32) {
    const int64_t q = c0 + lane;
    bool mine = false;
    if (q < p_end) {
      const uint32_t ob = min(a.offsets[2 * q], a.n_idx);
      const uint32_t oe = min(max(a.offsets[2 * q + 1], ob), a.n_idx);
      mine = (int)min((max(oe - ob, 1u) - 1u) >> 2, (uint32_t)(kNB - 1)) == b;
    }
    uint32_t todo = __ballot_sync(kFull, mine);
    while (todo) {
      const int src = __ffs(todo) - 1;
      todo &= todo - 1;
      const int64_t p = c0 + src;
    const float* xp = a.x + p * kIn;
    float xv[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) xv[i] = xp[lane + 32 * i];
    float v[16];
#pragma unroll
    for (int o = 0; o < 16; ++o) {
      float sacc = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) sacc += w1s[o * kIn + lane + 32 * i] * xv[i];
      v[o] = sacc;
    }
    // 16 outputs reduced over the 32 lanes: output o ends on lanes 2o, 2o+1
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
    const float y1 = clamp01(b1v + v[0]);  // output lane >> 1 (both lanes of the pair)
    float s2 = b2v;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      s2 += w2[q].x * __shfl_sync(kFull, y1, 8 * q) + w2[q].y * __shfl_sync(kFull, y1, 8 * q + 2) +
            w2[q].z * __shfl_sync(kFull, y1, 8 * q + 4) + w2[q].w * __shfl_sync(kFull, y1, 8 * q + 6);
    }
    float s3 = w3v * clamp01(s2);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s3 += __shfl_xor_sync(kFull, s3, o);
    if (lane == 0) a.out[p] = b3v + s3;
    }
  }
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
  return sizeof(WorkspaceHeader) + align_up((size_t)std::max<int64_t>(n_positions, 1) * kIn * 4, 256);
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
  a.out = d_out;
  a.n = n;
  a.status = &((WorkspaceHeader*)ws)->status;
  const int64_t lists = 2 * n;
  const unsigned g1 = (unsigned)std::max<int64_t>(1, std::min<int64_t>((lists + kWarps - 1) / kWarps,
                                                                        (int64_t)m->sms * 16));
  f_gather_kernel<<<g1, kWarps * 32, 0, s>>>(a);
  if (int e = check_launch_error("f_gather_kernel")) return e;
  // parts per bucket: about 4 positions per warp, at most 4 CTAs per SM overall
  const int64_t parts = std::max<int64_t>(1, std::min<int64_t>((n + kNB * kWarps * 4 - 1) / (kNB * kWarps * 4),
                                                              (int64_t)m->sms * 4 / kNB));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(kNB * parts));
  cfg.blockDim = dim3(kWarps * 32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, f_stack_kernel, a);
  if (e != cudaSuccess) return cuda_error(e, "cudaLaunchKernelEx(f_stack_kernel)");
  return check_launch_error("f_stack_kernel");
}

}  // extern "C"
