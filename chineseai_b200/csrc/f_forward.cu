// f_forward.cu - fp32 HalfKA NNUE evaluation on sm_100a.
//
// Same shape as the quantised evaluator: one group of 128 threads per
// position, warps 0-1 on perspective 0 and 2-3 on perspective 1; thread c of a
// perspective owns FT columns [4c, 4c+4) (one 16-byte load per 1 KB row).
// Each column is summed bias-first in index order with plain fp32 adds, which
// is the order of the scalar evaluator, so the FT output is bit-identical to
// it; the stack's dot products use a fixed warp-tree order instead.
// Positions are walked in bucket order so the bucket's 16x512 L1 weights stay
// in registers (16 float4 per thread).
#include <algorithm>

#include "common.cuh"

namespace cnnue {
namespace f {

constexpr int kF = CNNUE_F_FEATURES;
constexpr int kCols = CNNUE_F_COLS;
constexpr int kRowBytes = kCols * 4;
constexpr int kNB = CNNUE_F_BUCKETS;
constexpr int kIn = 2 * kCols;
constexpr int kGroup = 128;
constexpr int kGroupsPerCta = 2;
constexpr int kCta = kGroup * kGroupsPerCta;
constexpr int kUnroll = 8;
constexpr unsigned kFull = 0xffffffffu;

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
  float* out;
  int64_t n;
  const uint32_t* perm;
  const uint8_t* sorted_bucket;
  uint32_t* status;
};

__device__ __forceinline__ void add4(float4& a, const float4& b) {
  a.x += b.x;
  a.y += b.y;
  a.z += b.z;
  a.w += b.w;
}

__device__ __forceinline__ float clamp01(float v) { return fminf(fmaxf(v, 0.f), 1.f); }

__global__ void __launch_bounds__(kCta, 2) f_eval_kernel(const Args a) {
  __shared__ float red[kGroupsPerCta][2][4][16];
  __shared__ __align__(16) float h1s[kGroupsPerCta][16];

  const int g = threadIdx.x / kGroup;
  const int t = threadIdx.x % kGroup;
  const int warp = t >> 5, lane = t & 31;
  const int persp = t >> 6;
  const int c = t & 63;

  const int64_t n_groups = (int64_t)gridDim.x * kGroupsPerCta;
  const int64_t gid = (int64_t)blockIdx.x * kGroupsPerCta + g;
  const int64_t begin = a.n * gid / n_groups;
  const int64_t end = a.n * (gid + 1) / n_groups;

  const char* ftc = (const char*)a.w.ft + c * 16;
  const float4 bias = __ldg((const float4*)(a.w.bias + 4 * c));

  int cur_bucket = -1;
  float4 w1[16];
  float4 w2[4];
  float b1v = 0.f, b2v = 0.f, w3v = 0.f, b3v = 0.f;
  int parity = 0;

  for (int64_t i = begin; i < end; ++i) {
    const uint32_t pos = a.perm[i];
    const int bucket = a.sorted_bucket[i];
    if (bucket != cur_bucket) {
      cur_bucket = bucket;
      const float* w1p = a.w.l1w + (size_t)bucket * 16 * kIn + persp * kCols + 4 * c;
#pragma unroll
      for (int k = 0; k < 16; ++k) w1[k] = __ldg((const float4*)(w1p + (size_t)k * kIn));
      const float* w2p = a.w.l2w + ((size_t)bucket * 32 + lane) * 16;
#pragma unroll
      for (int q = 0; q < 4; ++q) w2[q] = __ldg((const float4*)(w2p + 4 * q));
      b2v = __ldg(a.w.l2b + bucket * 32 + lane);
      w3v = __ldg(a.w.l3w + bucket * 32 + lane);
      b1v = lane < 16 ? __ldg(a.w.l1b + bucket * 16 + lane) : 0.f;
      b3v = __ldg(a.w.l3b + bucket);
    }

    const int64_t ps = 2 * (int64_t)pos + persp;
    float4 acc = bias;
    const uint32_t ob = min(a.offsets[ps], a.n_idx);
    const uint32_t oe = min(max(a.offsets[ps + 1], ob), a.n_idx);
    for (uint32_t base = ob; base < oe; base += 32) {
      const int cnt = (int)min(32u, oe - base);
      uint32_t my = lane < cnt ? (uint32_t)a.idx[base + lane] : 0u;
      const bool bad = lane < cnt && my >= (uint32_t)kF;
      if (__any_sync(kFull, bad)) {
        if (bad) atomicOr(a.status, CNNUE_STATUS_BAD_INDEX);
      }
      if (bad) my = 0xffffffffu;
      for (int r0 = 0; r0 < cnt; r0 += kUnroll) {
        float4 v[kUnroll];
        bool ok[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const uint32_t f = __shfl_sync(kFull, my, r0 + u);
          ok[u] = r0 + u < cnt && f != 0xffffffffu;
          if (ok[u]) v[u] = ldg_stream16f(ftc + (size_t)f * kRowBytes);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          if (ok[u]) add4(acc, v[u]);
      }
    }

    const float x0 = clamp01(acc.x), x1 = clamp01(acc.y), x2 = clamp01(acc.z), x3 = clamp01(acc.w);
    float v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = w1[k].x * x0 + w1[k].y * x1 + w1[k].z * x2 + w1[k].w * x3;
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
    if ((lane & 1) == 0) red[g][parity][warp][lane >> 1] = v[0];
    named_bar_sync(1 + g, kGroup);

    if (warp == 0) {
      if (lane < 16) {
        const float s = b1v + red[g][parity][0][lane] + red[g][parity][1][lane] +
                        red[g][parity][2][lane] + red[g][parity][3][lane];
        h1s[g][lane] = clamp01(s);
      }
      __syncwarp();
      float s2 = b2v;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 h = *(const float4*)&h1s[g][4 * q];
        s2 += w2[q].x * h.x + w2[q].y * h.y + w2[q].z * h.z + w2[q].w * h.w;
      }
      float s3 = w3v * clamp01(s2);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s3 += __shfl_xor_sync(kFull, s3, o);
      if (lane == 0) a.out[pos] = b3v + s3;
      __syncwarp();
    }
    parity ^= 1;
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
  int grid = 0;
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
  int sms = 0, occ = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, f_eval_kernel, kCta, 0);
  m->grid = sms * std::max(occ, 1);
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

int cnnue_f_forward(const cnnue_f_model* m, const uint16_t* d_idx, uint32_t n_idx,
                    const uint32_t* d_offsets, int64_t n, float* d_out, void* ws, size_t ws_bytes,
                    void* stream) {
  if (!m) return set_error(CNNUE_ERR_INVALID_ARG, "model is null");
  if (n < 0 || n > (int64_t)INT32_MAX) return set_error(CNNUE_ERR_INVALID_ARG, "bad n_positions");
  if (n == 0) return CNNUE_OK;
  if (!d_offsets || !d_out || (n_idx && !d_idx) || !ws)
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer");
  if (ws_bytes < bucket_workspace_bytes(n))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu < %zu", ws_bytes, bucket_workspace_bytes(n));
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  int st = launch_bucket_sort(d_offsets, n_idx, nullptr, n, 2, kNB, ws, s);
  if (st) return st;
  WorkspaceView v = carve_workspace(ws, n);
  Args a{};
  a.w = m->w;
  a.idx = d_idx;
  a.n_idx = n_idx;
  a.offsets = d_offsets;
  a.out = d_out;
  a.n = n;
  a.perm = v.perm;
  a.sorted_bucket = v.sorted_bucket;
  a.status = &v.hdr->status;
  const int grid = (int)std::min<int64_t>(m->grid, (n + kGroupsPerCta - 1) / kGroupsPerCta);
  f_eval_kernel<<<grid, kCta, 0, s>>>(a);
  return check_launch_error("f_eval_kernel");
}

}  // extern "C"
