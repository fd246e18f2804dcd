// q_forward.cu - quantised HalfKA NNUE evaluation on sm_100a.
//
// Work per position: two perspectives x (bias + ~17 gathered int16 rows of
// 2 KB), the pairwise clipped-ReLU pack to 1024 uint8, then the bucket's int8
// stack 1024->16->32->1.  The gather dominates (69.6 KB of rows per position
// against 16 K int8 MACs), so the kernel is built around memory-level
// parallelism on the FT rows:
//
//   * one group of 128 threads (4 warps) evaluates one position; warps 0-1
//     take perspective 0, warps 2-3 perspective 1.  Thread c of a perspective
//     owns FT columns [8c, 8c+8) and [512+8c, 512+8c+8): two 16-byte loads per
//     row, and exactly the two halves its pack needs, so the pack is local;
//   * rows are streamed with ld.global.nc.L1::no_allocate, kUnroll rows (2 x
//     kUnroll 16-byte loads per thread) in flight before the adds;
//   * int16 wraparound is __vadd2/__vsub2 on packed halfword pairs;
//   * positions are first grouped by bucket (a two-kernel counting sort), and
//     each group walks a contiguous slice of that order, so the 16 KB of L1
//     weights of the current bucket live in registers (16 x 8 bytes per
//     thread) and are reloaded only when the bucket changes;
//   * L1 = 32 dp4a per thread + a 16-way warp reduce-scatter (16 shuffles) +
//     a 4-warp sum through shared memory (one named barrier per position,
//     double-buffered); warp 0 then runs L2/L3 while warps 1-3 move on.
#include <algorithm>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace cnnue {
namespace q {

constexpr int kF = CNNUE_Q_FEATURES;
constexpr int kCols = CNNUE_Q_COLS;
constexpr int kRowBytes = kCols * 2;
constexpr int kNB = CNNUE_Q_BUCKETS;
constexpr int kL1 = CNNUE_Q_L1;
constexpr int kL2 = CNNUE_Q_L2;
constexpr int kGroup = 128;
constexpr int kGroupsPerCta = 2;
constexpr int kCta = kGroup * kGroupsPerCta;
constexpr int kUnroll = 8;
constexpr int kMinBlocks = 2;
constexpr unsigned kFull = 0xffffffffu;

struct DevWeights {
  const int16_t* ft;
  const int16_t* bias;
  const int8_t* l1w;
  const int32_t* l1b;
  const int8_t* l2w;
  const int32_t* l2b;
  const int8_t* l3w;
  const int32_t* l3b;
};

// ---------------------------------------------------------------------------
// Stage 3: fused gather + pack + bucket stack.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 vadd(uint4 a, uint4 b) {
  return make_uint4(__vadd2(a.x, b.x), __vadd2(a.y, b.y), __vadd2(a.z, b.z), __vadd2(a.w, b.w));
}
__device__ __forceinline__ uint4 vsub(uint4 a, uint4 b) {
  return make_uint4(__vsub2(a.x, b.x), __vsub2(a.y, b.y), __vsub2(a.z, b.z), __vsub2(a.w, b.w));
}

// Two packed outputs from one int16 pair of the low half and the matching
// pair of the high half: (clamp(a,0,127) * clamp(b,0,127)) >> 7 per lane.
__device__ __forceinline__ uint32_t pack_pair(uint32_t lo, uint32_t hi) {
  const uint32_t a = __vmaxs2(__vmins2(lo, 0x007f007fu), 0u);
  const uint32_t b = __vmaxs2(__vmins2(hi, 0x007f007fu), 0u);
  const uint32_t p0 = ((a & 0xffffu) * (b & 0xffffu)) >> 7;
  const uint32_t p1 = ((a >> 16) * (b >> 16)) >> 7;
  return p0 | (p1 << 8);
}

// Adds (kSub: subtracts) the rows listed in idx[begin, end) to this thread's
// two 16-byte column chunks.  `ftc` points at the thread's low chunk of row 0.
template <bool kSub>
__device__ __forceinline__ void gather_rows(const char* __restrict__ ftc,
                                            const uint16_t* __restrict__ idx, uint32_t begin,
                                            uint32_t end, uint4& alo, uint4& ahi, int lane,
                                            uint32_t* status) {
  for (uint32_t base = begin; base < end; base += 32) {
    const int cnt = (int)min(32u, end - base);
    uint32_t my = lane < cnt ? (uint32_t)idx[base + lane] : 0u;
    const bool bad = lane < cnt && my >= (uint32_t)kF;
    if (__any_sync(kFull, bad)) {
      if (bad) atomicOr(status, CNNUE_STATUS_BAD_INDEX);
    }
    if (bad) my = 0xffffffffu;
    for (int r0 = 0; r0 < cnt; r0 += kUnroll) {
      uint4 vlo[kUnroll], vhi[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const uint32_t f = __shfl_sync(kFull, my, r0 + u);
        if (r0 + u < cnt && f != 0xffffffffu) {
          const char* row = ftc + (size_t)f * kRowBytes;
          vlo[u] = ldg_stream16(row);
          vhi[u] = ldg_stream16(row + kRowBytes / 2);
        } else {
          vlo[u] = make_uint4(0, 0, 0, 0);
          vhi[u] = make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (kSub) {
          alo = vsub(alo, vlo[u]);
          ahi = vsub(ahi, vhi[u]);
        } else {
          alo = vadd(alo, vlo[u]);
          ahi = vadd(ahi, vhi[u]);
        }
      }
    }
  }
}

struct ForwardArgs {
  DevWeights w;
  const uint16_t* idx;        // forward: active lists; update: added lists
  uint32_t n_idx;
  const uint32_t* offsets;    // [2n+1]
  const uint16_t* rem;        // update only
  uint32_t n_rem;
  const uint32_t* rem_offsets;
  const int16_t* parent;      // update only, [n][2][1024]
  const uint8_t* flags;       // update only, [2n]
  int16_t* acc_out;           // [n][2][1024] or null
  int32_t* scores;
  int64_t n;
  const uint32_t* perm;
  const uint8_t* sorted_bucket;
  uint32_t* status;
};

template <bool kUpdate, bool kWriteAcc>
__global__ void __launch_bounds__(kCta, kMinBlocks) q_eval_kernel(const ForwardArgs a) {
  __shared__ int32_t red[kGroupsPerCta][2][4][16];
  __shared__ __align__(16) uint8_t y1s[kGroupsPerCta][16];

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
  const uint4 bias_lo = __ldg((const uint4*)((const char*)a.w.bias + c * 16));
  const uint4 bias_hi = __ldg((const uint4*)((const char*)a.w.bias + kRowBytes / 2 + c * 16));

  int cur_bucket = -1;
  uint2 w1[kL1];
  uint4 w2row = make_uint4(0, 0, 0, 0);
  int32_t b1v = 0, b2v = 0, w3v = 0, b3v = 0;
  int parity = 0;

  for (int64_t i = begin; i < end; ++i) {
    const uint32_t pos = a.perm[i];
    const int bucket = a.sorted_bucket[i];
    if (bucket != cur_bucket) {
      cur_bucket = bucket;
      const int8_t* w1p = a.w.l1w + (size_t)bucket * kL1 * kCols + persp * (kCols / 2) + 8 * c;
#pragma unroll
      for (int k = 0; k < kL1; ++k) w1[k] = __ldg((const uint2*)(w1p + (size_t)k * kCols));
      w2row = __ldg((const uint4*)(a.w.l2w + ((size_t)bucket * kL2 + lane) * kL1));
      b2v = __ldg(a.w.l2b + bucket * kL2 + lane);
      w3v = __ldg(a.w.l3w + bucket * kL2 + lane);
      b1v = lane < kL1 ? __ldg(a.w.l1b + bucket * kL1 + lane) : 0;
      b3v = __ldg(a.w.l3b + bucket);
    }

    // ---- accumulator of this thread's columns --------------------------------
    const int64_t ps = 2 * (int64_t)pos + persp;
    uint4 alo, ahi;
    if (kUpdate) {
      const bool refresh = (a.flags[ps] & 1) != 0;
      if (refresh) {
        alo = bias_lo;
        ahi = bias_hi;
      } else {
        const char* par = (const char*)(a.parent + ps * kCols) + c * 16;
        alo = __ldg((const uint4*)par);
        ahi = __ldg((const uint4*)(par + kRowBytes / 2));
        const uint32_t rb = min(a.rem_offsets[ps], a.n_rem);
        const uint32_t re = min(max(a.rem_offsets[ps + 1], rb), a.n_rem);
        gather_rows<true>(ftc, a.rem, rb, re, alo, ahi, lane, a.status);
      }
    } else {
      alo = bias_lo;
      ahi = bias_hi;
    }
    {
      const uint32_t ob = min(a.offsets[ps], a.n_idx);
      const uint32_t oe = min(max(a.offsets[ps + 1], ob), a.n_idx);
      gather_rows<false>(ftc, a.idx, ob, oe, alo, ahi, lane, a.status);
    }
    if (kWriteAcc) {
      char* out = (char*)(a.acc_out + ps * kCols) + c * 16;
      *(uint4*)out = alo;
      *(uint4*)(out + kRowBytes / 2) = ahi;
    }

    // ---- pack + L1 partial sums ----------------------------------------------
    const uint32_t x0 = pack_pair(alo.x, ahi.x) | (pack_pair(alo.y, ahi.y) << 16);
    const uint32_t x1 = pack_pair(alo.z, ahi.z) | (pack_pair(alo.w, ahi.w) << 16);
    int32_t v[kL1];
#pragma unroll
    for (int k = 0; k < kL1; ++k) v[k] = __dp4a((int)x1, (int)w1[k].y, __dp4a((int)x0, (int)w1[k].x, 0));

    // Reduce-scatter of the 16 sums over the warp: afterwards lane l holds
    // the warp total of output k = l >> 1.
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const bool up = lane & 16;
      const int32_t send = up ? v[j] : v[j + 8];
      const int32_t keep = up ? v[j + 8] : v[j];
      v[j] = keep + __shfl_xor_sync(kFull, send, 16);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool up = lane & 8;
      const int32_t send = up ? v[j] : v[j + 4];
      const int32_t keep = up ? v[j + 4] : v[j];
      v[j] = keep + __shfl_xor_sync(kFull, send, 8);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const bool up = lane & 4;
      const int32_t send = up ? v[j] : v[j + 2];
      const int32_t keep = up ? v[j + 2] : v[j];
      v[j] = keep + __shfl_xor_sync(kFull, send, 4);
    }
    {
      const bool up = lane & 2;
      const int32_t send = up ? v[0] : v[1];
      const int32_t keep = up ? v[1] : v[0];
      v[0] = keep + __shfl_xor_sync(kFull, send, 2);
    }
    v[0] += __shfl_xor_sync(kFull, v[0], 1);
    if ((lane & 1) == 0) red[g][parity][warp][lane >> 1] = v[0];
    named_bar_sync(1 + g, kGroup);

    // ---- L1 epilogue, L2, L3 on warp 0 -------------------------------------
    if (warp == 0) {
      if (lane < kL1) {
        const int32_t s = b1v + red[g][parity][0][lane] + red[g][parity][1][lane] +
                          red[g][parity][2][lane] + red[g][parity][3][lane];
        y1s[g][lane] = (uint8_t)min(max(s >> 6, 0), 127);
      }
      __syncwarp();
      const uint4 y = *(const uint4*)y1s[g];
      int32_t s2 = b2v;
      s2 = __dp4a((int)y.x, (int)w2row.x, s2);
      s2 = __dp4a((int)y.y, (int)w2row.y, s2);
      s2 = __dp4a((int)y.z, (int)w2row.z, s2);
      s2 = __dp4a((int)y.w, (int)w2row.w, s2);
      const int32_t y2 = min(max(s2 >> 6, 0), 127);
      int32_t s3 = (int32_t)(int8_t)w3v * y2;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s3 += __shfl_xor_sync(kFull, s3, o);
      if (lane == 0) a.scores[pos] = b3v + s3;
      __syncwarp();
    }
    parity ^= 1;
  }
}

}  // namespace q
}  // namespace cnnue

// ===========================================================================
// Host side
// ===========================================================================
using namespace cnnue;
using namespace cnnue::q;

struct cnnue_q_model {
  int device = 0;
  DevWeights w{};
  void* blob = nullptr;
  int sm_count = 0;
  int grid_eval = 0;
  int grid_update = 0;
  // Staging for cnnue_q_forward_host.
  void* stage = nullptr;
  size_t stage_bytes = 0;
};

namespace {

int check_launch(const char* what) { return check_launch_error(what); }

int validate_common(const cnnue_q_model* m, int64_t n, void* ws, size_t ws_bytes) {
  if (!m) return set_error(CNNUE_ERR_INVALID_ARG, "model is null");
  if (n < 0 || n > (int64_t)INT32_MAX)
    return set_error(CNNUE_ERR_INVALID_ARG, "n_positions %lld out of range", (long long)n);
  if (n > 0 && !ws) return set_error(CNNUE_ERR_INVALID_ARG, "workspace is null");
  if (n > 0 && ws_bytes < bucket_workspace_bytes(n))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu bytes < %zu required", ws_bytes,
                     bucket_workspace_bytes(n));
  return CNNUE_OK;
}

int launch_sort(const cnnue_q_model* m, const uint32_t* d_offsets, uint32_t n_indices,
                const uint8_t* d_count0, int64_t n, void* ws, cudaStream_t s) {
  (void)m;
  return launch_bucket_sort(d_offsets, n_indices, d_count0, n, 1, kNB, ws, s);
}

int launch_eval(const cnnue_q_model* m, const uint16_t* d_idx, uint32_t n_idx,
                const uint32_t* d_offsets, int64_t n, int32_t* d_scores, int16_t* d_acc, void* ws,
                cudaStream_t s) {
  WorkspaceView v = carve_workspace(ws, n);
  ForwardArgs a{};
  a.w = m->w;
  a.idx = d_idx;
  a.n_idx = n_idx;
  a.offsets = d_offsets;
  a.acc_out = d_acc;
  a.scores = d_scores;
  a.n = n;
  a.perm = v.perm;
  a.sorted_bucket = v.sorted_bucket;
  a.status = &v.hdr->status;
  const int grid = (int)std::min<int64_t>(m->grid_eval, (n + kGroupsPerCta - 1) / kGroupsPerCta);
  if (d_acc)
    q_eval_kernel<false, true><<<grid, kCta, 0, s>>>(a);
  else
    q_eval_kernel<false, false><<<grid, kCta, 0, s>>>(a);
  return check_launch("q_eval_kernel");
}

int check_indices_args(const void* idx, uint32_t n_idx, const void* offsets, const void* out,
                       int64_t n) {
  if (n == 0) return CNNUE_OK;
  if (!offsets || !out) return set_error(CNNUE_ERR_INVALID_ARG, "null offsets or output");
  if (n_idx > 0 && !idx) return set_error(CNNUE_ERR_INVALID_ARG, "null indices");
  return CNNUE_OK;
}

}  // namespace

extern "C" {

int cnnue_q_model_create(const cnnue_q_weights* w, int device, cnnue_q_model** out) {
  if (!w || !out) return set_error(CNNUE_ERR_INVALID_ARG, "null weights or out");
  if (!w->ft_weight || !w->ft_bias || !w->l1_weight || !w->l1_bias || !w->l2_weight ||
      !w->l2_bias || !w->l3_weight || !w->l3_bias)
    return set_error(CNNUE_ERR_INVALID_ARG, "a weight pointer is null");
  *out = nullptr;
  int n_dev = 0;
  if (cudaGetDeviceCount(&n_dev) != cudaSuccess || n_dev == 0)
    return set_error(CNNUE_ERR_NO_DEVICE, "no CUDA device");
  if (device < 0 || device >= n_dev)
    return set_error(CNNUE_ERR_NO_DEVICE, "device %d out of range (%d devices)", device, n_dev);
  DeviceGuard guard(device);
  if (guard.status) return guard.status;

  const size_t sz_ft = (size_t)kF * kCols * 2, sz_bias = kCols * 2;
  const size_t sz_l1w = (size_t)kNB * kL1 * kCols, sz_l1b = kNB * kL1 * 4;
  const size_t sz_l2w = (size_t)kNB * kL2 * kL1, sz_l2b = kNB * kL2 * 4;
  const size_t sz_l3w = kNB * kL2, sz_l3b = kNB * 4;
  const size_t sizes[8] = {sz_ft, sz_bias, sz_l1w, sz_l1b, sz_l2w, sz_l2b, sz_l3w, sz_l3b};
  const void* srcs[8] = {w->ft_weight, w->ft_bias, w->l1_weight, w->l1_bias,
                         w->l2_weight, w->l2_bias, w->l3_weight, w->l3_bias};
  size_t offs[8], total = 0;
  for (int i = 0; i < 8; ++i) {
    offs[i] = total;
    total += align_up(sizes[i], 256);
  }
  auto* m = new cnnue_q_model();
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
  char* b = (char*)m->blob;
  m->w.ft = (const int16_t*)(b + offs[0]);
  m->w.bias = (const int16_t*)(b + offs[1]);
  m->w.l1w = (const int8_t*)(b + offs[2]);
  m->w.l1b = (const int32_t*)(b + offs[3]);
  m->w.l2w = (const int8_t*)(b + offs[4]);
  m->w.l2b = (const int32_t*)(b + offs[5]);
  m->w.l3w = (const int8_t*)(b + offs[6]);
  m->w.l3b = (const int32_t*)(b + offs[7]);

  cudaDeviceGetAttribute(&m->sm_count, cudaDevAttrMultiProcessorCount, device);
  int occ_eval = 0, occ_upd = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_eval, q_eval_kernel<false, false>, kCta, 0);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_upd, q_eval_kernel<true, true>, kCta, 0);
  m->grid_eval = m->sm_count * std::max(occ_eval, 1);
  m->grid_update = m->sm_count * std::max(occ_upd, 1);
  *out = m;
  return CNNUE_OK;
}

int cnnue_q_model_destroy(cnnue_q_model* m) {
  if (!m) return CNNUE_OK;
  DeviceGuard guard(m->device);
  if (m->blob) cudaFree(m->blob);
  if (m->stage) cudaFree(m->stage);
  delete m;
  return CNNUE_OK;
}

size_t cnnue_q_workspace_bytes(int64_t n_positions) { return bucket_workspace_bytes(n_positions); }

int cnnue_q_bucket_sort(const cnnue_q_model* m, const uint32_t* d_offsets, uint32_t n_indices,
                        int64_t n, void* ws, size_t ws_bytes, void* stream) {
  int st = validate_common(m, n, ws, ws_bytes);
  if (st) return st;
  if (n == 0) return CNNUE_OK;
  if (!d_offsets) return set_error(CNNUE_ERR_INVALID_ARG, "null offsets");
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  return launch_sort(m, d_offsets, n_indices, nullptr, n, ws, (cudaStream_t)stream);
}

int cnnue_q_forward_sorted(const cnnue_q_model* m, const uint16_t* d_idx, uint32_t n_idx,
                           const uint32_t* d_offsets, int64_t n, int32_t* d_scores, void* ws,
                           size_t ws_bytes, void* stream) {
  int st = validate_common(m, n, ws, ws_bytes);
  if (st) return st;
  st = check_indices_args(d_idx, n_idx, d_offsets, d_scores, n);
  if (st) return st;
  if (n == 0) return CNNUE_OK;
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  return launch_eval(m, d_idx, n_idx, d_offsets, n, d_scores, nullptr, ws, (cudaStream_t)stream);
}

int cnnue_q_forward_acc(const cnnue_q_model* m, const uint16_t* d_idx, uint32_t n_idx,
                        const uint32_t* d_offsets, int64_t n, int32_t* d_scores, int16_t* d_acc,
                        void* ws, size_t ws_bytes, void* stream) {
  int st = validate_common(m, n, ws, ws_bytes);
  if (st) return st;
  st = check_indices_args(d_idx, n_idx, d_offsets, d_scores, n);
  if (st) return st;
  if (n == 0) return CNNUE_OK;
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  st = launch_sort(m, d_offsets, n_idx, nullptr, n, ws, s);
  if (st) return st;
  return launch_eval(m, d_idx, n_idx, d_offsets, n, d_scores, d_acc, ws, s);
}

int cnnue_q_forward(const cnnue_q_model* m, const uint16_t* d_idx, uint32_t n_idx,
                    const uint32_t* d_offsets, int64_t n, int32_t* d_scores, void* ws,
                    size_t ws_bytes, void* stream) {
  return cnnue_q_forward_acc(m, d_idx, n_idx, d_offsets, n, d_scores, nullptr, ws, ws_bytes,
                             stream);
}

int cnnue_q_forward_host(cnnue_q_model* m, const uint16_t* h_idx, uint32_t n_idx,
                         const uint32_t* h_offsets, int64_t n, int32_t* h_scores, void* stream) {
  if (!m) return set_error(CNNUE_ERR_INVALID_ARG, "model is null");
  if (n < 0 || n > (int64_t)INT32_MAX) return set_error(CNNUE_ERR_INVALID_ARG, "bad n_positions");
  if (n == 0) return CNNUE_OK;
  if (!h_offsets || !h_scores || (n_idx > 0 && !h_idx))
    return set_error(CNNUE_ERR_INVALID_ARG, "null host buffer");
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t b_idx = align_up((size_t)n_idx * 2, 256);
  const size_t b_off = align_up((size_t)(2 * n + 1) * 4, 256);
  const size_t b_sc = align_up((size_t)n * 4, 256);
  const size_t b_ws = align_up(bucket_workspace_bytes(n), 256);
  const size_t need = b_idx + b_off + b_sc + b_ws;
  if (need > m->stage_bytes) {
    if (m->stage) {
      CNNUE_CUDA_TRY(cudaStreamSynchronize(s));
      cudaFree(m->stage);
      m->stage = nullptr;
      m->stage_bytes = 0;
    }
    CNNUE_CUDA_TRY(cudaMalloc(&m->stage, need));
    m->stage_bytes = need;
  }
  char* p = (char*)m->stage;
  uint16_t* d_idx = (uint16_t*)p;
  uint32_t* d_off = (uint32_t*)(p + b_idx);
  int32_t* d_sc = (int32_t*)(p + b_idx + b_off);
  void* ws = p + b_idx + b_off + b_sc;
  if (n_idx) CNNUE_CUDA_TRY(cudaMemcpyAsync(d_idx, h_idx, (size_t)n_idx * 2, cudaMemcpyHostToDevice, s));
  CNNUE_CUDA_TRY(cudaMemcpyAsync(d_off, h_offsets, (size_t)(2 * n + 1) * 4, cudaMemcpyHostToDevice, s));
  int st = launch_sort(m, d_off, n_idx, nullptr, n, ws, s);
  if (st) return st;
  st = launch_eval(m, d_idx, n_idx, d_off, n, d_sc, nullptr, ws, s);
  if (st) return st;
  CNNUE_CUDA_TRY(cudaMemcpyAsync(h_scores, d_sc, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
  int status = CNNUE_OK;
  st = cnnue_read_status(ws, stream, &status);
  if (st) return st;
  return status;
}

int cnnue_q_update(const cnnue_q_model* m, const int16_t* d_parent, const uint8_t* d_flags,
                   const uint16_t* d_rem, uint32_t n_rem, const uint32_t* d_rem_offsets,
                   const uint16_t* d_add, uint32_t n_add, const uint32_t* d_add_offsets,
                   const uint8_t* d_count0, int64_t n, int16_t* d_child, int32_t* d_scores,
                   void* ws, size_t ws_bytes, void* stream) {
  int st = validate_common(m, n, ws, ws_bytes);
  if (st) return st;
  if (n == 0) return CNNUE_OK;
  if (!d_parent || !d_flags || !d_rem_offsets || !d_add_offsets || !d_count0 || !d_child ||
      !d_scores || (n_rem && !d_rem) || (n_add && !d_add))
    return set_error(CNNUE_ERR_INVALID_ARG, "null update buffer");
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  st = launch_sort(m, nullptr, 0, d_count0, n, ws, s);
  if (st) return st;
  st = launch_offsets_check(d_rem_offsets, n_rem, 2 * n, ws, s);
  if (st) return st;
  st = launch_offsets_check(d_add_offsets, n_add, 2 * n, ws, s);
  if (st) return st;
  WorkspaceView v = carve_workspace(ws, n);
  ForwardArgs a{};
  a.w = m->w;
  a.idx = d_add;
  a.n_idx = n_add;
  a.offsets = d_add_offsets;
  a.rem = d_rem;
  a.n_rem = n_rem;
  a.rem_offsets = d_rem_offsets;
  a.parent = d_parent;
  a.flags = d_flags;
  a.acc_out = d_child;
  a.scores = d_scores;
  a.n = n;
  a.perm = v.perm;
  a.sorted_bucket = v.sorted_bucket;
  a.status = &v.hdr->status;
  const int grid = (int)std::min<int64_t>(m->grid_update, (n + kGroupsPerCta - 1) / kGroupsPerCta);
  q_eval_kernel<true, true><<<grid, kCta, 0, s>>>(a);
  return check_launch("q_eval_kernel<update>");
}

}  // extern "C"
