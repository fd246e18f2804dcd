// segreduce.cuh - atomic-free, deterministic segmented reduction
//   grad_table[r][h] = sum of grad_src[src(e)][h] over every contribution e
//   whose row is r,
// used by the feature-pool backward and by the training step's FT backward.
//
// A decoder describes the contributions: kSlots contributions per item
// (items = rows of an item array, or entries of an index list); decode(item)
// gives their rows (returns the number of valid rows, 0 for padding, -1 when a
// row is outside the table) and src(item) the gradient row they read.
//   1. per-chunk row histograms (chunk = kChunkItems consecutive items);
//   2. per-row exclusive prefix over chunks + row totals;
//   3. exclusive scans of row totals (segment starts) and of the rows' work
//      units (a unit = up to kSeg contributions of one row);
//   4. stable scatter: one warp per chunk walks its contributions in
//      enumeration order, ranking equal rows with __match_any_sync, and writes
//      the source row of every contribution into its row's segment;
//   5. one warp per unit sums the source rows of its contributions in order;
//      a row with one unit writes its result directly;
//   6. rows with several units sum their unit partials in order; rows with no
//      contribution are written as zero.
// The summation order is fixed by the input alone, so results are
// deterministic run to run; a row with at most kSeg contributions is summed in
// exactly enumeration order.
#pragma once

#include <algorithm>

#include "common.cuh"

namespace cnnue {
namespace seg {
// Internal linkage: every translation unit that includes this header gets its
// own copy of the kernels.
namespace {

constexpr int kChunkItems = 2048;
constexpr int kSeg = 256;
constexpr unsigned kFull = 0xffffffffu;

struct BwdView {
  uint32_t* status;
  uint32_t* chunk_hist;  // [n_chunks][n_rows]
  uint32_t* row_total;   // [n_rows]
  uint32_t* row_start;   // [n_rows + 1]
  uint32_t* unit_start;  // [n_rows + 1]
  uint32_t* sorted_b;    // [n_items * slots]
  float* partial;        // [max_units][hidden]
};

inline int64_t n_chunks_of(int64_t n_items) { return (n_items + kChunkItems - 1) / kChunkItems; }
inline int64_t max_units_of(int64_t n_contrib, int64_t n_rows) { return n_contrib / kSeg + n_rows + 1; }

inline size_t bwd_bytes(int64_t n_items, int slots, int64_t n_rows, int64_t hidden) {
  const int64_t nc = std::max<int64_t>(n_chunks_of(n_items), 1);
  const int64_t contrib = n_items * slots;
  size_t b = 256;
  b += align_up((size_t)nc * n_rows * 4, 256);
  b += align_up((size_t)n_rows * 4, 256);
  b += 2 * align_up((size_t)(n_rows + 1) * 4, 256);
  b += align_up((size_t)std::max<int64_t>(contrib, 1) * 4, 256);
  b += align_up((size_t)max_units_of(contrib, n_rows) * hidden * 4, 256);
  return b;
}

inline BwdView carve_bwd(void* ws, int64_t n_items, int slots, int64_t n_rows) {
  const int64_t nc = std::max<int64_t>(n_chunks_of(n_items), 1);
  const int64_t contrib = n_items * slots;
  char* p = (char*)ws;
  BwdView v;
  v.status = (uint32_t*)p;
  p += 256;
  v.chunk_hist = (uint32_t*)p;
  p += align_up((size_t)nc * n_rows * 4, 256);
  v.row_total = (uint32_t*)p;
  p += align_up((size_t)n_rows * 4, 256);
  v.row_start = (uint32_t*)p;
  p += align_up((size_t)(n_rows + 1) * 4, 256);
  v.unit_start = (uint32_t*)p;
  p += align_up((size_t)(n_rows + 1) * 4, 256);
  v.sorted_b = (uint32_t*)p;
  p += align_up((size_t)std::max<int64_t>(contrib, 1) * 4, 256);
  v.partial = (float*)p;
  return v;
}

template <class Dec>
__global__ void bwd_hist_kernel(int64_t n_items, Dec dec, BwdView v) {
  extern __shared__ uint32_t hist[];
  const int64_t n_rows = dec.n_rows;
  for (int64_t r = threadIdx.x; r < n_rows; r += blockDim.x) hist[r] = 0;
  __syncthreads();
  const int64_t i0 = (int64_t)blockIdx.x * kChunkItems;
  const int64_t i1 = i0 + kChunkItems < n_items ? i0 + kChunkItems : n_items;
  bool bad = false;
  for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    uint32_t rows[Dec::kSlots];
    const int nr = dec.decode(i, rows);
    if (nr < 0) {
      bad = true;
      continue;
    }
    for (int r = 0; r < nr; ++r) atomicAdd(&hist[rows[r]], 1u);
  }
  if (bad) atomicOr(v.status, CNNUE_STATUS_BAD_INDEX);
  __syncthreads();
  uint32_t* out = v.chunk_hist + (int64_t)blockIdx.x * n_rows;
  for (int64_t r = threadIdx.x; r < n_rows; r += blockDim.x) out[r] = hist[r];
}

__global__ void bwd_chunk_prefix_kernel(int64_t n_chunks, int64_t n_rows, BwdView v) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n_rows) return;
  uint32_t run = 0;
  int64_t c = 0;
  // batches of 8 independent loads, then the sequential prefix
  for (; c + 8 <= n_chunks; c += 8) {
    uint32_t x[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) x[q] = v.chunk_hist[(c + q) * n_rows + r];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      v.chunk_hist[(c + q) * n_rows + r] = run;
      run += x[q];
    }
  }
  for (; c < n_chunks; ++c) {
    uint32_t* h = v.chunk_hist + c * n_rows + r;
    const uint32_t x = *h;
    *h = run;
    run += x;
  }
  v.row_total[r] = run;
}

// Single block: exclusive scans of row totals and of work units per row.
__global__ void bwd_row_scan_kernel(int64_t n_rows, BwdView v) {
  __shared__ uint32_t warp_sum_c[32], warp_sum_u[32];
  __shared__ uint32_t carry_c, carry_u;
  if (threadIdx.x == 0) {
    carry_c = 0;
    carry_u = 0;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int64_t base = 0; base < n_rows; base += blockDim.x) {
    const int64_t r = base + threadIdx.x;
    const uint32_t c = r < n_rows ? v.row_total[r] : 0u;
    const uint32_t u = (c + kSeg - 1) / kSeg;
    uint32_t ic = c, iu = u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t tc = __shfl_up_sync(kFull, ic, o);
      const uint32_t tu = __shfl_up_sync(kFull, iu, o);
      if (lane >= o) {
        ic += tc;
        iu += tu;
      }
    }
    if (lane == 31) {
      warp_sum_c[warp] = ic;
      warp_sum_u[warp] = iu;
    }
    __syncthreads();
    if (warp == 0) {
      uint32_t sc = lane < nw ? warp_sum_c[lane] : 0u, su = lane < nw ? warp_sum_u[lane] : 0u;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t tc = __shfl_up_sync(kFull, sc, o);
        const uint32_t tu = __shfl_up_sync(kFull, su, o);
        if (lane >= o) {
          sc += tc;
          su += tu;
        }
      }
      if (lane < nw) {
        warp_sum_c[lane] = sc;
        warp_sum_u[lane] = su;
      }
    }
    __syncthreads();
    const uint32_t pre_c = carry_c + (warp ? warp_sum_c[warp - 1] : 0u) + ic - c;
    const uint32_t pre_u = carry_u + (warp ? warp_sum_u[warp - 1] : 0u) + iu - u;
    if (r < n_rows) {
      v.row_start[r] = pre_c;
      v.unit_start[r] = pre_u;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      carry_c += warp_sum_c[nw - 1];
      carry_u += warp_sum_u[nw - 1];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    v.row_start[n_rows] = carry_c;
    v.unit_start[n_rows] = carry_u;
  }
}

// One warp per chunk; contributions are walked in (item, slot) order.
template <class Dec>
__global__ void bwd_scatter_kernel(int64_t n_items, Dec dec, BwdView v) {
  extern __shared__ uint32_t cnt[];
  const int64_t n_rows = dec.n_rows;
  const int lane = threadIdx.x;
  for (int64_t r = lane; r < n_rows; r += 32) cnt[r] = 0;
  __syncwarp();
  const int64_t i0 = (int64_t)blockIdx.x * kChunkItems;
  const int64_t i1 = i0 + kChunkItems < n_items ? i0 + kChunkItems : n_items;
  const uint32_t* base_off = v.chunk_hist + (int64_t)blockIdx.x * n_rows;
  const int64_t e0 = i0 * Dec::kSlots, e1 = i1 * Dec::kSlots;
  const uint32_t lt_mask = (1u << lane) - 1u;
  for (int64_t e = e0; e < e1; e += 32) {
    const int64_t my_e = e + lane;
    uint32_t row = 0xffffffffu;
    int64_t item = 0;
    if (my_e < e1) {
      item = my_e / Dec::kSlots;
      const int slot = (int)(my_e - item * Dec::kSlots);
      uint32_t rows[Dec::kSlots];
      const int nr = dec.decode(item, rows);
      if (nr > 0) row = rows[slot];
    }
    const uint32_t peers = __match_any_sync(kFull, row);
    const int leader = __ffs(peers) - 1;
    uint32_t base = 0;
    if (lane == leader && row != 0xffffffffu) {
      base = cnt[row];
      cnt[row] = base + __popc(peers);
    }
    base = __shfl_sync(kFull, base, leader);
    if (row != 0xffffffffu) {
      const uint32_t dest = v.row_start[row] + base_off[row] + base + __popc(peers & lt_mask);
      v.sorted_b[dest] = dec.src(item);
    }
    __syncwarp();
  }
}

// Finds the row owning work unit u (unit_start is non-decreasing).
__device__ __forceinline__ int64_t unit_row(const uint32_t* unit_start, int64_t n_rows, uint32_t u) {
  int64_t lo = 0, hi = n_rows;  // unit_start[lo] <= u < unit_start[hi]
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (unit_start[mid] <= u) lo = mid; else hi = mid;
  }
  return lo;
}

// Units of rows [row_begin, row_end) (all rows by default).
template <bool kVec4>
__global__ void bwd_reduce_kernel(const float* __restrict__ grad_out, int64_t hidden,
                                  int64_t n_rows, BwdView v, float* __restrict__ grad_table,
                                  int64_t row_begin = 0, int64_t row_end = -1) {
  const int lane = threadIdx.x & 31;
  if (row_end < 0) row_end = n_rows;
  const int64_t u = v.unit_start[row_begin] + (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const uint32_t n_units = v.unit_start[row_end];
  if (u >= n_units) return;
  const int64_t r = unit_row(v.unit_start, n_rows, (uint32_t)u);
  const uint32_t k = (uint32_t)u - v.unit_start[r];
  const uint32_t units_r = v.unit_start[r + 1] - v.unit_start[r];
  const uint32_t j0 = v.row_start[r] + k * kSeg;
  const uint32_t j1 = min(j0 + (uint32_t)kSeg, v.row_start[r + 1]);
  float* dst = units_r == 1 ? grad_table + r * hidden : v.partial + u * hidden;
  const int64_t n_chunks = kVec4 ? hidden / 4 : hidden;
  for (int64_t h0 = 0; h0 < n_chunks; h0 += 32) {
    const int64_t hc = h0 + lane;
    if (hc >= n_chunks) break;
    if (kVec4) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      uint32_t j = j0;
      for (; j + 4 <= j1; j += 4) {
        float4 g[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          g[q] = __ldg((const float4*)(grad_out + (int64_t)v.sorted_b[j + q] * hidden) + hc);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc.x += g[q].x;
          acc.y += g[q].y;
          acc.z += g[q].z;
          acc.w += g[q].w;
        }
      }
      for (; j < j1; ++j) {
        const float4 g = __ldg((const float4*)(grad_out + (int64_t)v.sorted_b[j] * hidden) + hc);
        acc.x += g.x;
        acc.y += g.y;
        acc.z += g.z;
        acc.w += g.w;
      }
      *((float4*)dst + hc) = acc;
    } else {
      float acc = 0.f;
      for (uint32_t j = j0; j < j1; ++j) acc += __ldg(grad_out + (int64_t)v.sorted_b[j] * hidden + hc);
      dst[hc] = acc;
    }
  }
}

// Rows with several units sum their unit partials in unit order; rows
// without contributions get zeros; rows with one unit were written by the
// reduction itself.  Grid: (row groups of 8, column chunks of 256); warp w of
// a CTA takes row 8 blockIdx.x + w and its lanes 8 columns each of the
// chunk, so the few rows with many units (the FT bias row: every list) are
// summed by many lanes with independent loads.
constexpr int kFinRows = 8;
constexpr int kFinCols = 256;
__global__ void bwd_finalize_kernel(int64_t hidden, int64_t n_rows, BwdView v,
                                    float* __restrict__ grad_table, int64_t row_begin = 0, int64_t row_end = -1) {
  if (row_end < 0) row_end = n_rows;
  const int64_t r = row_begin + (int64_t)blockIdx.x * kFinRows + (threadIdx.x >> 5);
  if (r >= row_end) return;
  const uint32_t u0 = v.unit_start[r], u1 = v.unit_start[r + 1];
  if (u1 - u0 == 1) return;
  const int64_t h0 = (int64_t)blockIdx.y * kFinCols + (threadIdx.x & 31) * 8;
  if (h0 >= hidden) return;
  const int nh = (int)min((int64_t)8, hidden - h0);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (uint32_t u = u0; u < u1; ++u) {  // unit order; the 8 columns are independent loads
    const float* pr = v.partial + (int64_t)u * hidden + h0;
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (q < nh) acc[q] += pr[q];
  }
#pragma unroll
  for (int q = 0; q < 8; ++q)
    if (q < nh) grad_table[r * hidden + h0 + q] = acc[q];
}

// The reduction of rows [row_begin, row_end) after launch_bwd_prepare (any
// split of the rows into ranges, in any order, gives the same results).
inline int launch_bwd_rows(int64_t n_items, int slots, const float* grad_out, int64_t hidden, int64_t n_rows,
                           float* grad_table, void* ws, int64_t row_begin, int64_t row_end, cudaStream_t s) {
  BwdView v = carve_bwd(ws, n_items, slots, n_rows);
  if (row_begin >= row_end) return CNNUE_OK;
  const int64_t max_units = max_units_of(n_items * slots, n_rows);
  const bool vec4 = hidden % 4 == 0 && ((uintptr_t)grad_out % 16 == 0) &&
                    ((uintptr_t)grad_table % 16 == 0);
  const unsigned rblocks = (unsigned)((max_units * 32 + 255) / 256);
  if (vec4)
    bwd_reduce_kernel<true><<<rblocks, 256, 0, s>>>(grad_out, hidden, n_rows, v, grad_table, row_begin, row_end);
  else
    bwd_reduce_kernel<false><<<rblocks, 256, 0, s>>>(grad_out, hidden, n_rows, v, grad_table, row_begin, row_end);
  int st = check_launch_error("bwd_reduce_kernel");
  if (st) return st;
  const dim3 fgrid((unsigned)((row_end - row_begin + kFinRows - 1) / kFinRows),
                   (unsigned)((hidden + kFinCols - 1) / kFinCols));
  bwd_finalize_kernel<<<fgrid, 32 * kFinRows, 0, s>>>(hidden, n_rows, v, grad_table, row_begin, row_end);
  return check_launch_error("bwd_finalize_kernel");
}

// Steps 1-4 (histograms, prefixes, scans, stable scatter) of launch_bwd.
template <class Dec>
int launch_bwd_prepare(int64_t n_items, Dec dec, void* ws, cudaStream_t s) {
  const int64_t n_rows = dec.n_rows;
  const int64_t nc = n_chunks_of(n_items);
  BwdView v = carve_bwd(ws, n_items, Dec::kSlots, n_rows);
  CNNUE_CUDA_TRY(cudaMemsetAsync(v.status, 0, 4, s));
  const size_t hist_smem = (size_t)n_rows * 4;
  if (hist_smem > 200 * 1024) return set_error(CNNUE_ERR_INVALID_ARG, "table has too many rows");
  if (hist_smem > 48 * 1024) {
    CNNUE_CUDA_TRY(cudaFuncSetAttribute(bwd_hist_kernel<Dec>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)hist_smem));
    CNNUE_CUDA_TRY(cudaFuncSetAttribute(bwd_scatter_kernel<Dec>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hist_smem));
  }
  if (nc > 0) {
    bwd_hist_kernel<Dec><<<(unsigned)nc, 256, hist_smem, s>>>(n_items, dec, v);
    int st = check_launch_error("bwd_hist_kernel");
    if (st) return st;
  }
  bwd_chunk_prefix_kernel<<<(unsigned)((n_rows + 255) / 256), 256, 0, s>>>(nc, n_rows, v);
  int st = check_launch_error("bwd_chunk_prefix_kernel");
  if (st) return st;
  bwd_row_scan_kernel<<<1, 1024, 0, s>>>(n_rows, v);
  st = check_launch_error("bwd_row_scan_kernel");
  if (st) return st;
  if (nc > 0) {
    bwd_scatter_kernel<Dec><<<(unsigned)nc, 32, hist_smem, s>>>(n_items, dec, v);
    st = check_launch_error("bwd_scatter_kernel");
    if (st) return st;
  }
  return CNNUE_OK;
}

template <class Dec>
int launch_bwd(int64_t n_items, const float* grad_out, int64_t hidden, Dec dec, float* grad_table,
               void* ws, cudaStream_t s) {
  const int64_t n_rows = dec.n_rows;
  const int64_t nc = n_chunks_of(n_items);
  BwdView v = carve_bwd(ws, n_items, Dec::kSlots, n_rows);
  CNNUE_CUDA_TRY(cudaMemsetAsync(v.status, 0, 4, s));
  const size_t hist_smem = (size_t)n_rows * 4;
  if (hist_smem > 200 * 1024) return set_error(CNNUE_ERR_INVALID_ARG, "table has too many rows");
  if (hist_smem > 48 * 1024) {
    CNNUE_CUDA_TRY(cudaFuncSetAttribute(bwd_hist_kernel<Dec>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)hist_smem));
    CNNUE_CUDA_TRY(cudaFuncSetAttribute(bwd_scatter_kernel<Dec>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hist_smem));
  }
  if (nc > 0) {
    bwd_hist_kernel<Dec><<<(unsigned)nc, 256, hist_smem, s>>>(n_items, dec, v);
    int st = check_launch_error("bwd_hist_kernel");
    if (st) return st;
  }
  bwd_chunk_prefix_kernel<<<(unsigned)((n_rows + 255) / 256), 256, 0, s>>>(nc, n_rows, v);
  int st = check_launch_error("bwd_chunk_prefix_kernel");
  if (st) return st;
  bwd_row_scan_kernel<<<1, 1024, 0, s>>>(n_rows, v);
  st = check_launch_error("bwd_row_scan_kernel");
  if (st) return st;
  if (nc > 0) {
    bwd_scatter_kernel<Dec><<<(unsigned)nc, 32, hist_smem, s>>>(n_items, dec, v);
    st = check_launch_error("bwd_scatter_kernel");
    if (st) return st;
  }
  const int64_t max_units = max_units_of(n_items * Dec::kSlots, n_rows);
  const bool vec4 = hidden % 4 == 0 && ((uintptr_t)grad_out % 16 == 0) &&
                    ((uintptr_t)grad_table % 16 == 0);
  const unsigned rblocks = (unsigned)((max_units * 32 + 255) / 256);
  if (vec4)
    bwd_reduce_kernel<true><<<rblocks, 256, 0, s>>>(grad_out, hidden, n_rows, v, grad_table);
  else
    bwd_reduce_kernel<false><<<rblocks, 256, 0, s>>>(grad_out, hidden, n_rows, v, grad_table);
  st = check_launch_error("bwd_reduce_kernel");
  if (st) return st;
  const dim3 fgrid((unsigned)((n_rows + kFinRows - 1) / kFinRows), (unsigned)((hidden + kFinCols - 1) / kFinCols));
  bwd_finalize_kernel<<<fgrid, 32 * kFinRows, 0, s>>>(hidden, n_rows, v, grad_table, 0, n_rows);
  return check_launch_error("bwd_finalize_kernel");
}

}  // namespace
}  // namespace seg
}  // namespace cnnue
