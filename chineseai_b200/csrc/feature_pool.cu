// feature_pool.cu - the AZ-NNUE trunk feature transformer (feature pool) and
// the threat table pool: forward gather-accumulate and atomic-free backward.
//
// Forward: one warp per batch row; lanes own 4 consecutive hidden columns
// (one 16-byte load per table row) when hidden % 4 == 0, else one column.
// Every output column is summed from 0 in item order, the item's rows in the
// fixed order (feature, piece, rank, file, king(us), king(them)) - the order of
// the reference's CPU twin - so forward results are bit-identical to it.
//
// Backward (grad_table[r] = sum of grad_out[b] over every contribution (b,
// item, slot) whose row is r), without atomics, by the segmented reduction of
// segreduce.cuh:
//   1. per-chunk row histograms (chunk = kChunkItems consecutive items);
//   2. per-row exclusive prefix over chunks + row totals;
//   3. exclusive scans of row totals (segment starts) and of the rows' work
//      units (a unit = up to kSeg contributions of one row);
//   4. stable scatter: one warp per chunk walks its contributions in
//      enumeration order, ranking equal rows with __match_any_sync, and writes
//      the batch row b of every contribution into its row's segment;
//   5. one warp per unit sums grad_out rows of its contributions in order;
//      a row with one unit writes its result directly;
//   6. rows with several units sum their unit partials in order; rows with no
//      contribution are written as zero.
// The summation order is fixed by the input alone, so results are
// deterministic run to run; a row with at most kSeg contributions is summed in
// exactly the reference CPU order.
//
// The AZ feature pool's backward, and plain tables of more than kSegMaxRows
// rows (the 57,702-row threat table, whose per-chunk histograms would not fit
// in shared memory), take the radix-sorted row scatter of scatter.cuh
// instead: same order, same exactness, and parallel over rows rather than
// over chunks of items (the segmented form keeps the C4 training step).
#include <algorithm>

#include "common.cuh"
#include "scatter.cuh"
#include "segreduce.cuh"

namespace cnnue {
namespace pool {

constexpr uint32_t kPad = CNNUE_POOL_PADDING;
constexpr int kRows = CNNUE_POOL_ROWS;
constexpr unsigned kFull = 0xffffffffu;

// Row decoders. rows[] gets the item's rows; returns the number of valid rows
// (0 for padding), or -1 when a row falls outside the table.
struct AzDecoder {
  static constexpr int kSlots = 6;
  int64_t n_rows;                   // 1545
  const uint32_t* items = nullptr;  // [batch][item_count] (backward)
  int64_t item_count = 1;
  __device__ __forceinline__ uint32_t src(int64_t item) const { return (uint32_t)(item / item_count); }
  __device__ __forceinline__ int decode(int64_t item, uint32_t rows[6]) const {
    return decode_item(items[item], rows);
  }
  __device__ __forceinline__ int decode_item(uint32_t packed, uint32_t rows[6]) const {
    if (packed == kPad) return 0;
    const uint32_t feature = packed & 0x7ffu;
    const uint32_t us = (packed >> 11) & 0xfu;
    const uint32_t them = (packed >> 15) & 0xfu;
    const uint32_t piece = feature / 90u, square = feature - piece * 90u;
    rows[0] = feature;
    rows[1] = 1260u + piece;
    rows[2] = 1274u + square / 9u;
    rows[3] = 1284u + square % 9u;
    rows[4] = 1293u + us * 14u + piece;
    rows[5] = 1293u + (9u + them) * 14u + piece;
    bool ok = true;
#pragma unroll
    for (int r = 0; r < 6; ++r) ok &= rows[r] < (uint32_t)kRows;
    return ok ? 6 : -1;
  }
};

struct PlainDecoder {
  static constexpr int kSlots = 1;
  int64_t n_rows;
  const uint32_t* items = nullptr;  // [batch][item_count] (backward)
  int64_t item_count = 1;
  __device__ __forceinline__ uint32_t src(int64_t item) const { return (uint32_t)(item / item_count); }
  __device__ __forceinline__ int decode(int64_t e, uint32_t rows[1]) const {
    return decode_item(items[e], rows);
  }
  __device__ __forceinline__ int decode_item(uint32_t item, uint32_t rows[1]) const {
    if (item == kPad) return 0;
    rows[0] = item;
    return (int64_t)item < n_rows ? 1 : -1;
  }
};

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <class Dec, bool kVec4>
__global__ void pool_fwd_kernel(const float* __restrict__ table, const uint32_t* __restrict__ items,
                                int64_t batch, int64_t item_count, int64_t hidden, Dec dec,
                                float* __restrict__ out, uint32_t* status) {
  const int lane = threadIdx.x & 31;
  const int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (b >= batch) return;
  const int64_t n_chunks = kVec4 ? hidden / 4 : hidden;
  for (int64_t h0 = 0; h0 < n_chunks; h0 += 32) {
    const int64_t hc = h0 + lane;
    const bool active = hc < n_chunks;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t i0 = 0; i0 < item_count; i0 += 32) {
      const int cnt = (int)(item_count - i0 < 32 ? item_count - i0 : 32);
      const uint32_t my = lane < cnt ? items[b * item_count + i0 + lane] : kPad;
      for (int j = 0; j < cnt; ++j) {
        const uint32_t packed = __shfl_sync(kFull, my, j);
        uint32_t rows[Dec::kSlots];
        const int nr = dec.decode_item(packed, rows);
        if (nr < 0) {
          if (lane == 0 && h0 == 0) atomicOr(status, CNNUE_STATUS_BAD_INDEX);
          continue;
        }
        if (nr == 0 || !active) continue;
        if (kVec4) {
          float4 v[Dec::kSlots];
#pragma unroll
          for (int r = 0; r < Dec::kSlots; ++r)
            v[r] = __ldg((const float4*)(table + (int64_t)rows[r] * hidden) + hc);
#pragma unroll
          for (int r = 0; r < Dec::kSlots; ++r) {
            acc.x += v[r].x;
            acc.y += v[r].y;
            acc.z += v[r].z;
            acc.w += v[r].w;
          }
        } else {
          float v[Dec::kSlots];
#pragma unroll
          for (int r = 0; r < Dec::kSlots; ++r) v[r] = __ldg(table + (int64_t)rows[r] * hidden + hc);
#pragma unroll
          for (int r = 0; r < Dec::kSlots; ++r) acc.x += v[r];
        }
      }
    }
    if (active) {
      if (kVec4)
        *((float4*)(out + b * hidden) + hc) = acc;
      else
        out[b * hidden + hc] = acc.x;
    }
  }
}

template <class Dec>
int launch_fwd(const float* table, const uint32_t* items, int64_t batch, int64_t item_count,
               int64_t hidden, Dec dec, float* out, uint32_t* status, cudaStream_t s) {
  const int threads = 256;
  const int64_t blocks = (batch * 32 + threads - 1) / threads;
  const bool vec4 = hidden % 4 == 0 && ((uintptr_t)table % 16 == 0) && ((uintptr_t)out % 16 == 0);
  if (vec4)
    pool_fwd_kernel<Dec, true><<<(unsigned)blocks, threads, 0, s>>>(table, items, batch, item_count,
                                                                     hidden, dec, out, status);
  else
    pool_fwd_kernel<Dec, false><<<(unsigned)blocks, threads, 0, s>>>(table, items, batch, item_count,
                                                                      hidden, dec, out, status);
  return check_launch_error("pool_fwd_kernel");
}

constexpr int64_t kSegMaxRows = 16384;  // shared-memory row histogram of a chunk

// Plain-pool items as scatter keys: padding and out-of-range rows map to the
// drop key `rows` (out-of-range ones are flagged).
__global__ void plain_keys_kernel(const uint32_t* __restrict__ items, int64_t n, int64_t rows,
                                  uint32_t* __restrict__ keys, uint32_t* status) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t it = items[i];
    const bool pad = it == kPad, ok = (int64_t)it < rows;
    if (!pad && !ok) atomicOr(status, CNNUE_STATUS_BAD_INDEX);
    keys[i] = (!pad && ok) ? it : (uint32_t)rows;
  }
}

inline size_t sorted_bwd_bytes(int64_t n_items, int64_t hidden) {
  return sizeof(WorkspaceHeader) + align_up((size_t)std::max<int64_t>(n_items, 1) * 4, 256) +
         scat::workspace_bytes(n_items, hidden);
}

// Feature-pool items as scatter keys: contribution e = 6 * item + slot, the
// item's six rows in the reference order; padding and bad items map to the
// drop key (bad ones are flagged).
__global__ void az_keys_kernel(const uint32_t* __restrict__ items, int64_t n_items, uint32_t* __restrict__ keys,
                               uint32_t* status) {
  const AzDecoder dec{kRows};
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_items;
       i += (int64_t)gridDim.x * blockDim.x) {
    uint32_t rows[6];
    const int nr = dec.decode_item(items[i], rows);
    if (nr < 0) atomicOr(status, CNNUE_STATUS_BAD_INDEX);
#pragma unroll
    for (int r = 0; r < 6; ++r) keys[i * 6 + r] = nr == 6 ? rows[r] : (uint32_t)kRows;
  }
}

int check_shape(int64_t batch, int64_t item_count, int64_t hidden) {
  if (batch < 0 || item_count < 0 || hidden <= 0)
    return set_error(CNNUE_ERR_INVALID_ARG, "bad shape batch=%lld items=%lld hidden=%lld",
                     (long long)batch, (long long)item_count, (long long)hidden);
  if (batch * item_count * 6 >= (int64_t)UINT32_MAX || batch >= (int64_t)UINT32_MAX)
    return set_error(CNNUE_ERR_INVALID_ARG, "batch too large");
  return CNNUE_OK;
}

}  // namespace pool
}  // namespace cnnue

using namespace cnnue;
using namespace cnnue::pool;

extern "C" {

int cnnue_feature_pool_fwd(const float* d_tables, const uint32_t* d_items, int64_t batch,
                           int64_t item_count, int64_t hidden, float* d_out, uint32_t* d_status,
                           void* stream) {
  int st = check_shape(batch, item_count, hidden);
  if (st) return st;
  if (batch == 0) return CNNUE_OK;
  if (!d_tables || !d_out || !d_status || (item_count && !d_items))
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer");
  return launch_fwd(d_tables, d_items, batch, item_count, hidden, AzDecoder{kRows}, d_out, d_status,
                    (cudaStream_t)stream);
}

size_t cnnue_feature_pool_bwd_workspace_bytes(int64_t batch, int64_t item_count, int64_t hidden) {
  if (batch < 0 || item_count < 0 || hidden <= 0) return 0;
  return sorted_bwd_bytes(batch * item_count * 6, hidden);
}

int cnnue_feature_pool_bwd(const uint32_t* d_items, const float* d_grad_out, int64_t batch,
                           int64_t item_count, int64_t hidden, float* d_grad_tables,
                           void* d_workspace, size_t workspace_bytes, void* stream) {
  int st = check_shape(batch, item_count, hidden);
  if (st) return st;
  if (!d_grad_tables || !d_workspace || (batch && !d_grad_out) || (batch * item_count && !d_items))
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer");
  if (workspace_bytes < cnnue_feature_pool_bwd_workspace_bytes(batch, item_count, hidden))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace too small");
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t n_items = batch * item_count;
  CNNUE_CUDA_TRY(cudaMemsetAsync(d_workspace, 0, sizeof(WorkspaceHeader), s));
  uint32_t* status = &((WorkspaceHeader*)d_workspace)->status;
  uint32_t* keys = (uint32_t*)((char*)d_workspace + sizeof(WorkspaceHeader));
  void* scratch = (char*)keys + align_up((size_t)std::max<int64_t>(6 * n_items, 1) * 4, 256);
  if (n_items > 0) {
    const unsigned g = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n_items + 255) / 256, 148 * 16));
    az_keys_kernel<<<g, 256, 0, s>>>(d_items, n_items, keys, status);
    if (int e = check_launch_error("az_keys_kernel")) return e;
  }
  return scat::launch_scatter_add_rows(keys, d_grad_out, (uint32_t)(6 * item_count), hidden, 6 * n_items, kRows,
                                       d_grad_tables, scratch, s);
}

int cnnue_sparse_pool_fwd(const float* d_table, int64_t rows, const uint32_t* d_items,
                          int64_t batch, int64_t item_count, int64_t hidden, float* d_out,
                          uint32_t* d_status, void* stream) {
  int st = check_shape(batch, item_count, hidden);
  if (st) return st;
  if (rows <= 0 || rows >= (int64_t)UINT32_MAX) return set_error(CNNUE_ERR_INVALID_ARG, "bad rows");
  if (batch == 0) return CNNUE_OK;
  if (!d_table || !d_out || !d_status || (item_count && !d_items))
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer");
  return launch_fwd(d_table, d_items, batch, item_count, hidden, PlainDecoder{rows}, d_out,
                    d_status, (cudaStream_t)stream);
}

size_t cnnue_sparse_pool_bwd_workspace_bytes(int64_t rows, int64_t batch, int64_t item_count,
                                             int64_t hidden) {
  if (rows <= 0 || batch < 0 || item_count < 0 || hidden <= 0) return 0;
  if (rows > kSegMaxRows) return sorted_bwd_bytes(batch * item_count, hidden);
  return seg::bwd_bytes(batch * item_count, 1, rows, hidden);
}

int cnnue_sparse_pool_bwd(const uint32_t* d_items, const float* d_grad_out, int64_t rows,
                          int64_t batch, int64_t item_count, int64_t hidden, float* d_grad_table,
                          void* d_workspace, size_t workspace_bytes, void* stream) {
  int st = check_shape(batch, item_count, hidden);
  if (st) return st;
  if (rows <= 0 || rows >= (int64_t)UINT32_MAX) return set_error(CNNUE_ERR_INVALID_ARG, "bad rows");
  if (!d_grad_table || !d_workspace || (batch && !d_grad_out) || (batch * item_count && !d_items))
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer");
  if (workspace_bytes < cnnue_sparse_pool_bwd_workspace_bytes(rows, batch, item_count, hidden))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace too small");
  if (rows > kSegMaxRows) {
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t n = batch * item_count;
    CNNUE_CUDA_TRY(cudaMemsetAsync(d_workspace, 0, sizeof(WorkspaceHeader), s));
    uint32_t* status = &((WorkspaceHeader*)d_workspace)->status;
    uint32_t* keys = (uint32_t*)((char*)d_workspace + sizeof(WorkspaceHeader));
    void* scratch = (char*)keys + align_up((size_t)std::max<int64_t>(n, 1) * 4, 256);
    if (n > 0) {
      const unsigned g = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 16));
      plain_keys_kernel<<<g, 256, 0, s>>>(d_items, n, rows, keys, status);
      if (int e = check_launch_error("plain_keys_kernel")) return e;
    }
    return scat::launch_scatter_add_rows(keys, d_grad_out, (uint32_t)item_count, hidden, n, rows, d_grad_table,
                                         scratch, s);
  }
  PlainDecoder dec{rows, d_items, item_count};
  return seg::launch_bwd(batch * item_count, d_grad_out, hidden, dec, d_grad_table, d_workspace,
                         (cudaStream_t)stream);
}

}  // extern "C"
