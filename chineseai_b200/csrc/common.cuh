// common.cuh - shared helpers of the cnnue library (status handling, device
// loads, workspace layout).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/cnnue.h"

namespace cnnue {

// Sets the calling thread's last-error text and returns `status`.
int set_error(int status, const char* fmt, ...);

// Maps a CUDA error to CNNUE_ERR_CUDA with the runtime's message.
int cuda_error(cudaError_t err, const char* what);

#define CNNUE_CUDA_TRY(expr)                                       \
  do {                                                             \
    cudaError_t err__ = (expr);                                    \
    if (err__ != cudaSuccess) return ::cnnue::cuda_error(err__, #expr); \
  } while (0)

// Maps a kernel status word (CNNUE_STATUS_* bits) to a CNNUE_ERR_* code and
// records the detail as the thread's last error.
// AdamW on the device state (cnnue_adamw_state, optim.cu): the step's
// scalars once (advances the step), then any number of updates of disjoint
// ranges of the flat buffers with them (float4 groups, 16-byte aligned).
constexpr int kMaxAdamRanges = 8;
struct AdamWRanges {
  int64_t begin[kMaxAdamRanges];  // element offsets, multiples of 4
  int64_t len4[kMaxAdamRanges];   // lengths in float4 groups
  int n;
};
int adamw_prepare(cnnue_adamw_state* d_state, cudaStream_t s);
int adamw_ranges(float* d_params, float* d_m, float* d_v, const float* d_grads, const AdamWRanges& r,
                 const cnnue_adamw_state* d_state, cudaStream_t s);

int status_from_word(uint32_t word);

// Checks that `device` is the current device, switching to it if needed.
int use_device(int device);

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Two independent IEEE round-to-nearest fp32 additions (subtractions) in one
// packed sm_100 instruction: (a0, a1) += (b0, b1), the same results as two
// __fadd_rn (__fsub_rn).
__device__ __forceinline__ void fadd2_rn(float& a0, float& a1, float b0, float b1) {
  asm("{.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
}
__device__ __forceinline__ void fsub2_rn(float& a0, float& a1, float b0, float b1) {
  asm("{.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
}

// Workspace header shared by every entry point that takes a workspace.
// The status word is the first 4 bytes; kernels OR CNNUE_STATUS_* bits in.
struct WorkspaceHeader {
  uint32_t status;
  uint32_t pad0[31];
  uint32_t counts[32];   // per-bucket position counts
  uint32_t cursors[32];  // per-bucket scatter cursors
  uint32_t pad1[32];
};
static_assert(sizeof(WorkspaceHeader) == 512, "header size");

// Bucket-sort workspace: header, then bucket_of[n] (u8), perm[n] (u32),
// sorted_bucket[n] (u8), block_hist[ceil(n/256)][32] (u32), each 256-byte
// aligned.
struct WorkspaceView {
  WorkspaceHeader* hdr;    // counts[b] = positions of bucket b, cursors[b] = first slot of b
  uint8_t* bucket_of;      // [n]
  uint32_t* perm;          // [n] positions in bucket order (ascending within a bucket)
  uint8_t* sorted_bucket;  // [n] bucket of perm[i]
  uint32_t* block_hist;    // [ceil(n/256)][32] per-block counts, then per-block prefixes
};
size_t bucket_workspace_bytes(int64_t n);
WorkspaceView carve_workspace(void* ws, int64_t n);
// Buckets the n positions (bucket = min((max(n0,1)-1)
// >> shift, n_buckets-1), n0 from the offsets or from d_count0) and scatters
// them into bucket order, stably (ascending positions within a bucket), so
// everything computed in that order is deterministic.  Offsets are validated
// into the status word, which the sort writes (clearing earlier bits): the
// workspace needs no clearing before it.  n_buckets <= 31.
// When `inv` is not null it receives the inverse order: inv[p] = the sorted
// slot of position p.
// d_extra0 / d_extra1 (optional): further [2n + 1] list offsets arrays whose
// lists are checked with the sort (monotone, at most n_extra0 / n_extra1).
int launch_bucket_sort(const uint32_t* d_offsets, uint32_t n_indices, const uint8_t* d_count0,
                       int64_t n, int shift, int n_buckets, void* ws, cudaStream_t s,
                       uint32_t* inv = nullptr, const uint32_t* d_extra0 = nullptr, uint32_t n_extra0 = 0,
                       const uint32_t* d_extra1 = nullptr, uint32_t n_extra1 = 0);

// Tile g of the buckets' tiles in bucket order (each bucket's rows of the
// sorted order cut into tiles of `rows`): its bucket, first sorted slot and
// row count.  False past the last tile.
__device__ __forceinline__ bool bucket_tile(const WorkspaceHeader* hdr, int n_buckets, uint32_t rows, uint32_t g,
                                            int* bucket, int* start, int* count, uint32_t* first_tile) {
  uint32_t tiles_before = 0;
  for (int b = 0; b < n_buckets; ++b) {
    const uint32_t c = hdr->counts[b];
    const uint32_t tiles = (c + rows - 1) / rows;
    if (g < tiles) {
      *bucket = b;
      *start = (int)(hdr->cursors[b] + g * rows);
      *count = (int)min(rows, c - g * rows);
      *first_tile = tiles_before;
      return true;
    }
    g -= tiles;
    tiles_before += tiles;
  }
  return false;
}

// RAII switch to a device, restoring the caller's current device.
struct DeviceGuard {
  int prev = -1;
  bool switched = false;
  int status = CNNUE_OK;
  explicit DeviceGuard(int device);
  ~DeviceGuard();
};

int check_launch_error(const char* what);

// Streaming 16-byte load that bypasses L1 allocation (rows are read once per
// position; L1 is kept for the per-bucket stack weights).
__device__ __forceinline__ uint4 ldg_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float4 ldg_stream16f(const void* p) {
  float4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

// Named barrier over `nthreads` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace cnnue
