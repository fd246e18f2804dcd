// bucket_sort.cu - groups the positions of a batch by output bucket.
//
// A stable counting sort in three kernels: (1) the bucket of every position
// (from the perspective-0 active count, or from an explicit count array) and
// per-block bucket histograms, plus the offsets checks (the lists' own, and
// up to two further list arrays'); (2) one CTA turns the
// histograms into per-block prefixes, bucket totals and bucket starts; (3) a
// scatter of position ids into bucket order, ranked inside each block with
// warp match masks, so positions stay in ascending order within a bucket.
// The evaluators walk that order so the weights of one bucket stay resident;
// the training step also sums its bucketed gradients in it, which makes them
// deterministic.
#include "common.cuh"

namespace cnnue {

namespace {
constexpr int kSortThreads = 256;
constexpr unsigned kFull = 0xffffffffu;

inline size_t n_blocks(int64_t n) { return n > 0 ? (size_t)((n + kSortThreads - 1) / kSortThreads) : 0; }
}  // namespace

size_t bucket_workspace_bytes(int64_t n) {
  size_t nn = n > 0 ? (size_t)n : 0;
  return sizeof(WorkspaceHeader) + align_up(nn, 256) + align_up(nn * 4, 256) + align_up(nn, 256) +
         align_up(n_blocks(n) * 32 * 4, 256);
}

WorkspaceView carve_workspace(void* ws, int64_t n) {
  WorkspaceView v;
  const size_t nn = n > 0 ? (size_t)n : 0;
  char* p = (char*)ws;
  v.hdr = (WorkspaceHeader*)p;
  p += sizeof(WorkspaceHeader);
  v.bucket_of = (uint8_t*)p;
  p += align_up(nn, 256);
  v.perm = (uint32_t*)p;
  p += align_up(nn * 4, 256);
  v.sorted_bucket = (uint8_t*)p;
  p += align_up(nn, 256);
  v.block_hist = (uint32_t*)p;
  return v;
}

namespace {

// Slot 31 of a block's histogram row carries the block's status bits (at most
// 31 buckets); the scan ORs them into the header's status word, which it
// writes first - so nothing needs clearing before the sort.
constexpr int kStatusSlot = 31;

// Also checks the (perspective 0, perspective 1) list offsets of up to two
// further list arrays (an update's removed and added rows) for position p.
struct ExtraLists {
  const uint32_t* off[2];
  uint32_t n_values[2];
};

__global__ void __launch_bounds__(kSortThreads) bucket_count_kernel(
    const uint32_t* __restrict__ offsets, uint32_t n_indices, const uint8_t* __restrict__ count0,
    int64_t n, int shift, int max_bucket, uint8_t* __restrict__ bucket_of,
    WorkspaceHeader* __restrict__ hdr, uint32_t* __restrict__ block_hist, ExtraLists extra) {
  __shared__ uint32_t hist[32];
  if (threadIdx.x < 32) hist[threadIdx.x] = 0;
  __syncthreads();
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint32_t bad = 0;
  if (p < n) {
    uint32_t n0;
    if (count0 != nullptr) {
      n0 = count0[p];
    } else {
      const uint32_t o0 = offsets[2 * p], o1 = offsets[2 * p + 1], o2 = offsets[2 * p + 2];
      if (!(o0 <= o1 && o1 <= o2 && o2 <= n_indices)) {
        bad = CNNUE_STATUS_BAD_OFFSETS;
        n0 = 0;
      } else {
        n0 = o1 - o0;
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k)
      if (extra.off[k]) {
        const uint32_t e0 = extra.off[k][2 * p], e1 = extra.off[k][2 * p + 1], e2 = extra.off[k][2 * p + 2];
        if (!(e0 <= e1 && e1 <= e2 && e2 <= extra.n_values[k])) bad = CNNUE_STATUS_BAD_OFFSETS;
      }
    const uint32_t nn = n0 < 1u ? 1u : n0;
    const uint32_t b = min((nn - 1u) >> shift, (uint32_t)max_bucket);
    bucket_of[p] = (uint8_t)b;
    atomicAdd(&hist[b], 1u);  // order-free count
  }
  if (bad) atomicOr(&hist[kStatusSlot], bad);  // the block's status bits (the scan combines them)
  __syncthreads();
  if (threadIdx.x < 32) block_hist[(size_t)blockIdx.x * 32 + threadIdx.x] = hist[threadIdx.x];
}

// One CTA, one warp per bucket: block_hist[blk][b] becomes the number of
// bucket-b positions in blocks before blk; counts[b] gets the total and
// cursors[b] the bucket's first slot.  Up to 32 x kScanPerLane blocks, lane l
// scans a contiguous run of ceil(nblk / 32) blocks with all its loads issued
// together, then the warp scans the lanes' totals; larger batches walk the
// blocks 32 at a time.
constexpr int kScanPerLane = 32;  // one load round: nblk <= 1024 (262,144 positions)

__global__ void __launch_bounds__(1024) bucket_scan_kernel(uint32_t nblk, int n_buckets,
                                                           WorkspaceHeader* __restrict__ hdr,
                                                           uint32_t* __restrict__ block_hist) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < n_buckets) {
    uint32_t run = 0;
    const uint32_t per = (nblk + 31) / 32;
    if (per <= (uint32_t)kScanPerLane) {
      const uint32_t b0 = lane * per;
      uint32_t v[kScanPerLane];
      uint32_t tot = 0;
#pragma unroll
      for (int k = 0; k < kScanPerLane; ++k) {
        v[k] = (uint32_t)k < per && b0 + k < nblk ? block_hist[(size_t)(b0 + k) * 32 + warp] : 0u;
        tot += v[k];
      }
      uint32_t incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t x = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += x;
      }
      uint32_t acc = incl - tot;
#pragma unroll
      for (int k = 0; k < kScanPerLane; ++k)
        if ((uint32_t)k < per && b0 + k < nblk) {
          block_hist[(size_t)(b0 + k) * 32 + warp] = acc;
          acc += v[k];
        }
      run = __shfl_sync(kFull, incl, 31);
    } else {
      for (uint32_t base = 0; base < nblk; base += 32) {
        const uint32_t blk = base + lane;
        const uint32_t v = blk < nblk ? block_hist[(size_t)blk * 32 + warp] : 0u;
        uint32_t incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t x = __shfl_up_sync(kFull, incl, o);
          if (lane >= o) incl += x;
        }
        if (blk < nblk) block_hist[(size_t)blk * 32 + warp] = run + incl - v;
        run += __shfl_sync(kFull, incl, 31);
      }
    }
    if (lane == 0) hdr->counts[warp] = run;
  } else if (warp == n_buckets) {
    uint32_t bits = 0;
    for (uint32_t blk = lane; blk < nblk; blk += 32) bits |= block_hist[(size_t)blk * 32 + kStatusSlot];
#pragma unroll
    for (int o = 16; o; o >>= 1) bits |= __shfl_xor_sync(kFull, bits, o);
    if (lane == 0) hdr->status = bits;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t start = 0;
    for (int b = 0; b < 32; ++b) {
      hdr->cursors[b] = start;
      start += b < n_buckets ? hdr->counts[b] : 0u;
    }
  }
}

__global__ void __launch_bounds__(kSortThreads) bucket_scatter_kernel(
    int64_t n, const uint8_t* __restrict__ bucket_of, const WorkspaceHeader* __restrict__ hdr,
    const uint32_t* __restrict__ block_hist, uint32_t* __restrict__ perm,
    uint8_t* __restrict__ sorted_bucket, uint32_t* __restrict__ inv) {
  // the evaluator's gather may be scheduled now: its producers read only the
  // batch's lists; what reads this kernel's output waits (griddepcontrol.wait)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  constexpr int kWarps = kSortThreads / 32;
  __shared__ uint32_t wcount[kWarps][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kWarps * 32; i += kSortThreads) (&wcount[0][0])[i] = 0;
  __syncthreads();
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool valid = p < n;
  const uint32_t b = valid ? bucket_of[p] : 32u;
  const uint32_t peers = __match_any_sync(kFull, b);
  const uint32_t rank = __popc(peers & ((1u << lane) - 1u));
  if (valid && lane == __ffs(peers) - 1) wcount[warp][b] = __popc(peers);
  __syncthreads();
  if (valid) {
    uint32_t before = 0;
    for (int w = 0; w < warp; ++w) before += wcount[w][b];
    const uint32_t slot = hdr->cursors[b] + block_hist[(size_t)blockIdx.x * 32 + b] + before + rank;
    perm[slot] = (uint32_t)p;
    sorted_bucket[slot] = (uint8_t)b;
    if (inv) inv[p] = slot;
  }
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, what);
  return CNNUE_OK;
}

}  // namespace

int launch_bucket_sort(const uint32_t* d_offsets, uint32_t n_indices, const uint8_t* d_count0,
                       int64_t n, int shift, int n_buckets, void* ws, cudaStream_t s, uint32_t* inv,
                       const uint32_t* d_extra0, uint32_t n_extra0, const uint32_t* d_extra1, uint32_t n_extra1) {
  WorkspaceView v = carve_workspace(ws, n);
  if (n_buckets < 1 || n_buckets > kStatusSlot)
    return set_error(CNNUE_ERR_INVALID_ARG, "bucket sort: %d buckets (1..%d)", n_buckets, kStatusSlot);
  if (n <= 0) {
    CNNUE_CUDA_TRY(cudaMemsetAsync(v.hdr, 0, sizeof(WorkspaceHeader), s));
    return CNNUE_OK;
  }
  const unsigned blocks = (unsigned)n_blocks(n);
  ExtraLists extra{{d_extra0, d_extra1}, {n_extra0, n_extra1}};
  bucket_count_kernel<<<blocks, kSortThreads, 0, s>>>(d_offsets, n_indices, d_count0, n, shift,
                                                      n_buckets - 1, v.bucket_of, v.hdr, v.block_hist, extra);
  int st = check_launch("bucket_count_kernel");
  if (st) return st;
  // a warp per bucket, then one warp for the status bits
  bucket_scan_kernel<<<1, 32 * (n_buckets + 1), 0, s>>>(blocks, n_buckets, v.hdr, v.block_hist);
  st = check_launch("bucket_scan_kernel");
  if (st) return st;
  bucket_scatter_kernel<<<blocks, kSortThreads, 0, s>>>(n, v.bucket_of, v.hdr, v.block_hist, v.perm,
                                                        v.sorted_bucket, inv);
  return check_launch("bucket_scatter_kernel");
}

}  // namespace cnnue
