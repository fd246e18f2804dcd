// bucket_sort.cu - groups the positions of a batch by output bucket.
//
// Two kernels: (1) the bucket of every position (from the perspective-0
// active count, or from an explicit count array) with block-aggregated
// per-bucket counts, and the offsets check; (2) a scatter of position ids into
// bucket order.  The evaluators then walk that order so the weights of one
// bucket stay resident while a group of threads evaluates its positions.
#include "common.cuh"

namespace cnnue {

size_t bucket_workspace_bytes(int64_t n) {
  size_t nn = n > 0 ? (size_t)n : 0;
  return sizeof(WorkspaceHeader) + align_up(nn, 256) + align_up(nn * 4, 256) + align_up(nn, 256);
}

WorkspaceView carve_workspace(void* ws, int64_t n) {
  WorkspaceView v;
  char* p = (char*)ws;
  v.hdr = (WorkspaceHeader*)p;
  p += sizeof(WorkspaceHeader);
  v.bucket_of = (uint8_t*)p;
  p += align_up((size_t)(n > 0 ? n : 0), 256);
  v.perm = (uint32_t*)p;
  p += align_up((size_t)(n > 0 ? n : 0) * 4, 256);
  v.sorted_bucket = (uint8_t*)p;
  return v;
}

namespace {

__global__ void bucket_count_kernel(const uint32_t* __restrict__ offsets, uint32_t n_indices,
                                    const uint8_t* __restrict__ count0, int64_t n, int shift,
                                    int max_bucket, uint8_t* __restrict__ bucket_of,
                                    WorkspaceHeader* __restrict__ hdr) {
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
    const uint32_t nn = n0 < 1u ? 1u : n0;
    const uint32_t b = min((nn - 1u) >> shift, (uint32_t)max_bucket);
    bucket_of[p] = (uint8_t)b;
    atomicAdd(&hist[b], 1u);
  }
  if (bad) atomicOr(&hdr->status, bad);
  __syncthreads();
  if (threadIdx.x < 32 && hist[threadIdx.x]) atomicAdd(&hdr->counts[threadIdx.x], hist[threadIdx.x]);
}

__global__ void offsets_check_kernel(const uint32_t* __restrict__ offsets, uint32_t n_values,
                                     int64_t n_lists, WorkspaceHeader* __restrict__ hdr) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n_lists) {
    const uint32_t a = offsets[i], b = offsets[i + 1];
    if (!(a <= b && b <= n_values)) atomicOr(&hdr->status, CNNUE_STATUS_BAD_OFFSETS);
  }
}

__global__ void bucket_scatter_kernel(int64_t n, int n_buckets,
                                      const uint8_t* __restrict__ bucket_of,
                                      WorkspaceHeader* __restrict__ hdr,
                                      uint32_t* __restrict__ perm,
                                      uint8_t* __restrict__ sorted_bucket) {
  __shared__ uint32_t base[32], hist[32], block_base[32];
  if (threadIdx.x < 32) hist[threadIdx.x] = 0;
  if (threadIdx.x == 0) {
    uint32_t run = 0;
    for (int b = 0; b < 32; ++b) {
      base[b] = run;
      run += b < n_buckets ? hdr->counts[b] : 0u;
    }
  }
  __syncthreads();
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint32_t b = 0, rank = 0;
  if (p < n) {
    b = bucket_of[p];
    rank = atomicAdd(&hist[b], 1u);
  }
  __syncthreads();
  if (threadIdx.x < 32 && hist[threadIdx.x])
    block_base[threadIdx.x] = atomicAdd(&hdr->cursors[threadIdx.x], hist[threadIdx.x]);
  __syncthreads();
  if (p < n) {
    const uint32_t slot = base[b] + block_base[b] + rank;
    perm[slot] = (uint32_t)p;
    sorted_bucket[slot] = (uint8_t)b;
  }
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, what);
  return CNNUE_OK;
}

}  // namespace

int launch_bucket_sort(const uint32_t* d_offsets, uint32_t n_indices, const uint8_t* d_count0,
                       int64_t n, int shift, int n_buckets, void* ws, cudaStream_t s) {
  WorkspaceView v = carve_workspace(ws, n);
  CNNUE_CUDA_TRY(cudaMemsetAsync(v.hdr, 0, sizeof(WorkspaceHeader), s));
  const int threads = 256;
  const unsigned blocks = (unsigned)((n + threads - 1) / threads);
  bucket_count_kernel<<<blocks, threads, 0, s>>>(d_offsets, n_indices, d_count0, n, shift,
                                                  n_buckets - 1, v.bucket_of, v.hdr);
  int st = check_launch("bucket_count_kernel");
  if (st) return st;
  bucket_scatter_kernel<<<blocks, threads, 0, s>>>(n, n_buckets, v.bucket_of, v.hdr, v.perm,
                                                    v.sorted_bucket);
  return check_launch("bucket_scatter_kernel");
}

int launch_offsets_check(const uint32_t* d_offsets, uint32_t n_values, int64_t n_lists, void* ws,
                         cudaStream_t s) {
  WorkspaceView v = carve_workspace(ws, 0);
  const int threads = 256;
  const unsigned blocks = (unsigned)((n_lists + threads - 1) / threads);
  offsets_check_kernel<<<blocks, threads, 0, s>>>(d_offsets, n_values, n_lists, v.hdr);
  return check_launch("offsets_check_kernel");
}

}  // namespace cnnue
