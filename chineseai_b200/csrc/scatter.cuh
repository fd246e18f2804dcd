// scatter.cuh - deterministic scatter-add into large scalar tables:
//   out[k] = sum, in contribution order, of values[i] over every i with
//   keys[i] == k  (out[k] = 0 for keys nobody hits),
// for tables too large for per-chunk row histograms (the 2.4 M-entry policy
// sparse table, the 183 K-entry fused policy table, the 57,702 x 64 threat
// table as scalars).  The reference's CPU twins add contributions one at a
// time in enumeration order; that order is kept per key.
//
//   1. LSD radix sort of (key, contribution index) pairs, 8-bit digits, as
//      many passes as the key width needs; each pass is a stable counting
//      sort: per-block digit histograms, one scan kernel (digit starts and
//      per-block offsets), and a scatter in which each block ranks its items
//      digit by digit with __match_any_sync inside warps and per-warp counts
//      in shared memory, walking its items in order (so the sort is stable);
//   2. runs of equal keys are found (flags + a scan) and split into units of
//      at most 256 contributions; one thread sums a unit in index order, and
//      each key adds its units' partials in order.  A key with at most 256
//      contributions is thus summed exactly in contribution order; longer
//      runs are still deterministic.  Keys with no contribution read zero.
// Nothing is read back to the host: run and unit counts stay in device
// memory and the kernels after them loop up to those counts, so a scatter is
// asynchronous and can be captured in a CUDA graph.
// The row form (launch_scatter_add_rows) does the same for whole table rows:
// a contribution adds a `hidden`-wide row of values, one warp sums a unit
// with its lanes over the columns, and a key with a single unit is written
// directly.
#pragma once

#include "common.cuh"

namespace cnnue {
namespace scat {
namespace {

constexpr int kThreads = 256;
constexpr int kItemsPerThread = 4;
constexpr int kBlockItems = kThreads * kItemsPerThread;  // 1024
constexpr int kDigits = 256;
constexpr unsigned kFull = 0xffffffffu;

inline int64_t n_blocks(int64_t n) { return (n + kBlockItems - 1) / kBlockItems; }

inline int key_passes(int64_t n_keys) {
  int bits = 1;
  while (bits < 32 && ((int64_t)1 << bits) < n_keys) ++bits;
  return (bits + 7) / 8;
}

// ---- generic exclusive scan of uint32 (three levels, in place) ------------
constexpr int kScanBlock = 1024;  // elements per CTA (256 threads x 4)

__global__ void __launch_bounds__(256) scan_blocks_kernel(uint32_t* __restrict__ a, int64_t n,
                                                          uint32_t* __restrict__ sums) {
  __shared__ uint32_t ws[8];
  const int64_t base = (int64_t)blockIdx.x * kScanBlock + threadIdx.x * 4;
  uint32_t v[4], t = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[k] = base + k < n ? a[base + k] : 0u;
    t += v[k];
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = t;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += x;
  }
  if (lane == 31) ws[warp] = incl;
  __syncthreads();
  uint32_t wbase = 0;
  for (int w = 0; w < warp; ++w) wbase += ws[w];
  uint32_t run = wbase + incl - t;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (base + k < n) a[base + k] = run;
    run += v[k];
  }
  if (threadIdx.x == 255) sums[blockIdx.x] = wbase + incl;
}

__global__ void __launch_bounds__(256) add_blocks_kernel(uint32_t* __restrict__ a, int64_t n,
                                                         const uint32_t* __restrict__ offs) {
  const int64_t base = (int64_t)blockIdx.x * kScanBlock + threadIdx.x * 4;
  const uint32_t o = offs[blockIdx.x];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (base + k < n) a[base + k] += o;
}

inline int64_t scan_aux_len(int64_t n) { return (n + kScanBlock - 1) / kScanBlock; }
inline size_t scan_bytes(int64_t n) {
  int64_t total = 0, m = n;
  while (m > 1) {
    m = scan_aux_len(m);
    total += m + 1;
  }
  return align_up((size_t)(total + 1) * 4, 256);
}

// Exclusive scan of a[0..n) in place; aux holds scan_bytes(n) (the per-CTA
// sums of every level).
int launch_scan(uint32_t* a, int64_t n, uint32_t* aux, cudaStream_t s) {
  if (n <= 0) return CNNUE_OK;
  const int64_t nb = scan_aux_len(n);
  scan_blocks_kernel<<<(unsigned)nb, 256, 0, s>>>(a, n, aux);
  if (int st = check_launch_error("scan_blocks")) return st;
  if (nb > 1) {
    if (int st = launch_scan(aux, nb, aux + nb + 1, s)) return st;
    add_blocks_kernel<<<(unsigned)nb, 256, 0, s>>>(a, n, aux);
    if (int st = check_launch_error("add_blocks")) return st;
  }
  return CNNUE_OK;
}

// ---- radix sort -------------------------------------------------------------
// n_dev (optional): the live item count in device memory (<= n); keys >=
// drop_key are skipped (as items past the end).
__global__ void __launch_bounds__(kThreads) hist_kernel(const uint32_t* __restrict__ keys, int64_t n, int shift,
                                                        int64_t nb, uint32_t* __restrict__ hist,
                                                        const uint32_t* __restrict__ n_dev = nullptr,
                                                        uint32_t drop_key = 0xffffffffu) {
  __shared__ uint32_t h[kDigits];
  h[threadIdx.x] = 0;
  if (n_dev && (int64_t)*n_dev < n) n = (int64_t)*n_dev;
  __syncthreads();
  const int64_t base = (int64_t)blockIdx.x * kBlockItems;
#pragma unroll
  for (int r = 0; r < kItemsPerThread; ++r) {
    const int64_t i = base + r * kThreads + threadIdx.x;
    if (i < n) {
      const uint32_t k = keys[i];
      if (k < drop_key) atomicAdd(&h[(k >> shift) & 0xffu], 1u);  // counts are order-free
    }
  }
  __syncthreads();
  hist[(size_t)threadIdx.x * nb + blockIdx.x] = h[threadIdx.x];  // digit-major
}

// Stable scatter of one block's items: rounds of 256 items in order; inside a
// round, warp w's items come before warp w+1's and lanes in order.
__global__ void __launch_bounds__(kThreads) scatter_kernel(const uint32_t* __restrict__ keys_in,
                                                           const uint32_t* __restrict__ idx_in, int64_t n,
                                                           int shift, int64_t nb, const uint32_t* __restrict__ hist,
                                                           uint32_t* __restrict__ keys_out,
                                                           uint32_t* __restrict__ idx_out,
                                                           const uint32_t* __restrict__ n_dev = nullptr,
                                                           uint32_t drop_key = 0xffffffffu) {
  constexpr int kWarps = kThreads / 32;
  if (n_dev && (int64_t)*n_dev < n) n = (int64_t)*n_dev;
  __shared__ uint32_t base[kDigits];
  __shared__ uint32_t wcount[kWarps][kDigits];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  base[threadIdx.x] = hist[(size_t)threadIdx.x * nb + blockIdx.x];
  const int64_t b0 = (int64_t)blockIdx.x * kBlockItems;
  for (int r = 0; r < kItemsPerThread; ++r) {
    for (int i = threadIdx.x; i < kWarps * kDigits; i += kThreads) (&wcount[0][0])[i] = 0;
    __syncthreads();
    const int64_t i = b0 + r * kThreads + threadIdx.x;
    const uint32_t key = i < n ? keys_in[i] : 0u;
    const bool valid = i < n && key < drop_key;
    const uint32_t dig = valid ? (key >> shift) & 0xffu : 0x100u;  // 256 = no item
    const uint32_t peers = __match_any_sync(kFull, dig);
    const uint32_t rank = __popc(peers & ((1u << lane) - 1u));
    if (valid && lane == __ffs(peers) - 1) wcount[warp][dig] = __popc(peers);
    __syncthreads();
    if (valid) {
      uint32_t before = 0;
      for (int w = 0; w < warp; ++w) before += wcount[w][dig];
      const uint32_t slot = base[dig] + before + rank;
      if (slot < (uint64_t)n) {  // a self-check: the slots of n items are < n
        keys_out[slot] = key;
        idx_out[slot] = idx_in ? idx_in[i] : (uint32_t)i;
      }
    }
    __syncthreads();
    uint32_t add = 0;
    for (int w = 0; w < kWarps; ++w) add += wcount[w][threadIdx.x];
    base[threadIdx.x] += add;
    __syncthreads();
  }
}

// ---- segmented sums over the sorted runs ------------------------------------
constexpr int kUnit = 256;

__global__ void zero_kernel(float* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = 0.f;
}

// flag[i] = 1 at the start of a run of equal keys, flag[n] = 0 (scanned to
// run ids; the scan's entry n is then the run count).
__global__ void run_flag_kernel(const uint32_t* __restrict__ keys, int64_t n, uint32_t* __restrict__ flag) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i <= n; i += (int64_t)gridDim.x * blockDim.x)
    flag[i] = i == n ? 0u : ((i == 0 || keys[i] != keys[i - 1]) ? 1u : 0u);
}

// After the scan flag[i] is the number of runs starting before i; run starts
// record themselves, then each run its unit count.
__global__ void run_start_kernel(const uint32_t* __restrict__ keys, int64_t n, const uint32_t* __restrict__ run_of,
                                 uint32_t* __restrict__ run_start) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    if (i == 0 || keys[i] != keys[i - 1]) run_start[run_of[i]] = (uint32_t)i;
}

// units[r] = the unit count of run r (0 past the last run, up to entry n;
// the scan's entry n is then the unit count).
__global__ void run_units_kernel(const uint32_t* __restrict__ run_start, const uint32_t* __restrict__ n_runs_d,
                                 int64_t n, uint32_t unit, uint32_t* __restrict__ units) {
  const uint32_t n_runs = *n_runs_d;
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r <= n; r += (int64_t)gridDim.x * blockDim.x) {
    if (r < n_runs) {
      const uint32_t beg = run_start[r], end = r + 1 < n_runs ? run_start[r + 1] : (uint32_t)n;
      units[r] = (end - beg + unit - 1) / unit;
    } else {
      units[r] = 0;
    }
  }
}

// One thread per unit: the unit's <= 256 contributions in order, loads
// issued eight at a time.  Units of the drop key are skipped.
__global__ void unit_sum_kernel(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ idx,
                                const float* __restrict__ values, uint32_t div, int64_t n_keys,
                                const uint32_t* __restrict__ run_start, const uint32_t* __restrict__ unit_off,
                                const uint32_t* __restrict__ n_runs_d, const uint32_t* __restrict__ n_units_d,
                                int64_t n, float* __restrict__ partial) {
  const uint32_t n_runs = *n_runs_d, n_units = *n_units_d;
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < n_units; u += (int64_t)gridDim.x * blockDim.x) {
    // the run of unit u: last r with unit_off[r] <= u
    uint32_t lo = 0, hi = n_runs - 1;
    while (lo < hi) {
      const uint32_t mid = (lo + hi + 1) >> 1;
      if (unit_off[mid] <= (uint32_t)u) lo = mid;
      else hi = mid - 1;
    }
    const uint32_t r = lo;
    const uint32_t rbeg = run_start[r], rend = r + 1 < n_runs ? run_start[r + 1] : (uint32_t)n;
    if ((int64_t)keys[rbeg] >= n_keys) continue;
    const uint32_t beg = rbeg + ((uint32_t)u - unit_off[r]) * kUnit;
    const uint32_t end = min(rend, beg + kUnit);
    float s = 0.f;
    uint32_t j = beg;
    for (; j + 8 <= end; j += 8) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = __ldg(values + __ldg(idx + j + k) / div);
#pragma unroll
      for (int k = 0; k < 8; ++k) s += v[k];
    }
    for (; j < end; ++j) s += __ldg(values + __ldg(idx + j) / div);
    partial[u] = s;
  }
}

// Each run adds its unit partials in order and writes its key.
__global__ void run_sum_kernel(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ run_start,
                               const uint32_t* __restrict__ unit_off, const uint32_t* __restrict__ n_runs_d,
                               const uint32_t* __restrict__ n_units_d, const float* __restrict__ partial,
                               int64_t n_keys, float* __restrict__ out) {
  const uint32_t n_runs = *n_runs_d, n_units = *n_units_d;
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n_runs; r += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t k = keys[run_start[r]];
    if ((int64_t)k >= n_keys) continue;  // key n_keys: dropped contributions
    const uint32_t u0 = unit_off[r], u1 = r + 1 < n_runs ? unit_off[r + 1] : n_units;
    float s = partial[u0];
    for (uint32_t u = u0 + 1; u < u1; ++u) s += partial[u];
    out[k] = s;
  }
}

// Row form: one warp per (unit, 32-column block); lanes own one column each.
// A unit that is its run's only one writes the table row directly.  Val(e, h)
// gives column h of contribution e; Out(key, h) the output element.
template <class Val, class Out>
__global__ void unit_sum_rows_kernel(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ idx, Val val,
                                     int64_t hidden, const uint32_t* __restrict__ run_start,
                                     const uint32_t* __restrict__ unit_off, const uint32_t* __restrict__ n_runs_d,
                                     const uint32_t* __restrict__ n_units_d, int64_t n, int64_t n_keys,
                                     float* __restrict__ partial, Out out) {
  const uint32_t n_runs = *n_runs_d, n_units = *n_units_d;
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t col_blocks = (hidden + 31) >> 5;
  for (int64_t q = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; q < (int64_t)n_units * col_blocks;
       q += warps) {
    const int64_t u = q / col_blocks, h = (q - u * col_blocks) * 32 + lane;
    uint32_t lo = 0, hi = n_runs - 1;
    while (lo < hi) {
      const uint32_t mid = (lo + hi + 1) >> 1;
      if (unit_off[mid] <= (uint32_t)u) lo = mid;
      else hi = mid - 1;
    }
    const uint32_t r = lo;
    const uint32_t rbeg = run_start[r], rend = r + 1 < n_runs ? run_start[r + 1] : (uint32_t)n;
    const uint32_t u1 = r + 1 < n_runs ? unit_off[r + 1] : n_units;
    const uint32_t beg = rbeg + ((uint32_t)u - unit_off[r]) * kUnit;
    const uint32_t end = min(rend, beg + kUnit);
    const uint32_t key = keys[rbeg];
    const bool single = u1 - unit_off[r] == 1;
    if ((int64_t)key >= n_keys || h >= hidden) continue;  // dropped contributions: never evaluated
    float s = 0.f;
    uint32_t j = beg;
    for (; j + 8 <= end; j += 8) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = val(__ldg(idx + j + k), h);
#pragma unroll
      for (int k = 0; k < 8; ++k) s += v[k];
    }
    for (; j < end; ++j) s += val(__ldg(idx + j), h);
    if (single) out(key, h) = s;
    else partial[u * hidden + h] = s;
  }
}

// Runs of several units add their partial rows in order (one thread per
// (run, column); single-unit runs were written by unit_sum_rows_kernel).
template <class Out>
__global__ void run_sum_rows_kernel(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ run_start,
                                    const uint32_t* __restrict__ unit_off, const uint32_t* __restrict__ n_runs_d,
                                    const uint32_t* __restrict__ n_units_d, const float* __restrict__ partial,
                                    int64_t hidden, int64_t n_keys, Out out) {
  const uint32_t n_runs = *n_runs_d, n_units = *n_units_d;
  const int64_t total = (int64_t)n_runs * hidden;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < total; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = q / hidden, h = q - r * hidden;
    const uint32_t u0 = unit_off[r], u1 = r + 1 < n_runs ? unit_off[r + 1] : n_units;
    if (u1 - u0 < 2) continue;
    const uint32_t k = keys[run_start[r]];
    if ((int64_t)k >= n_keys) continue;
    float s = partial[(int64_t)u0 * hidden + h];
    for (uint32_t u = u0 + 1; u < u1; ++u) s += partial[(int64_t)u * hidden + h];
    out(k, h) = s;
  }
}

// Values of a plain row-major buffer: contribution e adds row e / div.
struct BufferRows {
  const float* values;
  uint32_t div;
  int64_t hidden;
  __device__ __forceinline__ float operator()(uint32_t e, int64_t h) const {
    return __ldg(values + (int64_t)(e / div) * hidden + h);
  }
};
// A dense row-major table out[key][hidden].
struct DenseRows {
  float* out;
  int64_t hidden;
  __device__ __forceinline__ float& operator()(uint32_t key, int64_t h) const { return out[(int64_t)key * hidden + h]; }
};

// Workspace of launch_scatter_add(_rows) for n contributions of `hidden`
// values each.
inline size_t workspace_bytes(int64_t n, int64_t hidden = 1) {
  const size_t nn = (size_t)(n > 0 ? n : 1);
  const int64_t nb = n_blocks(n > 0 ? n : 1);
  size_t b = 4 * align_up(nn * 4, 256);                       // keys / idx ping-pong
  b += align_up((size_t)nb * kDigits * 4, 256);               // histograms
  b += scan_bytes(std::max<int64_t>((int64_t)nb * kDigits, (int64_t)nn + 1));  // scan scratch
  b += 3 * align_up((nn + 1) * 4, 256);                       // flags / run starts / unit offsets
  b += align_up((nn + 1) * 4 * (size_t)hidden, 256);          // unit partials
  b += 256;
  return b;
}

// The sorted contributions and their runs and units.
struct Runs {
  const uint32_t* keys;   // [n] sorted keys
  const uint32_t* idx;    // [n] contribution index of each sorted slot
  uint32_t* run_start;    // [n_runs]
  uint32_t* unit_off;     // [n_runs] first unit of each run
  float* partial;         // unit partials
  const uint32_t* n_runs;   // device word: number of runs
  const uint32_t* n_units;  // device word: number of units
  const uint32_t* run_of;   // [n + 1]: at a run's first slot, the run's index
};

// Sorts (key, contribution) pairs stably by key and finds runs and units of
// at most `unit` contributions (counts left in device memory).  Requires
// 0 < n < 2^32 - 1.
// Workspace of radix_sort for n pairs.
inline size_t sort_bytes(int64_t n) {
  const size_t nn = (size_t)(n > 0 ? n : 1);
  const int64_t nb = n_blocks(n > 0 ? n : 1);
  return 4 * align_up(nn * 4, 256) + align_up((size_t)nb * kDigits * 4, 256) + scan_bytes((int64_t)nb * kDigits);
}

// Stable LSD radix sort of (key, contribution index) pairs by key, as many
// 8-bit passes as keys <= n_keys need; the sorted keys and indices are left
// in ws (*keys_out, *idx_out).  Requires 0 < n < 2^32 - 1.  With d_live
// (the number of keys below drop_key, in device memory) the first pass
// drops the keys >= drop_key and the later passes sort the d_live others.
// payload (optional): what the sorted slots carry instead of the items'
// indices.
int radix_sort(const uint32_t* keys, int64_t n, int64_t n_keys, void* ws, cudaStream_t s,
               const uint32_t** keys_out, const uint32_t** idx_out, const uint32_t* d_live = nullptr,
               uint32_t drop_key = 0xffffffffu, const uint32_t* payload = nullptr) {
  const size_t nn = (size_t)n;
  const int64_t nb = n_blocks(n);
  char* p = (char*)ws;
  auto take = [&](size_t bytes) {
    char* q = p;
    p += align_up(bytes, 256);
    return q;
  };
  uint32_t* k0 = (uint32_t*)take(nn * 4);
  uint32_t* k1 = (uint32_t*)take(nn * 4);
  uint32_t* i0 = (uint32_t*)take(nn * 4);
  uint32_t* i1 = (uint32_t*)take(nn * 4);
  uint32_t* hist = (uint32_t*)take((size_t)nb * kDigits * 4);
  uint32_t* aux = (uint32_t*)p;
  const int passes = key_passes(n_keys + 1);
  const uint32_t* kin = keys;
  const uint32_t* iin = payload;
  uint32_t* kout = k0;
  uint32_t* iout = i0;
  for (int pass = 0; pass < passes; ++pass) {
    const int shift = 8 * pass;
    const uint32_t* nd = pass > 0 ? d_live : nullptr;
    const uint32_t dk = pass == 0 && d_live ? drop_key : 0xffffffffu;
    hist_kernel<<<(unsigned)nb, kThreads, 0, s>>>(kin, n, shift, nb, hist, nd, dk);
    if (int st = check_launch_error("sort hist")) return st;
    if (int st = launch_scan(hist, nb * kDigits, aux, s)) return st;
    scatter_kernel<<<(unsigned)nb, kThreads, 0, s>>>(kin, iin, n, shift, nb, hist, kout, iout, nd, dk);
    if (int st = check_launch_error("sort scatter")) return st;
    kin = kout;
    iin = iout;
    kout = kout == k0 ? k1 : k0;
    iout = iout == i0 ? i1 : i0;
  }
  *keys_out = kin;
  *idx_out = iin;
  return CNNUE_OK;
}

int sort_runs(const uint32_t* keys, int64_t n, int64_t n_keys, void* ws, cudaStream_t s, Runs* out,
              uint32_t unit = kUnit) {
  const size_t nn = (size_t)n;
  const int64_t nb = n_blocks(n);
  char* p = (char*)ws;
  auto take = [&](size_t bytes) {
    char* q = p;
    p += align_up(bytes, 256);
    return q;
  };
  uint32_t* k0 = (uint32_t*)take(nn * 4);
  uint32_t* k1 = (uint32_t*)take(nn * 4);
  uint32_t* i0 = (uint32_t*)take(nn * 4);
  uint32_t* i1 = (uint32_t*)take(nn * 4);
  uint32_t* hist = (uint32_t*)take((size_t)nb * kDigits * 4);
  uint32_t* aux = (uint32_t*)take(scan_bytes(std::max<int64_t>((int64_t)nb * kDigits, (int64_t)nn + 1)));
  uint32_t* flag = (uint32_t*)take((nn + 1) * 4);
  uint32_t* rstart = (uint32_t*)take((nn + 1) * 4);
  uint32_t* uoff = (uint32_t*)take((nn + 1) * 4);
  out->partial = (float*)p;
  const int passes = key_passes(n_keys + 1);
  const uint32_t* kin = keys;
  const uint32_t* iin = nullptr;
  uint32_t* kout = k0;
  uint32_t* iout = i0;
  for (int pass = 0; pass < passes; ++pass) {
    const int shift = 8 * pass;
    hist_kernel<<<(unsigned)nb, kThreads, 0, s>>>(kin, n, shift, nb, hist);
    if (int st = check_launch_error("scatter hist")) return st;
    if (int st = launch_scan(hist, nb * kDigits, aux, s)) return st;
    scatter_kernel<<<(unsigned)nb, kThreads, 0, s>>>(kin, iin, n, shift, nb, hist, kout, iout);
    if (int st = check_launch_error("scatter scatter")) return st;
    kin = kout;
    iin = iout;
    kout = kout == k0 ? k1 : k0;
    iout = iout == i0 ? i1 : i0;
  }
  const unsigned gb = (unsigned)std::min<int64_t>((n + 256) / 256, 148 * 16);
  run_flag_kernel<<<gb, 256, 0, s>>>(kin, n, flag);
  if (int st = check_launch_error("scatter flags")) return st;
  if (int st = launch_scan(flag, n + 1, aux, s)) return st;  // run ids; flag[n] = run count
  run_start_kernel<<<gb, 256, 0, s>>>(kin, n, flag, rstart);
  if (int st = check_launch_error("scatter run starts")) return st;
  run_units_kernel<<<gb, 256, 0, s>>>(rstart, flag + n, n, unit, uoff);
  if (int st = check_launch_error("scatter run units")) return st;
  if (int st = launch_scan(uoff, n + 1, aux, s)) return st;  // unit offsets; uoff[n] = unit count
  out->keys = kin;
  out->idx = iin;
  out->run_start = rstart;
  out->unit_off = uoff;
  out->n_runs = flag + n;
  out->n_units = uoff + n;
  out->run_of = flag;
  return CNNUE_OK;
}

// out[k] = sum over i (in index order, in units of 256 per key) of
// values[i / div] with keys[i] == k; keys nobody hits read 0.  Every key must
// be <= n_keys (the sort covers only those bits); key n_keys marks a
// contribution to drop (callers map padding and out-of-range indices to it).
int launch_scatter_add(const uint32_t* keys, const float* values, uint32_t div, int64_t n, int64_t n_keys,
                       float* out, void* ws, cudaStream_t s) {
  const unsigned zb = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n_keys + 255) / 256, 148 * 8));
  zero_kernel<<<zb, 256, 0, s>>>(out, n_keys);
  if (int st = check_launch_error("scatter zero")) return st;
  if (n <= 0) return CNNUE_OK;
  if (n >= (int64_t)UINT32_MAX) return set_error(CNNUE_ERR_INVALID_ARG, "too many contributions");
  Runs r;
  if (int st = sort_runs(keys, n, n_keys, ws, s, &r)) return st;
  // grids for the upper bounds (units, runs <= n); the kernels stop at the counts
  const unsigned gb = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 16));
  unit_sum_kernel<<<gb, 256, 0, s>>>(r.keys, r.idx, values, div, n_keys, r.run_start, r.unit_off, r.n_runs,
                                     r.n_units, n, r.partial);
  if (int st = check_launch_error("scatter unit sums")) return st;
  run_sum_kernel<<<gb, 256, 0, s>>>(r.keys, r.run_start, r.unit_off, r.n_runs, r.n_units, r.partial, n_keys, out);
  return check_launch_error("scatter run sums");
}

// Row form over functors: for every key k < n_keys hit by a contribution,
// out(k, h) = sum over contributions e with keys[e] == k (in order, units of
// 256) of val(e, h).  Rows nobody hits are not written (the caller zeroes
// them); keys must be <= n_keys, key n_keys is dropped.
template <class Val, class Out>
int launch_scatter_rows(const uint32_t* keys, Val val, Out out, int64_t hidden, int64_t n, int64_t n_keys, void* ws,
                        cudaStream_t s) {
  if (n <= 0) return CNNUE_OK;
  if (n >= (int64_t)UINT32_MAX) return set_error(CNNUE_ERR_INVALID_ARG, "too many contributions");
  Runs r;
  if (int st = sort_runs(keys, n, n_keys, ws, s, &r)) return st;
  // grids for the upper bounds (units, runs <= n); the kernels stop at the counts
  const unsigned ub =
      (unsigned)std::max<int64_t>(1, std::min<int64_t>((n * ((hidden + 31) / 32) * 32 + 255) / 256, 148 * 16));
  unit_sum_rows_kernel<<<ub, 256, 0, s>>>(r.keys, r.idx, val, hidden, r.run_start, r.unit_off, r.n_runs, r.n_units,
                                          n, n_keys, r.partial, out);
  if (int st = check_launch_error("scatter unit row sums")) return st;
  const unsigned rb = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n * hidden + 255) / 256, 148 * 16));
  run_sum_rows_kernel<<<rb, 256, 0, s>>>(r.keys, r.run_start, r.unit_off, r.n_runs, r.n_units, r.partial, hidden,
                                         n_keys, out);
  return check_launch_error("scatter run row sums");
}

// Dense form: out[k][h] = sum over i (same order) of values[(i / div) *
// hidden + h] with keys[i] == k, for a table out[n_keys][hidden] (zeroed
// first).
int launch_scatter_add_rows(const uint32_t* keys, const float* values, uint32_t div, int64_t hidden, int64_t n,
                            int64_t n_keys, float* out, void* ws, cudaStream_t s) {
  const int64_t total = n_keys * hidden;
  const unsigned zb = (unsigned)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, 148 * 8));
  zero_kernel<<<zb, 256, 0, s>>>(out, total);
  if (int st = check_launch_error("scatter zero")) return st;
  return launch_scatter_rows(keys, BufferRows{values, div, hidden}, DenseRows{out, hidden}, hidden, n, n_keys, ws, s);
}

}  // namespace
}  // namespace scat
}  // namespace cnnue
