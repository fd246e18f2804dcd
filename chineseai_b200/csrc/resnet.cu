// resnet.cu - AlphaZero policy/value ResNet inference for MCTS leaf batches
// (the dense tensor-core part of the evaluator).
//
// Trunk: 21 3x3 convolutions (stem 15->128, 10 residual blocks of two
// 128->128), each an implicit GEMM on the 5th-generation tensor cores:
// rows = board squares of the batch, columns = 128 output channels, K = 9
// taps x input channels.  Activations are bf16 with channels contiguous; the
// stem input is packed to 64 channels.  Three conv kernels compute the same
// convolution (cnnue_rn_set_conv_kernel): the default rn_hconv_kernel on a
// padded, 8-board-interleaved row layout (described at its definition), and
// two on the square-major layout ([B*90][C]) described here.
//
// rn_conv_kernel, one CTA per 128 x 128 output tile, 6 warps:
//   warp 4     allocates the 128 TMEM columns of the fp32 accumulator and
//              loads each 64-wide K block: the A tile (one tap, 64 channels
//              of 128 squares) with one 2-D TMA of the tap-shifted row range
//              (square-major rows make a tap a constant row shift), the B tile
//              with one bulk copy of weights pre-tiled in the same 128-byte
//              swizzled K-major layout;
//   warps 0-3  zero the rows whose tap leaves the board (a row is one
//              128-byte line of the swizzled tile), then are the epilogue
//              (TMEM -> registers, + bias (+ residual), ReLU, bf16, store);
//   warp 5     one thread issues tcgen05.mma (M128 N128 K16, 4 per K block)
//              and commits each stage back to its producers.
// A 3-stage ring of (16 KB A + 16 KB B) stages with three mbarriers each
// (loaded, ready, empty); every wait is bounded (1 s) and reports
// CNNUE_STATUS_TIMEOUT.  No load uses cluster multicast.
//
// Heads, fp32 on CUDA cores: rn_head_conv_kernel (1x1 convs to 2 policy and
// 1 value planes, two lanes per trunk row), rn_heads_kernel (its blocks are
// either policy FC 180 -> 2086 tiles of a tiled GEMM, 128 boards x 128 moves,
// or value FC 90 -> 256 -> 1 with tanh, 8 boards), rn_softmax_kernel (one
// warp per board, the row held in registers).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <mutex>

#include <cstring>
#include <new>
#include <vector>

#include "common.cuh"
#include "pipeline.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace cnnue {
namespace rn {
namespace {

constexpr int kSq = 90;
constexpr int kC = CNNUE_RN_CHANNELS;
constexpr int kMoves = CNNUE_RN_MOVES;
constexpr int kConvs = 1 + 2 * CNNUE_RN_BLOCKS;
constexpr int kTileM = 128;
constexpr int kTileBytes = 128 * 64 * 2;  // 128 rows x 64 bf16
constexpr int kStages = 3;
constexpr int kConvThreads = 192;
constexpr int kStemKb = 9;   // 9 taps x 64 (packed) channels / 64
constexpr int kBlockKb = 18; // 9 taps x 128 channels / 64

inline size_t conv_tile_offset(int conv) { return conv == 0 ? 0 : (size_t)kStemKb + (size_t)(conv - 1) * kBlockKb; }
constexpr size_t kTotalKb = kStemKb + (size_t)(kConvs - 1) * kBlockKb;

struct ConvSmem {
  alignas(1024) uint8_t a[kStages][kTileBytes];
  alignas(1024) uint8_t b[kStages][kTileBytes];
  uint64_t loaded[kStages];  // A (TMA) and B (bulk copy) bytes landed
  uint64_t ready[kStages];   // off-board rows of A zeroed
  uint64_t empty[kStages];   // the stage's MMAs completed
  uint64_t accum;
  uint32_t tmem_base;
  int abort;
};

// Byte offset of (row, k) inside a 128 x 64 bf16 tile in the 128B-swizzled
// K-major layout: row r is the 128-byte line r, its 16-byte chunk c is stored
// at chunk position c ^ (r % 8).
__host__ __device__ constexpr uint32_t tile_offset(int row, int k) {
  return (uint32_t)(row * 128 + ((((k >> 3) ^ row) & 7) << 4) + (k & 7) * 2);
}

template <int CIN>
__global__ void __launch_bounds__(kConvThreads) rn_conv_kernel(const __grid_constant__ CUtensorMap tmap_in,
                                                               const uint8_t* __restrict__ wtiles,
                                                               const float* __restrict__ bias,
                                                               const __nv_bfloat16* __restrict__ resid,
                                                               __nv_bfloat16* __restrict__ out, int M,
                                                               uint32_t* status) {
  constexpr int kKbPerTap = CIN / 64;
  constexpr int kKb = 9 * kKbPerTap;
  extern __shared__ uint8_t smem_raw[];
  ConvSmem& sm = *reinterpret_cast<ConvSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * kTileM;

  if (warp == 4) {
    tc::tmem_alloc(pipe::smem_addr(&sm.tmem_base), 128);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      pipe::mbar_init(&sm.loaded[s], 1);
      pipe::mbar_init(&sm.ready[s], 128);
      pipe::mbar_init(&sm.empty[s], 1);
    }
    pipe::mbar_init(&sm.accum, 1);
    sm.abort = 0;
    pipe::mbar_init_fence();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;

  if (warp < 4) {
    // ---- edge fix-up: the TMA copied rows m0+shift .. m0+shift+127 of the
    // activations; row t whose tap leaves the board must read zeros.
    const int row = tid, m = m0 + row;
    const int p = (m < M ? m : 0) % kSq, r = p / 9, f = p - (p / 9) * 9;
    for (int kb = 0; kb < kKb; ++kb) {
      const int s = kb % kStages, u = kb / kStages;
      if (!pipe::mbar_wait(&sm.loaded[s], u & 1, &sm.abort, status)) break;
      const int tap = kb % 9;
      const int r2 = r + tap / 3 - 1, f2 = f + tap % 3 - 1;
      if (m < M && (r2 < 0 || r2 > 9 || f2 < 0 || f2 > 8)) {
        uint8_t* line = sm.a[s] + row * 128;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          *reinterpret_cast<uint4*>(line + (((i + row) & 7) << 4)) = make_uint4(0u, 0u, 0u, 0u);
      }
      pipe::fence_proxy_async_smem();
      pipe::mbar_arrive(&sm.ready[s]);
    }
    // ---- epilogue: TMEM lane = row.
    const bool ok = pipe::mbar_wait(&sm.accum, 0, &sm.abort, status);
    tc::fence_after_sync();
    const uint32_t taddr = tmem + ((uint32_t)(32 * warp) << 16);
    const bool active = ok && m < M;
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      uint32_t v[32];
      __syncwarp();  // converged for the .sync.aligned TMEM load
      tc::tmem_ld32(taddr + 32 * j, v);
      tc::wait_ld();
      if (!active) continue;
      float res[32];
      if (resid != nullptr) {
        const uint4* rp = reinterpret_cast<const uint4*>(resid + (size_t)m * kC + 32 * j);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 w = __ldg(rp + q);
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&ws[e]);
            res[8 * q + 2 * e] = __bfloat162float(h2.x);
            res[8 * q + 2 * e + 1] = __bfloat162float(h2.y);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) res[i] = 0.f;
      }
      uint32_t packed[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float x0 = __uint_as_float(v[2 * i]) + __ldg(bias + 32 * j + 2 * i) + res[2 * i];
        float x1 = __uint_as_float(v[2 * i + 1]) + __ldg(bias + 32 * j + 2 * i + 1) + res[2 * i + 1];
        x0 = fmaxf(x0, 0.f);
        x1 = fmaxf(x1, 0.f);
        const __nv_bfloat162 h2 = __floats2bfloat162_rn(x0, x1);
        packed[i] = *reinterpret_cast<const uint32_t*>(&h2);
      }
      uint4* op = reinterpret_cast<uint4*>(out + (size_t)m * kC + 32 * j);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        op[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
    }
  } else if (warp == 4) {
    // ---- loads: A by one 2-D TMA of the tap-shifted rows (zeros past the
    // buffer's ends), B by one bulk copy of the pre-tiled weights.
    if (lane == 0) {
      for (int kb = 0; kb < kKb; ++kb) {
        const int s = kb % kStages, u = kb / kStages;
        if (u > 0 && !pipe::mbar_wait(&sm.empty[s], (u - 1) & 1, &sm.abort, status)) break;
        const int tap = kb % 9, c0 = (kb / 9) * 64;
        const int shift = (tap / 3 - 1) * 9 + (tap % 3 - 1);
        pipe::mbar_arrive_expect_tx(&sm.loaded[s], 2 * kTileBytes);
        tc::tma_load_2d(pipe::smem_addr(sm.a[s]), &tmap_in, c0, m0 + shift, pipe::smem_addr(&sm.loaded[s]));
        pipe::bulk_copy_g2s(sm.b[s], wtiles + (size_t)kb * kTileBytes, kTileBytes, &sm.loaded[s]);
      }
    }
    __syncwarp();
  } else {
    // ---- MMA issuer.
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(128, 128);
      for (int kb = 0; kb < kKb; ++kb) {
        const int s = kb % kStages, u = kb / kStages;
        if (!pipe::mbar_wait(&sm.ready[s], u & 1, &sm.abort, status)) break;
        tc::fence_after_sync();
        const uint32_t a0 = pipe::smem_addr(sm.a[s]), b0 = pipe::smem_addr(sm.b[s]);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = tc::smem_desc(a0 + kk * 32, 0, 1024, tc::kSwizzle128B);
          const uint64_t bd = tc::smem_desc(b0 + kk * 32, 0, 1024, tc::kSwizzle128B);
          tc::mma_bf16(tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
        }
        tc::commit(pipe::smem_addr(&sm.empty[s]));
      }
      tc::commit(pipe::smem_addr(&sm.accum));
    }
    __syncwarp();
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 4) tc::tmem_dealloc(tmem, 128);
}

// ---- persistent variant: two M tiles per K block, double-buffered TMEM ----
// One CTA per SM loops over pairs of 128-row tiles.  Per K block the loader
// issues two A boxes (one per tile) and one B tile, so each 16 KB weight tile
// feeds 8 MMAs; a 4-stage ring of 48 KB stages hides load latency, and the
// two 256-column TMEM buffers let the epilogue of one pair overlap the main
// loop of the next.  Warps: 0 loader, 1 MMA issuer (and TMEM owner), 2-5
// edge fix-up (rows t and 128 + t), 6-13 epilogue (warps 6-9 the first tile,
// 10-13 the second; TMEM lane quadrant w % 4), with the bias in shared memory
// and each row's residual loads issued before its TMEM reads.
constexpr int kPStages = 4;
constexpr int kPThreads = 448;  // 14 warps

struct PConvSmem {
  alignas(1024) uint8_t a[kPStages][2][kTileBytes];
  alignas(1024) uint8_t b[kPStages][kTileBytes];
  uint64_t loaded[kPStages];
  uint64_t ready[kPStages];
  uint64_t empty[kPStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  float bias[CNNUE_RN_CHANNELS];
  uint32_t tmem_base;
  int abort;
};

template <int CIN>
__global__ void __launch_bounds__(kPThreads, 1) rn_pconv_kernel(const __grid_constant__ CUtensorMap tmap_in,
                                                               const uint8_t* __restrict__ wtiles,
                                                               const float* __restrict__ bias,
                                                               const __nv_bfloat16* __restrict__ resid,
                                                               __nv_bfloat16* __restrict__ out, int M,
                                                               uint32_t* status) {
  constexpr int kKbPerTap = CIN / 64;
  constexpr int kKb = 9 * kKbPerTap;
  extern __shared__ uint8_t smem_raw[];
  PConvSmem& sm = *reinterpret_cast<PConvSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_pairs = (M + 2 * kTileM - 1) / (2 * kTileM);

  if (warp == 1) {
    tc::tmem_alloc(pipe::smem_addr(&sm.tmem_base), 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < kPStages; ++s) {
      pipe::mbar_init(&sm.loaded[s], 1);
      pipe::mbar_init(&sm.ready[s], 128);
      pipe::mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      pipe::mbar_init(&sm.acc_full[b], 1);
      pipe::mbar_init(&sm.acc_empty[b], 256);
    }
    sm.abort = 0;
    pipe::mbar_init_fence();
  }
  if (tid < kC) sm.bias[tid] = bias[tid];
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ---- loader
    if (lane == 0) {
      uint32_t g = 0;
      for (int pair = blockIdx.x; pair < n_pairs; pair += gridDim.x) {
        const int m0 = pair * 2 * kTileM;
        for (int kb = 0; kb < kKb; ++kb, ++g) {
          const uint32_t s = g % kPStages, u = g / kPStages;
          if (u > 0 && !pipe::mbar_wait(&sm.empty[s], (u - 1) & 1, &sm.abort, status)) goto done_load;
          const int tap = kb % 9, c0 = (kb / 9) * 64;
          const int shift = (tap / 3 - 1) * 9 + (tap % 3 - 1);
          pipe::mbar_arrive_expect_tx(&sm.loaded[s], 3 * kTileBytes);
          tc::tma_load_2d(pipe::smem_addr(sm.a[s][0]), &tmap_in, c0, m0 + shift, pipe::smem_addr(&sm.loaded[s]));
          tc::tma_load_2d(pipe::smem_addr(sm.a[s][1]), &tmap_in, c0, m0 + kTileM + shift,
                          pipe::smem_addr(&sm.loaded[s]));
          pipe::bulk_copy_g2s(sm.b[s], wtiles + (size_t)kb * kTileBytes, kTileBytes, &sm.loaded[s]);
        }
      }
    done_load:;
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(128, 128);
      uint32_t g = 0;
      int it = 0;
      for (int pair = blockIdx.x; pair < n_pairs; pair += gridDim.x, ++it) {
        const int buf = it & 1, use = it >> 1;
        if (use > 0 && !pipe::mbar_wait(&sm.acc_empty[buf], (use - 1) & 1, &sm.abort, status)) break;
        tc::fence_after_sync();
        const uint32_t d0 = tmem + (uint32_t)(buf * 256), d1 = d0 + 128;
        bool ok = true;
        // K blocks two at a time: both stages' waits, one fence, 16 MMAs,
        // then both stages released (one fence per 1024 cycles of MMA work)
        for (int kb = 0; kb < kKb; kb += 2) {
          const int nk = kb + 1 < kKb ? 2 : 1;
          for (int j = 0; j < nk; ++j) {
            const uint32_t s = (g + j) % kPStages, u = (g + j) / kPStages;
            if (!pipe::mbar_wait(&sm.ready[s], u & 1, &sm.abort, status)) {
              ok = false;
              break;
            }
          }
          if (!ok) break;
          tc::fence_after_sync();
          for (int j = 0; j < nk; ++j) {
            const uint32_t s = (g + j) % kPStages;
            const uint32_t a0 = pipe::smem_addr(sm.a[s][0]), a1 = pipe::smem_addr(sm.a[s][1]);
            const uint32_t b0 = pipe::smem_addr(sm.b[s]);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t bd = tc::smem_desc(b0 + kk * 32, 0, 1024, tc::kSwizzle128B);
              const uint32_t acc = ((kb + j) | kk) != 0 ? 1u : 0u;
              tc::mma_bf16(d0, tc::smem_desc(a0 + kk * 32, 0, 1024, tc::kSwizzle128B), bd, idesc, acc);
              tc::mma_bf16(d1, tc::smem_desc(a1 + kk * 32, 0, 1024, tc::kSwizzle128B), bd, idesc, acc);
            }
            tc::commit(pipe::smem_addr(&sm.empty[s]));
          }
          g += nk;
        }
        tc::commit(pipe::smem_addr(&sm.acc_full[buf]));
        if (!ok) break;
      }
    }
    __syncwarp();
  } else if (warp < 6) {
    // ---- edge fix-up: rows t and 128 + t of the two A boxes
    const int t = tid - 64;
    int r[2], f[2];
    bool live[2];
    uint32_t g = 0;
    for (int pair = blockIdx.x; pair < n_pairs; pair += gridDim.x) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int m = pair * 2 * kTileM + h * kTileM + t;
        live[h] = m < M;
        const int p = (live[h] ? m : 0) % kSq;
        r[h] = p / 9;
        f[h] = p - r[h] * 9;
      }
      bool ok = true;
      for (int kb = 0; kb < kKb; ++kb, ++g) {
        const uint32_t s = g % kPStages, u = g / kPStages;
        if (!pipe::mbar_wait(&sm.loaded[s], u & 1, &sm.abort, status)) {
          ok = false;
          break;
        }
        const int tap = kb % 9;
        const int dr = tap / 3 - 1, df = tap % 3 - 1;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r2 = r[h] + dr, f2 = f[h] + df;
          if (live[h] && (r2 < 0 || r2 > 9 || f2 < 0 || f2 > 8)) {
            uint8_t* line = sm.a[s][h] + t * 128;
#pragma unroll
            for (int i = 0; i < 8; ++i)
              *reinterpret_cast<uint4*>(line + (((i + t) & 7) << 4)) = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        pipe::fence_proxy_async_smem();
        pipe::mbar_arrive(&sm.ready[s]);
      }
      if (!ok) break;
    }
  } else {
    // ---- epilogue: warps 6-9 tile 0, 10-13 tile 1; TMEM lane quadrant w % 4
    const int h = (warp - 6) >> 2, q = warp & 3, row = q * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16);
    int it = 0;
    for (int pair = blockIdx.x; pair < n_pairs; pair += gridDim.x, ++it) {
      const int buf = it & 1, use = it >> 1;
      const int m = pair * 2 * kTileM + h * kTileM + row;
      // residual row first: its 16 loads overlap the accumulator wait
      uint4 rv[16];
      const bool in_range = m < M;
      if (resid != nullptr && in_range) {
        const uint4* rp = reinterpret_cast<const uint4*>(resid + (size_t)m * kC);
#pragma unroll
        for (int i = 0; i < 16; ++i) rv[i] = __ldg(rp + i);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) rv[i] = make_uint4(0u, 0u, 0u, 0u);
      }
      const bool ok = pipe::mbar_wait(&sm.acc_full[buf], use & 1, &sm.abort, status);
      tc::fence_after_sync();
      const bool active = ok && in_range;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t v[32];
        __syncwarp();
        tc::tmem_ld32(lane_addr + (uint32_t)(buf * 256 + h * 128 + 32 * j), v);
        tc::wait_ld();
        if (!active) continue;
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint32_t rw = (&rv[4 * j].x)[i];
          const float2 r2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rw));
          const float x0 = __uint_as_float(v[2 * i]) + sm.bias[32 * j + 2 * i] + r2.x;
          const float x1 = __uint_as_float(v[2 * i + 1]) + sm.bias[32 * j + 2 * i + 1] + r2.y;
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(fmaxf(x0, 0.f), fmaxf(x1, 0.f));
          packed[i] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        uint4* op = reinterpret_cast<uint4*>(out + (size_t)m * kC + 32 * j);
#pragma unroll
        for (int qq = 0; qq < 4; ++qq)
          op[qq] = make_uint4(packed[4 * qq], packed[4 * qq + 1], packed[4 * qq + 2], packed[4 * qq + 3]);
      }
      tc::fence_before_sync();
      pipe::mbar_arrive(&sm.acc_empty[buf]);
      if (!ok) break;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tmem, 512);
}

// ---- halo variant: padded, 8-board-interleaved activations ----------------
// Layout: boards are taken in groups of 8; a group holds 11 padded ranks
// (rank 0 all zeros, ranks 1..10 the board's ranks 0..9) of 10 padded files
// (files 0..8, file 9 all zeros), and each (rank, file) cell holds the 8
// boards' rows:  row = ((group * 11 + rank + 1) * 10 + file) * 8 + board % 8.
// A 3x3 tap (dr, df) is then the constant row shift (10 dr + df) * 8 for
// every square of every board, and every neighbour off the board lands on a
// zero row (the zero file or zero rank of this group, or of the neighbouring
// group, or outside the buffer, which TMA fills with zeros).  The shifts are
// multiples of 8 rows, i.e. of the 1024-byte 128B-swizzle atom, so one halo
// tile of rows m0 - 88 .. m0 + 343 (432 rows, 64 channels, 54 KB) serves all
// nine taps of a 256-row pair as descriptor offsets: no per-tap A loads and
// no edge fix-up.  The cost is 880 rows per 8 boards instead of 720 (22 %
// more MMA rows); the epilogue writes zeros to the padding rows, so each
// conv's output is again a valid padded input.
//
// The MMA is the transposed product D[channel][row] = W[channel][k] .
// X[row][k]: A = a 128-channel weight tile, B = the pair's 256 activation
// rows, one M128 N256 K16 instruction per K step (128 tensor cycles; half
// the instructions, and a third less shared-memory operand traffic, than two
// M128 N128 ones with the activations as A).
//
// rn_hconv_kernel, one CTA per SM, loops over 256-row pairs.  K blocks run
// channel-half major (9 taps of channels 0-63, then of 64-127): a halo tile
// per channel half, double-buffered, so the next pair's first half loads
// while this pair's second half runs.  Weights stream through a 6-stage ring
// of 16 KB tiles.  Warps: 0 loader; 1 MMA issuer and TMEM owner (512
// columns: two pairs' accumulators of 256 rows); 2-9 epilogue (TMEM lane
// quadrant w % 4 is the channel block, warps 2-5 take rows 0-127 of the pair
// and 6-9 rows 128-255).  The issuing thread is the critical path -- an
// mbarrier wait costs it 100-250 cycles while the tensor core streams
// operands, against 512 tensor cycles per weight tile -- so its tap loop is
// unrolled into constant descriptor offsets with no per-block division.
// The epilogue turns each 32 x 32 (channel x row) accumulator block into
// row-major bf16 with a register transpose (butterfly shuffles), so its
// global loads and stores are 16-byte accesses covering 8 rows x 64 bytes
// per warp instruction.  Consecutive convs are programmatic dependent
// launches.  Bounded waits throughout; after an abort the loader waits for
// its copies in flight and the issuer for its MMAs before the CTA ends.
constexpr int kPitchF = 10;                           // padded files per rank
constexpr int kPitchR = 11;                           // padded ranks per group
constexpr int kGroupBoards = 8;                       // boards interleaved per group
constexpr int kGroupRows = kPitchF * kPitchR * kGroupBoards;  // 880
constexpr int kHalo = (kPitchF + 1) * kGroupBoards;   // 88: the largest tap shift
constexpr int kPairRows = 2 * kTileM;                 // 256: the MMA's N
constexpr int kHaloRows = kPairRows + 2 * kHalo;      // 432
constexpr int kHaloBox = kHaloRows / 2;               // 216 rows per TMA box (<= 256)
constexpr int kHaloBytes = kHaloRows * 128;           // 55,296 (54 x 1024)
constexpr int kWStages = 6;                           // weight stages of one K block (16 KB)
constexpr int kEpiWarps = 8;                          // epilogue warps (4 or 8: a multiple of the 4 lane quadrants)
constexpr int kEpiChunks = kPairRows / 32 / (kEpiWarps / 4);  // 32-row chunks per epilogue warp and pair
constexpr int kHThreads = 64 + 32 * kEpiWarps;
static_assert(kHaloBox % 8 == 0 && kHaloBytes % 1024 == 0, "halo boxes keep the swizzle atom");

__host__ __device__ inline int64_t padded_row(int64_t board, int square) {
  return (((board >> 3) * kPitchR + square / 9 + 1) * kPitchF + square % 9) * kGroupBoards + (board & 7);
}
inline int64_t padded_rows(int64_t batch) { return (batch + kGroupBoards - 1) / kGroupBoards * kGroupRows; }

struct HConvSmem {
  alignas(1024) uint8_t halo[2][kHaloBytes];
  alignas(1024) uint8_t w[kWStages][kTileBytes];
  uint64_t w_full[kWStages];
  uint64_t w_empty[kWStages];
  uint64_t halo_full[2];
  uint64_t halo_empty[2];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// One butterfly stage of a 32 x 32 register transpose across a warp: lanes
// l and l ^ K swap the halves of their register pairs (i, i + K) that the
// other side needs.  After the stages K = 16, 8, 4, 2, 1, lane l holds in
// v[i] what lane i held in v[l].
template <int K>
__device__ __forceinline__ void transpose32(float (&v)[32], int lane) {
  const bool upper = (lane & K) != 0;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    if (i & K) continue;
    const float recv = __shfl_xor_sync(0xffffffffu, upper ? v[i] : v[i + K], K);
    v[i] = upper ? recv : v[i];
    v[i + K] = upper ? v[i + K] : recv;
  }
}

template <int CIN>
__global__ void __launch_bounds__(kHThreads, 1) rn_hconv_kernel(const __grid_constant__ CUtensorMap tmap_in,
                                                               const uint8_t* __restrict__ wtiles,
                                                               const float* __restrict__ bias,
                                                               const __nv_bfloat16* __restrict__ resid,
                                                               __nv_bfloat16* __restrict__ out, int M,
                                                               uint32_t* status) {
  constexpr int kKh = CIN / 64;  // channel halves
  extern __shared__ uint8_t smem_raw[];
  HConvSmem& sm = *reinterpret_cast<HConvSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_pairs = (M + kPairRows - 1) / kPairRows;

  if (warp == 1) {
    tc::tmem_alloc(pipe::smem_addr(&sm.tmem_base), 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < kWStages; ++s) {
      pipe::mbar_init(&sm.w_full[s], 1);
      pipe::mbar_init(&sm.w_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      pipe::mbar_init(&sm.halo_full[b], 1);
      pipe::mbar_init(&sm.halo_empty[b], 1);
      pipe::mbar_init(&sm.acc_full[b], 1);
      pipe::mbar_init(&sm.acc_empty[b], 32 * kEpiWarps);
    }
    pipe::mbar_init(&sm.drain, 1);
    sm.abort = 0;
    pipe::mbar_init_fence();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  // Programmatic dependent launch: the next conv may be scheduled now (its
  // CTAs take SMs as this grid's CTAs exit, and set up there); every thread
  // waits here until the previous grid has completed and its writes are
  // visible, before any activation is read or written.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 0) {
    // ---- loader: per pair and channel half, the halo (two TMA boxes), then
    // the half's nine weight tiles.
    if (lane == 0) {
      uint32_t nw = 0, nh = 0;  // weight tiles / halos issued
      uint32_t ws = 0, wphase = 0;
      for (int pair = blockIdx.x; pair < n_pairs; pair += gridDim.x) {
        const int y0 = pair * kPairRows - kHalo;
        for (int kh = 0; kh < kKh; ++kh) {
          const uint32_t hb = nh & 1, hu = nh >> 1;
          if (hu > 0 && !pipe::mbar_wait(&sm.halo_empty[hb], (hu - 1) & 1, &sm.abort, status)) goto done_load;
          pipe::mbar_arrive_expect_tx(&sm.halo_full[hb], kHaloBytes);
          tc::tma_load_2d(pipe::smem_addr(sm.halo[hb]), &tmap_in, kh * 64, y0, pipe::smem_addr(&sm.halo_full[hb]));
          tc::tma_load_2d(pipe::smem_addr(sm.halo[hb]) + kHaloBox * 128, &tmap_in, kh * 64, y0 + kHaloBox,
                          pipe::smem_addr(&sm.halo_full[hb]));
          ++nh;
          const uint8_t* src = wtiles + (size_t)kh * 9 * kTileBytes;
          for (int tap = 0; tap < 9; ++tap, src += kTileBytes) {
            if (nw >= kWStages && !pipe::mbar_wait(&sm.w_empty[ws], wphase ^ 1, &sm.abort, status)) goto done_load;
            pipe::mbar_arrive_expect_tx(&sm.w_full[ws], kTileBytes);
            pipe::bulk_copy_g2s(sm.w[ws], src, kTileBytes, &sm.w_full[ws]);
            ++nw;
            if (++ws == kWStages) {
              ws = 0;
              wphase ^= 1;
            }
          }
        }
      }
    done_load:
      if (sm.abort) {
        // land every copy still in flight: the last use of each buffer
        for (uint32_t i = nw > kWStages ? nw - kWStages : 0; i < nw; ++i)
          pipe::mbar_wait_drain(&sm.w_full[i % kWStages], (i / kWStages) & 1, status);
        for (uint32_t i = nh > 2 ? nh - 2 : 0; i < nh; ++i)
          pipe::mbar_wait_drain(&sm.halo_full[i & 1], (i >> 1) & 1, status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer: per K step one M128 (channels) x N256 (rows) x K16.
    // The issuing thread is the critical path (each barrier wait costs it a
    // few hundred cycles while the tensor core streams operands), so the
    // tap loop is unrolled: tap shifts are constant descriptor offsets and
    // the stage index and phase advance without division.
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(128, kPairRows);
      const uint64_t wdesc0 = tc::smem_desc(pipe::smem_addr(sm.w[0]), 0, 1024, tc::kSwizzle128B);
      uint32_t nh = 0, ws = 0, wphase = 0;
      int it = 0;
      bool ok = true;
      for (int pair = blockIdx.x; pair < n_pairs && ok; pair += gridDim.x, ++it) {
        const int buf = it & 1, use = it >> 1;
        if (use > 0 && !pipe::mbar_wait(&sm.acc_empty[buf], (use - 1) & 1, &sm.abort, status)) break;
        const uint32_t d = tmem + (uint32_t)(buf * kPairRows);
        for (int kh = 0; kh < kKh && ok; ++kh) {
          const uint32_t hb = nh & 1;
          if (!pipe::mbar_wait(&sm.halo_full[hb], (nh >> 1) & 1, &sm.abort, status)) {
            ok = false;
            break;
          }
          ++nh;
          // descriptor of the halo row m0 (tap shift 0); a shift of r rows is + 8 r
          const uint64_t xdesc0 =
              tc::smem_desc(pipe::smem_addr(sm.halo[hb]) + kHalo * 128, 0, 1024, tc::kSwizzle128B);
#pragma unroll
          for (int tap = 0; tap < 9; ++tap) {
            if (!pipe::mbar_wait(&sm.w_full[ws], wphase, &sm.abort, status)) {
              ok = false;
              break;
            }
            tc::fence_after_sync();
            const int shift = ((tap / 3 - 1) * kPitchF + (tap % 3 - 1)) * kGroupBoards;
            const uint64_t ad = wdesc0 + (uint64_t)ws * (kTileBytes >> 4);
            const uint64_t bd = xdesc0 + (uint64_t)(int64_t)(shift * 8);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)  // +32 bytes per K step: +2 in the descriptor's address field
              tc::mma_bf16(d, ad + 2 * kk, bd + 2 * kk, idesc, (kh | tap | kk) != 0 ? 1u : 0u);
            tc::commit(pipe::smem_addr(&sm.w_empty[ws]));
            if (++ws == kWStages) {
              ws = 0;
              wphase ^= 1;
            }
          }
          if (!ok) break;
          tc::commit(pipe::smem_addr(&sm.halo_empty[hb]));
        }
        tc::commit(pipe::smem_addr(&sm.acc_full[buf]));
      }
      // every MMA issued has completed before TMEM is released
      tc::commit(pipe::smem_addr(&sm.drain));
      pipe::mbar_wait_drain(&sm.drain, 0, status);
    }
    __syncwarp();
  } else {
    // ---- epilogue: TMEM lane quadrant w % 4 is channels 32 (w % 4) .. + 31;
    // warp w covers rows part * 32 kEpiChunks .. of the pair (part =
    // (w - 2) / 4) in chunks of 32.  Per chunk a lane loads its channel's 32
    // rows (+ bias); three butterfly stages and a lane rotation then leave
    // lane l with rows 8t + l / 4 (t = 0..3), channels 8 (l % 4) .. + 7, so
    // each warp-wide 16-byte access covers 8 rows x 64 contiguous bytes.  The
    // 8 rows of one (rank, file) cell share real/padding: ReLU(acc + bias (+
    // residual)) in bf16, or zeros.
    const int q = warp & 3, part = (warp - 2) >> 2;
    const float bc = __ldg(bias + 32 * q + lane);
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(part * 32 * kEpiChunks);
    const int rsub = lane >> 2, csub = 32 * q + 8 * (lane & 3);
    const int rot_src = ((lane & 3) << 3) | (lane >> 2);
    int it = 0;
    for (int pair = blockIdx.x; pair < n_pairs; pair += gridDim.x, ++it) {
      const int buf = it & 1, use = it >> 1;
      const int m0 = pair * kPairRows + part * 32 * kEpiChunks;
      bool ok = true;
#pragma unroll 1
      for (int cg = 0; cg < kEpiChunks; cg += 4) {
        // real cells and residual rows of four chunks first: the loads
        // overlap the accumulator wait (and the previous chunks' work)
        uint32_t real_bits = 0;
        uint4 rv[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int cm = m0 + 32 * (cg + j) + 8 * t, cell = cm >> 3;  // the cell of rows cm .. cm + 7
            const bool real = cm < M && (cell / kPitchF) % kPitchR >= 1 && cell % kPitchF < 9;
            real_bits |= (uint32_t)real << (4 * j + t);
            rv[j][t] = (resid != nullptr && real)
                           ? __ldg(reinterpret_cast<const uint4*>(resid + (size_t)(cm + rsub) * kC + csub))
                           : make_uint4(0u, 0u, 0u, 0u);
          }
        if (cg == 0) {
          // warp-uniform, so that no lane skips the shuffles below
          ok = __all_sync(0xffffffffu, pipe::mbar_wait(&sm.acc_full[buf], use & 1, &sm.abort, status));
          tc::fence_after_sync();
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t v[32];
          __syncwarp();
          tc::tmem_ld32(lane_addr + (uint32_t)(buf * kPairRows + 32 * (cg + j)), v);
          tc::wait_ld();
          if (!ok) continue;
          float f[32];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {  // + bias, packed in pairs
            f[i] = __uint_as_float(v[i]);
            f[i + 1] = __uint_as_float(v[i + 1]);
            fadd2_rn(f[i], f[i + 1], bc, bc);
          }
          transpose32<4>(f, lane);
          transpose32<2>(f, lane);
          transpose32<1>(f, lane);
#pragma unroll
          for (int i = 0; i < 32; ++i) f[i] = __shfl_sync(0xffffffffu, f[i], rot_src);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int cm = m0 + 32 * (cg + j) + 8 * t;
            if (cm >= M) break;  // M is a multiple of 8: whole cells only
            uint32_t packed[4] = {0u, 0u, 0u, 0u};
            if ((real_bits >> (4 * j + t)) & 1u) {
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const uint32_t rw = (&rv[j][t].x)[e];
                const float2 r2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rw));
                float x0 = f[8 * t + 2 * e], x1 = f[8 * t + 2 * e + 1];
                fadd2_rn(x0, x1, r2.x, r2.y);
                const __nv_bfloat162 h2 = __floats2bfloat162_rn(fmaxf(x0, 0.f), fmaxf(x1, 0.f));
                packed[e] = *reinterpret_cast<const uint32_t*>(&h2);
              }
            }
            *reinterpret_cast<uint4*>(out + (size_t)(cm + rsub) * kC + csub) =
                make_uint4(packed[0], packed[1], packed[2], packed[3]);
          }
        }
      }
      tc::fence_before_sync();
      pipe::mbar_arrive(&sm.acc_empty[buf]);
      if (!ok) break;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tmem, 512);
}

// [B][15][90] bf16 planes -> the padded layout above, [rows][64] bf16,
// channels 15..63 zero, padding rows (and the boards past B in the last
// group) all zero.  One thread per 16-byte chunk of a padded row (8 channels),
// so a warp's stores are 512 contiguous bytes.
__global__ void rn_pack_padded_kernel(const __nv_bfloat16* __restrict__ planes, int64_t B, int64_t rows,
                                      __nv_bfloat16* __restrict__ out) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= rows * 8) return;
  const int64_t m = t >> 3;
  const int q = (int)(t & 7);
  const int64_t cell = m >> 3;
  const int file = (int)(cell % kPitchF), rank = (int)((cell / kPitchF) % kPitchR);
  const int64_t b = (cell / (kPitchF * kPitchR)) * kGroupBoards + (m & 7);
  uint32_t w[4] = {0u, 0u, 0u, 0u};
  if (q * 8 < CNNUE_RN_PLANES && rank >= 1 && file < 9 && b < B) {
    const int p = (rank - 1) * 9 + file;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int c = q * 8 + k;
      if (c < CNNUE_RN_PLANES) {
        const uint16_t v = reinterpret_cast<const uint16_t*>(planes)[(b * CNNUE_RN_PLANES + c) * kSq + p];
        w[k >> 1] |= (uint32_t)v << (16 * (k & 1));
      }
    }
  }
  reinterpret_cast<uint4*>(out + m * 64)[q] = make_uint4(w[0], w[1], w[2], w[3]);
}

// [B][15][90] bf16 planes -> [B*90][64] bf16, channels 15..63 zero.
__global__ void rn_pack_kernel(const __nv_bfloat16* __restrict__ planes, int64_t B, __nv_bfloat16* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * kSq) return;
  const int64_t b = i / kSq;
  const int p = (int)(i - b * kSq);
  uint32_t w[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) w[k] = 0u;
#pragma unroll
  for (int c = 0; c < CNNUE_RN_PLANES; ++c) {
    const uint16_t v = reinterpret_cast<const uint16_t*>(planes)[(b * CNNUE_RN_PLANES + c) * kSq + p];
    w[c >> 1] |= (uint32_t)v << (16 * (c & 1));
  }
  uint4* o = reinterpret_cast<uint4*>(out + i * 64);
#pragma unroll
  for (int q = 0; q < 8; ++q) o[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
}

struct HeadArgs {
  const __nv_bfloat16* trunk;  // [B*90][128]
  const float* pcw;            // [2][128]
  const float* pcb;            // [2]
  const float* pfw_t;          // [180][2086]
  const float* pfb;            // [2086]
  const float* vcw;            // [128]
  const float* vcb;            // [1]
  const float* v1w_t;          // [90][256]
  const float* v1b;            // [256]
  const float* v2w;            // [256]
  const float* v2b;            // [1]
  int64_t B;
  int padded;     // trunk in the padded 8-board layout (else [B*90][128])
  float* logits;  // [B][2086] or null
  float* probs;   // [B][2086]
  float* value;   // [B]
};


// 1x1 convs of the trunk: policy planes to pc_t [180][B] and the value plane
// to vc_t [90][B] (both after bias and ReLU).  A warp takes one square of 16
// consecutive boards, two lanes per board: lanes l and l + 16 read the
// even and the odd 16-byte chunks of board 16k + l's 128-channel row (eight
// loads each; in the padded layout a warp's rows are two runs of 8 adjacent
// rows), form partial dot products with the weights as shared-memory
// broadcasts, and add them with one shuffle; the warp's stores to pc_t / vc_t
// are 64 contiguous bytes each.
constexpr int kConvBoards = 16;
__global__ void __launch_bounds__(256) rn_head_conv_kernel(HeadArgs a, float* __restrict__ pc_t,
                                                           float* __restrict__ vc_t) {
  __shared__ __align__(16) float w[3][kC];  // policy plane 0, policy plane 1, value plane
  for (int i = threadIdx.x; i < 3 * kC; i += blockDim.x)
    (&w[0][0])[i] = i < 2 * kC ? __ldg(a.pcw + i) : __ldg(a.vcw + (i - 2 * kC));
  __syncthreads();
  const int lane = threadIdx.x & 31, half = lane >> 4;
  const int64_t item = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int64_t chunks = (a.B + kConvBoards - 1) / kConvBoards;
  if (item >= chunks * kSq) return;  // whole warp
  const int64_t chunk = item / kSq;
  const int p = (int)(item - chunk * kSq);
  const int64_t b = chunk * kConvBoards + (lane & 15);
  float s0 = 0.f, s1 = 0.f, s2 = 0.f;
  if (b < a.B) {
    const int64_t r = a.padded ? padded_row(b, p) : b * kSq + p;
    const uint4* row = reinterpret_cast<const uint4*>(a.trunk + (size_t)r * kC);
    uint4 x[kC / 16];
#pragma unroll
    for (int q = 0; q < kC / 16; ++q) x[q] = __ldg(row + 2 * q + half);
#pragma unroll
    for (int q = 0; q < kC / 16; ++q) {
      const uint32_t u[4] = {x[q].x, x[q].y, x[q].z, x[q].w};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = 16 * q + 8 * half + 4 * h;
        const float4 w0 = *reinterpret_cast<const float4*>(&w[0][c]);
        const float4 w1 = *reinterpret_cast<const float4*>(&w[1][c]);
        const float4 wv = *reinterpret_cast<const float4*>(&w[2][c]);
        const float2 xa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[2 * h]));
        const float2 xb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[2 * h + 1]));
        s0 = fmaf(xb.y, w0.w, fmaf(xb.x, w0.z, fmaf(xa.y, w0.y, fmaf(xa.x, w0.x, s0))));
        s1 = fmaf(xb.y, w1.w, fmaf(xb.x, w1.z, fmaf(xa.y, w1.y, fmaf(xa.x, w1.x, s1))));
        s2 = fmaf(xb.y, wv.w, fmaf(xb.x, wv.z, fmaf(xa.y, wv.y, fmaf(xa.x, wv.x, s2))));
      }
    }
  }
  s0 += __shfl_xor_sync(0xffffffffu, s0, 16);
  s1 += __shfl_xor_sync(0xffffffffu, s1, 16);
  s2 += __shfl_xor_sync(0xffffffffu, s2, 16);
  if (half == 0 && b < a.B) {
    pc_t[(size_t)p * a.B + b] = fmaxf(s0 + __ldg(a.pcb), 0.f);
    pc_t[(size_t)(kSq + p) * a.B + b] = fmaxf(s1 + __ldg(a.pcb + 1), 0.f);
    vc_t[(size_t)p * a.B + b] = fmaxf(s2 + __ldg(a.vcb), 0.f);
  }
}

// Value MLP 90 -> 256 (ReLU) -> 1 (tanh) for 8 boards per CTA: thread j is
// hidden unit j for all 8 boards (the value plane of the 8 boards staged in
// shared memory, read as broadcasts); the 256 -> 1 layer is a block reduction.
constexpr int kValueBoards = 8;
constexpr int kValueSmemFloats = kSq * kValueBoards + kValueBoards * 8;
__device__ __forceinline__ void value_block(const HeadArgs& a, const float* __restrict__ vc_t, int64_t blk,
                                            float* smem) {
  float (*vc)[kValueBoards] = reinterpret_cast<float (*)[kValueBoards]>(smem);
  float (*red)[8] = reinterpret_cast<float (*)[8]>(smem + kSq * kValueBoards);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t b0 = blk * kValueBoards;
  for (int i = tid; i < kSq * kValueBoards; i += 256) {
    const int p = i / kValueBoards, bl = i % kValueBoards;
    vc[p][bl] = b0 + bl < a.B ? vc_t[(size_t)p * a.B + b0 + bl] : 0.f;
  }
  __syncthreads();
  float h[kValueBoards];
#pragma unroll
  for (int bl = 0; bl < kValueBoards; ++bl) h[bl] = 0.f;
#pragma unroll 6
  for (int p = 0; p < kSq; ++p) {
    const float w = __ldg(a.v1w_t + (size_t)p * 256 + tid);
#pragma unroll
    for (int q = 0; q < kValueBoards / 4; ++q) {
      const float4 x = *reinterpret_cast<const float4*>(&vc[p][4 * q]);
      h[4 * q] = fmaf(x.x, w, h[4 * q]);
      h[4 * q + 1] = fmaf(x.y, w, h[4 * q + 1]);
      h[4 * q + 2] = fmaf(x.z, w, h[4 * q + 2]);
      h[4 * q + 3] = fmaf(x.w, w, h[4 * q + 3]);
    }
  }
  const float w2 = __ldg(a.v2w + tid), b1 = __ldg(a.v1b + tid);
#pragma unroll
  for (int bl = 0; bl < kValueBoards; ++bl) {
    float v = fmaxf(h[bl] + b1, 0.f) * w2;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[bl][warp] = v;
  }
  __syncthreads();
  if (tid < kValueBoards && b0 + tid < a.B) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) v += red[tid][w];
    a.value[b0 + tid] = tanhf(v + __ldg(a.v2b));
  }
}

// Policy FC logits[B][2086] = pc[B][180] . W^T + b, from pc_t [180][B]: CTA
// tile 128 boards x 128 moves, thread tile 8 x 8 (four 16-byte shared loads
// per 64 FMAs), K in chunks of 10 double-buffered through registers: the
// next chunk's global loads are in flight while this one is multiplied.
constexpr int kFcBoards = 128, kFcMoves = 128, kFcK = 10;
constexpr int kFcSmemFloats = 2 * kFcK * kFcBoards + 2 * kFcK * kFcMoves;
__device__ __forceinline__ void policy_fc_block(const float* __restrict__ pc_t, const float* __restrict__ pfw_t,
                                                const float* __restrict__ pfb, int64_t B,
                                                float* __restrict__ logits, int64_t bx, int by, float* smem) {
  float (*xs)[kFcK][kFcBoards] = reinterpret_cast<float (*)[kFcK][kFcBoards]>(smem);
  float (*ws)[kFcK][kFcMoves] = reinterpret_cast<float (*)[kFcK][kFcMoves]>(smem + 2 * kFcK * kFcBoards);
  constexpr int kPer = kFcK * kFcBoards / 256;  // elements of each operand a thread stages per chunk
  static_assert(kFcK * kFcBoards % 256 == 0 && kFcBoards == kFcMoves && (2 * kSq) % kFcK == 0, "tiles");
  const int tid = threadIdx.x;
  const int64_t b0 = bx * kFcBoards;
  const int j0 = by * kFcMoves;
  // thread tile: boards tb .. tb+7, moves tj .. tj+3 and tj+64 .. tj+67 (a
  // warp's two 16-byte weight reads are then 256 contiguous bytes each)
  const int tb = (tid >> 4) * 8, tj = (tid & 15) * 4;
  float rx[kPer], rw[kPer];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      const int i = tid + 256 * r, k = i / kFcBoards, c = i % kFcBoards;
      rx[r] = b0 + c < B ? __ldg(pc_t + (size_t)(k0 + k) * B + b0 + c) : 0.f;
      rw[r] = j0 + c < kMoves ? __ldg(pfw_t + (size_t)(k0 + k) * kMoves + j0 + c) : 0.f;
    }
  };
  auto stage = [&](int buf) {
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      const int i = tid + 256 * r, k = i / kFcBoards, c = i % kFcBoards;
      xs[buf][k][c] = rx[r];
      ws[buf][k][c] = rw[r];
    }
  };
  float acc[8][8] = {};
  fetch(0);
  stage(0);
  __syncthreads();
  int buf = 0;
  for (int k0 = 0; k0 < 2 * kSq; k0 += kFcK) {
    const bool more = k0 + kFcK < 2 * kSq;
    if (more) fetch(k0 + kFcK);
#pragma unroll 4
    for (int k = 0; k < kFcK; ++k) {
      const float4 xa = *reinterpret_cast<const float4*>(&xs[buf][k][tb]);
      const float4 xb = *reinterpret_cast<const float4*>(&xs[buf][k][tb + 4]);
      const float4 wa = *reinterpret_cast<const float4*>(&ws[buf][k][tj]);
      const float4 wb = *reinterpret_cast<const float4*>(&ws[buf][k][tj + kFcMoves / 2]);
      const float x[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
      const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[i][q] = fmaf(x[i], w[q], acc[i][q]);
    }
    if (more) {
      stage(buf ^ 1);
      __syncthreads();
      buf ^= 1;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t b = b0 + tb + i;
    if (b >= B) continue;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int j = j0 + tj + (q < 4 ? q : kFcMoves / 2 + q - 4);
      if (j < kMoves) logits[b * kMoves + j] = acc[i][q] + __ldg(pfb + j);
    }
  }
}

// The value MLP and the policy FC both read only rn_head_conv_kernel's
// outputs, so one launch runs them side by side: blocks [0, n_fc) are policy
// FC tiles (fc_x tiles of boards per row of moves), the rest value blocks.
// Each block computes exactly what the separate kernel would.
static_assert(kFcSmemFloats >= kValueSmemFloats, "head smem");
__global__ void __launch_bounds__(256, 2) rn_heads_kernel(HeadArgs a, const float* __restrict__ pc_t,
                                                       const float* __restrict__ vc_t, unsigned fc_x,
                                                       unsigned n_fc) {
  __shared__ __align__(16) float smem[kFcSmemFloats];
  if (blockIdx.x < n_fc)
    policy_fc_block(pc_t, a.pfw_t, a.pfb, a.B, a.logits, blockIdx.x % fc_x, (int)(blockIdx.x / fc_x), smem);
  else
    value_block(a, vc_t, blockIdx.x - n_fc, smem);
}

// Softmax over the 2086 logits of a board, one warp per board, 4 boards per
// CTA.  Lane l keeps logits l, l + 32, ... of its board in registers, so the
// row is read once and each exponential computed once (the sum runs in the
// same order as a strided loop over the row would).
constexpr int kSoftmaxBoards = 4;
constexpr int kSoftmaxPer = (kMoves + 31) / 32;
__global__ void __launch_bounds__(32 * kSoftmaxBoards) rn_softmax_kernel(const float* __restrict__ logits,
                                                                        int64_t B, float* __restrict__ probs) {
  const int64_t b = (int64_t)blockIdx.x * kSoftmaxBoards + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= B) return;
  const float* row = logits + b * kMoves;
  float e[kSoftmaxPer];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kSoftmaxPer; ++i) {
    const int j = lane + 32 * i;
    e[i] = j < kMoves ? __ldg(row + j) : -INFINITY;
    m = fmaxf(m, e[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kSoftmaxPer; ++i) {
    if (lane + 32 * i < kMoves) {
      e[i] = expf(e[i] - m);
      s += e[i];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float inv = 1.f / s;
  float* out = probs + b * kMoves;
#pragma unroll
  for (int i = 0; i < kSoftmaxPer; ++i) {
    const int j = lane + 32 * i;
    if (j < kMoves) out[j] = e[i] * inv;
  }
}

// Host: fp32 -> bf16 bits, round to nearest even.
inline uint16_t to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);  // quiet NaN
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

// One conv's weights (OIHW [128][cin][3][3]) as K-block tiles of the UMMA
// layout, channel-half major: K block kb covers tap kb % 9 and channels
// 64 * (kb / 9) .. + 63; channels >= cin are zero.
void tile_conv(const float* w, int cin, int cin_pad, uint8_t* dst) {
  const int kb_per_tap = cin_pad / 64;
  for (int kb = 0; kb < 9 * kb_per_tap; ++kb) {
    const int tap = kb % 9, c0 = (kb / 9) * 64;
    const int kh = tap / 3, kw = tap % 3;
    uint8_t* tile = dst + (size_t)kb * kTileBytes;
    for (int n = 0; n < kC; ++n)
      for (int k = 0; k < 64; ++k) {
        const int c = c0 + k;
        const float v = c < cin ? w[((n * cin + c) * 3 + kh) * 3 + kw] : 0.f;
        const uint16_t h = to_bf16(v);
        std::memcpy(tile + tile_offset(n, k), &h, 2);
      }
  }
}

size_t conv_smem_bytes() { return sizeof(ConvSmem) + 1024; }
size_t pconv_smem_bytes() { return sizeof(PConvSmem) + 1024; }
size_t hconv_smem_bytes() { return sizeof(HConvSmem) + 1024; }

// Tensor map of an activation buffer [M][cin] bf16 read in boxes of
// `box_rows` rows x 64 channels with the 128-byte swizzle; rows outside
// [0, M) read zeros.
int make_act_map(CUtensorMap* map, const void* base, int cin, int64_t M, int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = tma_encode_fn();
  if (!fn) return set_error(CNNUE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const cuuint64_t dims[2] = {(cuuint64_t)cin, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)cin * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(CNNUE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return CNNUE_OK;
}

}  // namespace
}  // namespace rn
}  // namespace cnnue

struct cnnue_rn_model {
  int device = 0;
  int sms = 148;
  int conv_kind = 2;  // 2: rn_hconv_kernel, 1: rn_pconv_kernel, 0: the one-tile-per-CTA rn_conv_kernel
  void* blob = nullptr;
  uint8_t* tiles = nullptr;  // [kTotalKb][16 KB]
  float* conv_bias = nullptr;  // [21][128]
  float* head = nullptr;       // heads, see HeadArgs
  cnnue::rn::HeadArgs h{};
};

using namespace cnnue;
using namespace cnnue::rn;

extern "C" {

size_t cnnue_rn_workspace_bytes(int64_t batch) {
  // rows of the padded layout (>= 90 per board, so either layout fits)
  const size_t m = batch > 0 ? (size_t)padded_rows(batch) : 0;
  const size_t b = batch > 0 ? (size_t)batch : 0;
  return sizeof(WorkspaceHeader) + align_up(m * 64 * 2, 256) + 3 * align_up(m * kC * 2, 256) +
         align_up(b * 2 * kSq * 4, 256) + align_up(b * kSq * 4, 256) + align_up(b * kMoves * 4, 256);
}

int cnnue_rn_model_create(const cnnue_rn_weights* w, int device, cnnue_rn_model** out) {
  if (!w || !out || !w->stem_w || !w->stem_b || !w->block_w || !w->block_b || !w->policy_conv_w ||
      !w->policy_conv_b || !w->policy_fc_w || !w->policy_fc_b || !w->value_conv_w || !w->value_conv_b ||
      !w->value_fc1_w || !w->value_fc1_b || !w->value_fc2_w || !w->value_fc2_b)
    return set_error(CNNUE_ERR_INVALID_ARG, "null weights");
  *out = nullptr;
  DeviceGuard guard(device);
  if (guard.status) return guard.status;
  // host staging: tiles, biases, heads (transposed where the kernel reads columns)
  std::vector<uint8_t> tiles(kTotalKb * kTileBytes);
  tile_conv(w->stem_w, CNNUE_RN_PLANES, 64, tiles.data());
  for (int j = 0; j < 2 * CNNUE_RN_BLOCKS; ++j)
    tile_conv(w->block_w + (size_t)j * kC * kC * 9, kC, kC, tiles.data() + conv_tile_offset(1 + j) * kTileBytes);
  std::vector<float> bias((size_t)kConvs * kC);
  std::memcpy(bias.data(), w->stem_b, sizeof(float) * kC);
  std::memcpy(bias.data() + kC, w->block_b, sizeof(float) * 2 * CNNUE_RN_BLOCKS * kC);
  const size_t n_pfw = (size_t)2 * kSq * kMoves, n_v1 = (size_t)kSq * 256;
  std::vector<float> head(2 * kC + 2 + n_pfw + kMoves + kC + 1 + n_v1 + 256 + 256 + 1);
  float* hp = head.data();
  float* pcw = hp; std::memcpy(pcw, w->policy_conv_w, sizeof(float) * 2 * kC); hp += 2 * kC;
  float* pcb = hp; std::memcpy(pcb, w->policy_conv_b, sizeof(float) * 2); hp += 2;
  float* pfw_t = hp;
  for (int j = 0; j < kMoves; ++j)
    for (int k = 0; k < 2 * kSq; ++k) pfw_t[(size_t)k * kMoves + j] = w->policy_fc_w[(size_t)j * 2 * kSq + k];
  hp += n_pfw;
  float* pfb = hp; std::memcpy(pfb, w->policy_fc_b, sizeof(float) * kMoves); hp += kMoves;
  float* vcw = hp; std::memcpy(vcw, w->value_conv_w, sizeof(float) * kC); hp += kC;
  float* vcb = hp; vcb[0] = w->value_conv_b[0]; hp += 1;
  float* v1w_t = hp;
  for (int i = 0; i < 256; ++i)
    for (int p = 0; p < kSq; ++p) v1w_t[(size_t)p * 256 + i] = w->value_fc1_w[(size_t)i * kSq + p];
  hp += n_v1;
  float* v1b = hp; std::memcpy(v1b, w->value_fc1_b, sizeof(float) * 256); hp += 256;
  float* v2w = hp; std::memcpy(v2w, w->value_fc2_w, sizeof(float) * 256); hp += 256;
  float* v2b = hp; v2b[0] = w->value_fc2_b[0];

  auto* m = new (std::nothrow) cnnue_rn_model;
  if (!m) return set_error(CNNUE_ERR_INVALID_ARG, "out of host memory");
  m->device = device;
  const size_t t_bytes = align_up(tiles.size(), 1024), b_bytes = align_up(bias.size() * 4, 256);
  const size_t h_bytes = align_up(head.size() * 4, 256);
  cudaError_t e = cudaMalloc(&m->blob, t_bytes + b_bytes + h_bytes);
  if (e != cudaSuccess) {
    delete m;
    return cuda_error(e, "cudaMalloc(resnet model)");
  }
  m->tiles = (uint8_t*)m->blob;
  m->conv_bias = (float*)((char*)m->blob + t_bytes);
  m->head = (float*)((char*)m->blob + t_bytes + b_bytes);
  int st = CNNUE_OK;
  if ((e = cudaMemcpy(m->tiles, tiles.data(), tiles.size(), cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemcpy(m->conv_bias, bias.data(), bias.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemcpy(m->head, head.data(), head.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess)
    st = cuda_error(e, "resnet weight upload");
  if (!st) {
    const int smem = (int)conv_smem_bytes();
    if ((e = cudaFuncSetAttribute(rn_conv_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) !=
            cudaSuccess ||
        (e = cudaFuncSetAttribute(rn_conv_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) !=
            cudaSuccess ||
        (e = cudaFuncSetAttribute(rn_pconv_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)pconv_smem_bytes())) != cudaSuccess ||
        (e = cudaFuncSetAttribute(rn_pconv_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)pconv_smem_bytes())) != cudaSuccess ||
        (e = cudaFuncSetAttribute(rn_hconv_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)hconv_smem_bytes())) != cudaSuccess ||
        (e = cudaFuncSetAttribute(rn_hconv_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)hconv_smem_bytes())) != cudaSuccess)
      st = cuda_error(e, "cudaFuncSetAttribute(rn_conv_kernel)");
    int sms = 0;
    if (!st && (e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess)
      st = cuda_error(e, "cudaDeviceGetAttribute");
    m->sms = sms > 0 ? sms : 148;
  }
  if (st) {
    cudaFree(m->blob);
    delete m;
    return st;
  }
  float* dh = m->head;
  auto off = [&](const float* host_ptr) { return dh + (host_ptr - head.data()); };
  m->h.pcw = off(pcw);
  m->h.pcb = off(pcb);
  m->h.pfw_t = off(pfw_t);
  m->h.pfb = off(pfb);
  m->h.vcw = off(vcw);
  m->h.vcb = off(vcb);
  m->h.v1w_t = off(v1w_t);
  m->h.v1b = off(v1b);
  m->h.v2w = off(v2w);
  m->h.v2b = off(v2b);
  *out = m;
  return CNNUE_OK;
}

int cnnue_rn_model_destroy(cnnue_rn_model* m) {
  if (!m) return CNNUE_OK;
  DeviceGuard guard(m->device);
  if (m->blob) cudaFree(m->blob);
  delete m;
  return guard.status;
}

int cnnue_rn_forward(const cnnue_rn_model* m, const uint16_t* d_planes, int64_t batch, float* d_probs,
                     float* d_logits, float* d_value, void* ws, size_t ws_bytes, void* stream) {
  if (!m || !ws || batch < 0 || (batch > 0 && (!d_planes || !d_probs || !d_value)))
    return set_error(CNNUE_ERR_INVALID_ARG, "null model, workspace, planes, probs or value, or batch < 0");
  if (batch > (int64_t)1 << 22) return set_error(CNNUE_ERR_INVALID_ARG, "batch %lld too large", (long long)batch);
  if (ws_bytes < cnnue_rn_workspace_bytes(batch))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu < %zu bytes", ws_bytes, cnnue_rn_workspace_bytes(batch));
  if ((uintptr_t)d_planes & 1u) return set_error(CNNUE_ERR_INVALID_ARG, "planes must be 2-byte aligned");
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  CNNUE_CUDA_TRY(cudaMemsetAsync(ws, 0, sizeof(WorkspaceHeader), s));
  if (batch == 0) return CNNUE_OK;
  const bool padded = m->conv_kind == 2;
  const int M = (int)(padded ? padded_rows(batch) : batch * kSq);
  char* p = (char*)ws + sizeof(WorkspaceHeader);
  const size_t rows_cap = (size_t)padded_rows(batch);
  auto* in64 = (__nv_bfloat16*)p;
  p += align_up(rows_cap * 64 * 2, 256);
  __nv_bfloat16* act[3];
  for (int i = 0; i < 3; ++i) {
    act[i] = (__nv_bfloat16*)p;
    p += align_up(rows_cap * kC * 2, 256);
  }
  float* pc = (float*)p;  // pc_t [180][B]
  p += align_up((size_t)batch * 2 * kSq * 4, 256);
  float* vc = (float*)p;  // vc_t [90][B]
  p += align_up((size_t)batch * kSq * 4, 256);
  float* logits = d_logits ? d_logits : (float*)p;
  uint32_t* status = &((WorkspaceHeader*)ws)->status;
  if (padded)
    rn_pack_padded_kernel<<<(unsigned)((M * 8 + 255) / 256), 256, 0, s>>>((const __nv_bfloat16*)d_planes, batch,
                                                                          M, in64);
  else
    rn_pack_kernel<<<(unsigned)((M + 255) / 256), 256, 0, s>>>((const __nv_bfloat16*)d_planes, batch, in64);
  if (int st = check_launch_error("rn_pack_kernel")) return st;
  const int box_rows = padded ? kHaloBox : kTileM;
  CUtensorMap map_in, map_act[3];
  if (int st = make_act_map(&map_in, in64, 64, M, box_rows)) return st;
  for (int i = 0; i < 3; ++i)
    if (int st = make_act_map(&map_act[i], act[i], kC, M, box_rows)) return st;
  const unsigned tiles = (unsigned)((M + kTileM - 1) / kTileM);
  const int pairs = (M + 2 * kTileM - 1) / (2 * kTileM);
  const unsigned pgrid = (unsigned)(pairs < m->sms ? pairs : m->sms);
  auto conv = [&](bool stem, const CUtensorMap& map, int c, const __nv_bfloat16* resid, __nv_bfloat16* dst) {
    const uint8_t* wt = m->tiles + conv_tile_offset(c) * kTileBytes;
    const float* b = m->conv_bias + c * kC;
    switch (m->conv_kind) {
      case 2: {
        // launched as a programmatic dependent of the previous kernel in the
        // stream: launch and set-up overlap that kernel's tail
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(pgrid);
        cfg.blockDim = dim3(kHThreads);
        cfg.dynamicSmemBytes = hconv_smem_bytes();
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t e = stem ? cudaLaunchKernelEx(&cfg, rn_hconv_kernel<64>, map, wt, b, resid, dst, M, status)
                             : cudaLaunchKernelEx(&cfg, rn_hconv_kernel<128>, map, wt, b, resid, dst, M, status);
        if (e != cudaSuccess) return cuda_error(e, "cudaLaunchKernelEx(rn_hconv_kernel)");
        break;
      }
      case 1:
        if (stem) rn_pconv_kernel<64><<<pgrid, kPThreads, pconv_smem_bytes(), s>>>(map, wt, b, resid, dst, M, status);
        else rn_pconv_kernel<128><<<pgrid, kPThreads, pconv_smem_bytes(), s>>>(map, wt, b, resid, dst, M, status);
        break;
      default:
        if (stem) rn_conv_kernel<64><<<tiles, kConvThreads, conv_smem_bytes(), s>>>(map, wt, b, resid, dst, M, status);
        else rn_conv_kernel<128><<<tiles, kConvThreads, conv_smem_bytes(), s>>>(map, wt, b, resid, dst, M, status);
    }
    return check_launch_error("rn conv");
  };
  if (int st = conv(true, map_in, 0, nullptr, act[0])) return st;
  int x = 0;
  for (int blk = 0; blk < CNNUE_RN_BLOCKS; ++blk) {
    const int h = (x + 1) % 3, y = (x + 2) % 3;
    const int c1 = 1 + 2 * blk, c2 = c1 + 1;
    if (int st = conv(false, map_act[x], c1, nullptr, act[h])) return st;
    if (int st = conv(false, map_act[h], c2, act[x], act[y])) return st;
    x = y;
  }
  HeadArgs h = m->h;
  h.trunk = act[x];
  h.B = batch;
  h.padded = padded ? 1 : 0;
  h.logits = logits;
  h.probs = d_probs;
  h.value = d_value;
  const int64_t conv_warps = (batch + kConvBoards - 1) / kConvBoards * kSq;
  rn_head_conv_kernel<<<(unsigned)((conv_warps + 7) / 8), 256, 0, s>>>(h, pc, vc);
  if (int st = check_launch_error("rn_head_conv_kernel")) return st;
  const unsigned fc_x = (unsigned)((batch + kFcBoards - 1) / kFcBoards);
  const unsigned n_fc = fc_x * ((kMoves + kFcMoves - 1) / kFcMoves);
  const unsigned n_value = (unsigned)((batch + kValueBoards - 1) / kValueBoards);
  rn_heads_kernel<<<n_fc + n_value, 256, 0, s>>>(h, pc, vc, fc_x, n_fc);
  if (int st = check_launch_error("rn_heads_kernel")) return st;
  rn_softmax_kernel<<<(unsigned)((batch + kSoftmaxBoards - 1) / kSoftmaxBoards), 32 * kSoftmaxBoards, 0, s>>>(
      logits, batch, d_probs);
  return check_launch_error("rn_softmax_kernel");
}

int cnnue_rn_set_conv_kernel(cnnue_rn_model* m, int kind) {
  if (!m || kind < 0 || kind > 2) return set_error(CNNUE_ERR_INVALID_ARG, "model or conv kernel kind (0, 1 or 2)");
  m->conv_kind = kind;
  return CNNUE_OK;
}

}  // extern "C"
