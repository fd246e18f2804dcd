// policy.cu - the AZ-NNUE policy-head training ops (Candle custom ops of the
// reference): fused_policy (src/az/fused_policy.rs) and the sparse / tactical
// table lookups (src/az/fused_sparse_policy.rs), forward and backward.
//
// Forward kernels keep the CPU twins' operation order (one product and one
// add per term, no fused multiply-add), so outputs are bit-identical to them;
// fused_policy runs a warp per board with lanes over its moves.
// Backward passes are atomic-free and deterministic (scatter.cuh):
//   - fused_policy: the table gradient splits by section.  Feature rows (the
//     consequence rows and the accumulator feature rows, 1260 x 32 each) take
//     one radix sort of up to three keys per item (to, from, captured) and a
//     64-wide row sum per key; move rows (bias, move context, accumulator
//     move factors) one sort by move index and a 49-wide row sum; the 32
//     consequence weights, hit by every item, an ordered reduction in chunks
//     of 256 items.  Values are formed on the fly from the item, in the CPU
//     twin's operation order.  The context gradient of a board is summed over
//     its moves in order by one thread per (board, context column);
//   - sparse / tactical: scalar (entry, output) pairs through the scalar
//     scatter.
#include <algorithm>

#include "common.cuh"
#include "scatter.cuh"

namespace cnnue {
namespace pol {
namespace {

// fused_policy.rs:10-35: item bit fields and table offsets.
constexpr int kMoveBits = 12, kFeatureBits = 11;
constexpr int kMoveValidBit = kMoveBits + 3 * kFeatureBits;  // 45
constexpr int kCaptureValidBit = kMoveValidBit + 1;          // 46
constexpr int kPolicyValidBit = kCaptureValidBit + 1;        // 47
constexpr uint32_t kConsequence = 40320, kBias = 40352, kContext = 42438, kAccFeature = 75814, kAccMove = 116134;
constexpr uint32_t kTableLen = CNNUE_POLICY_TABLE_LEN;
constexpr int kCtx = CNNUE_POLICY_CONTEXT;  // 16 move context + 32 accumulator context

struct Item {
  bool policy, move, capture;
  uint32_t mv, from, to, cap;
};

__device__ __forceinline__ Item decode(int64_t packed_s) {
  const uint64_t p = (uint64_t)packed_s;
  Item it;
  it.policy = (p >> kPolicyValidBit) & 1u;
  it.move = (p >> kMoveValidBit) & 1u;
  it.capture = (p >> kCaptureValidBit) & 1u;
  it.mv = (uint32_t)(p & 0xfffu);
  it.from = (uint32_t)((p >> kMoveBits) & 0x7ffu);
  it.to = (uint32_t)((p >> (kMoveBits + kFeatureBits)) & 0x7ffu);
  it.cap = (uint32_t)((p >> (kMoveBits + 2 * kFeatureBits)) & 0x7ffu);
  return it;
}

// The table rows an item reads stay inside their table sections.
__device__ __forceinline__ bool in_range(const Item& it) {
  return it.mv < (uint32_t)CNNUE_AZ_DENSE_MOVES &&
         (!it.move || (it.from < (uint32_t)CNNUE_AZ_INPUT && it.to < (uint32_t)CNNUE_AZ_INPUT &&
                       (!it.capture || it.cap < (uint32_t)CNNUE_AZ_INPUT)));
}

// One warp per board, lane l taking the board's moves l, l + 32, ...: the
// board's 48 context values and the 32 consequence weights sit in shared
// memory, and a move's table rows are read as vectors (float4 for the
// 32-float rows of the consequence section, which start on 16-byte
// boundaries; float2 for the move-context, accumulator-feature and
// accumulator-move sections, whose offsets are 2 mod 4 floats).  Each move's
// 80 terms are added in the CPU twin's order (one product and one add per
// term, no contraction), so outputs stay bit-identical to it.
constexpr int kFwdWarps = 8;

__device__ __forceinline__ float4 ld4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float2 ld2(const float* p) { return __ldg(reinterpret_cast<const float2*>(p)); }

__global__ void __launch_bounds__(32 * kFwdWarps) fused_fwd_kernel(const float* __restrict__ t,
                                                                   const float* __restrict__ ctx,
                                                                   const int64_t* __restrict__ items, int64_t batch,
                                                                   int64_t moves, float* __restrict__ out,
                                                                   uint32_t* status) {
  __shared__ float cons[32];
  __shared__ float cs[kFwdWarps][kCtx];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x < 32) cons[threadIdx.x] = t[kConsequence + threadIdx.x];
  __syncthreads();
  const int64_t n_warps = (int64_t)gridDim.x * kFwdWarps;
  for (int64_t b = (int64_t)blockIdx.x * kFwdWarps + warp; b < batch; b += n_warps) {
    __syncwarp();
    cs[warp][lane] = ctx[b * kCtx + lane];
    if (lane < kCtx - 32) cs[warp][32 + lane] = ctx[b * kCtx + 32 + lane];
    __syncwarp();
    const float* c = cs[warp];
    for (int64_t m = lane; m < moves; m += 32) {
      const int64_t i = b * moves + m;
      const Item it = decode(items[i]);
      if (!it.policy) {
        out[i] = 0.f;
        continue;
      }
      if (!in_range(it)) {
        atomicOr(status, CNNUE_STATUS_BAD_INDEX);
        out[i] = 0.f;
        continue;
      }
      float v = __ldg(t + kBias + it.mv);
      if (it.move) {
        const float* rt = t + it.to * 32;
        const float* rf = t + it.from * 32;
        const float* rc = t + it.cap * 32;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 a = ld4(rt + 4 * q), f = ld4(rf + 4 * q);
          float4 d = make_float4(__fsub_rn(a.x, f.x), __fsub_rn(a.y, f.y), __fsub_rn(a.z, f.z), __fsub_rn(a.w, f.w));
          if (it.capture) {
            const float4 e = ld4(rc + 4 * q);
            d = make_float4(__fsub_rn(d.x, e.x), __fsub_rn(d.y, e.y), __fsub_rn(d.z, e.z), __fsub_rn(d.w, e.w));
          }
          v = __fadd_rn(v, __fmul_rn(d.x, cons[4 * q]));
          v = __fadd_rn(v, __fmul_rn(d.y, cons[4 * q + 1]));
          v = __fadd_rn(v, __fmul_rn(d.z, cons[4 * q + 2]));
          v = __fadd_rn(v, __fmul_rn(d.w, cons[4 * q + 3]));
        }
        const float* mc = t + kContext + it.mv * 16;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float2 w = ld2(mc + 2 * q);
          v = __fadd_rn(v, __fmul_rn(c[2 * q], w.x));
          v = __fadd_rn(v, __fmul_rn(c[2 * q + 1], w.y));
        }
        const float* at = t + kAccFeature + it.to * 32;
        const float* af = t + kAccFeature + it.from * 32;
        const float* ac = t + kAccFeature + it.cap * 32;
        const float* am = t + kAccMove + it.mv * 32;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float2 x = ld2(at + 2 * q), y = ld2(af + 2 * q), w = ld2(am + 2 * q);
          float a0 = __fsub_rn(__fadd_rn(c[16 + 2 * q], x.x), y.x);
          float a1 = __fsub_rn(__fadd_rn(c[17 + 2 * q], x.y), y.y);
          if (it.capture) {
            const float2 z = ld2(ac + 2 * q);
            a0 = __fsub_rn(a0, z.x);
            a1 = __fsub_rn(a1, z.y);
          }
          v = __fadd_rn(v, __fmul_rn(a0, w.x));
          v = __fadd_rn(v, __fmul_rn(a1, w.y));
        }
      }
      out[i] = v;
    }
  }
}

constexpr uint32_t kFeatureKeys = CNNUE_AZ_INPUT;  // drop key of the feature-row sort
constexpr uint32_t kMoveKeys = CNNUE_AZ_DENSE_MOVES;
constexpr int kConsChunk = 256;  // items per ordered chunk of the consequence-weight sums

__device__ __forceinline__ bool live_move(const Item& it) { return it.policy && it.move && in_range(it); }

// Feature-row keys: contribution e = 3 i + slot (slot 0 to, 1 from, 2 captured).
__global__ void fused_feature_keys_kernel(const int64_t* __restrict__ items, int64_t n, uint32_t* __restrict__ keys,
                                          uint32_t* status) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < 3 * n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / 3;
    const int slot = (int)(e - 3 * i);
    const Item it = decode(items[i]);
    if (slot == 0 && it.policy && !in_range(it)) atomicOr(status, CNNUE_STATUS_BAD_INDEX);
    uint32_t k = kFeatureKeys;
    if (live_move(it)) {
      if (slot == 0) k = it.to;
      else if (slot == 1) k = it.from;
      else if (it.capture) k = it.cap;
    }
    keys[e] = k;
  }
}

__global__ void fused_move_keys_kernel(const int64_t* __restrict__ items, int64_t n, uint32_t* __restrict__ keys) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const Item it = decode(items[i]);
    keys[i] = it.policy && in_range(it) ? it.mv : kMoveKeys;
  }
}

// Column h < 32: consequence row; h >= 32: accumulator feature row.
struct FeatureVal {
  const float* t;
  const int64_t* items;
  const float* g;
  __device__ __forceinline__ float operator()(uint32_t e, int64_t h) const {
    const uint32_t i = e / 3u, slot = e - 3u * i;
    const Item it = decode(__ldg(items + i));
    const float w = h < 32 ? __ldg(t + kConsequence + h) : __ldg(t + kAccMove + it.mv * 32 + (h - 32));
    const float gw = __fmul_rn(__ldg(g + i), w);
    return slot == 0 ? gw : -gw;  // grad[from] -= g*w is grad[from] + (-(g*w)), exactly
  }
};
struct FeatureOut {
  float* gt;
  __device__ __forceinline__ float& operator()(uint32_t key, int64_t h) const {
    return h < 32 ? gt[key * 32 + h] : gt[kAccFeature + key * 32 + (h - 32)];
  }
};

// Column 0: move bias; 1..16: move context; 17..48: accumulator move factors.
struct MoveVal {
  const float* t;
  const float* ctx;
  const int64_t* items;
  const float* g;
  int64_t moves;
  __device__ __forceinline__ float operator()(uint32_t i, int64_t h) const {
    const float gi = __ldg(g + i);
    if (h == 0) return gi;
    const Item it = decode(__ldg(items + i));
    if (!it.move) return 0.f;  // adds +0: partial sums here never hold -0
    const float* c = ctx + (i / moves) * kCtx;
    if (h <= 16) return __fmul_rn(gi, __ldg(c + h - 1));
    const int64_t hh = h - 17;
    float after = __fsub_rn(__fadd_rn(__ldg(c + 16 + hh), __ldg(t + kAccFeature + it.to * 32 + hh)),
                            __ldg(t + kAccFeature + it.from * 32 + hh));
    if (it.capture) after = __fsub_rn(after, __ldg(t + kAccFeature + it.cap * 32 + hh));
    return __fmul_rn(gi, after);
  }
};
struct MoveOut {
  float* gt;
  __device__ __forceinline__ float& operator()(uint32_t key, int64_t h) const {
    if (h == 0) return gt[kBias + key];
    if (h <= 16) return gt[kContext + key * 16 + (h - 1)];
    return gt[kAccMove + key * 32 + (h - 17)];
  }
};

// Consequence weights: chunk c of kConsChunk items summed in item order per
// column (8 items' loads in flight); a single chunk writes the result.
__global__ void cons_chunk_kernel(const float* __restrict__ t, const int64_t* __restrict__ items,
                                  const float* __restrict__ g, int64_t n, int64_t n_chunks, float* __restrict__ partial,
                                  float* __restrict__ gt) {
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n_chunks * 32;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = q >> 5;
    const int h = (int)(q & 31);
    const int64_t i0 = c * kConsChunk, i1 = min(n, i0 + kConsChunk);
    float s = 0.f;
    for (int64_t i = i0; i < i1; i += 8) {
      float v[8];
      bool live[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        live[k] = false;
        v[k] = 0.f;
        if (i + k < i1) {
          const Item it = decode(__ldg(items + i + k));
          if (live_move(it)) {
            float delta = __fsub_rn(__ldg(t + it.to * 32 + h), __ldg(t + it.from * 32 + h));
            if (it.capture) delta = __fsub_rn(delta, __ldg(t + it.cap * 32 + h));
            v[k] = __fmul_rn(__ldg(g + i + k), delta);
            live[k] = true;
          }
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (live[k]) s = __fadd_rn(s, v[k]);
    }
    if (n_chunks == 1) gt[kConsequence + h] = s;
    else partial[c * 32 + h] = s;
  }
}

// Chunk partials of one column: lane l sums chunks l, l+32, ... in order,
// then the lanes combine in a fixed butterfly.  One warp per column.
__global__ void cons_final_kernel(const float* __restrict__ partial, int64_t n_chunks, float* __restrict__ gt) {
  const int h = blockIdx.x, lane = threadIdx.x;
  float s = 0.f;
  for (int64_t c = lane; c < n_chunks; c += 32) s = __fadd_rn(s, partial[c * 32 + h]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  if (lane == 0) gt[kConsequence + h] = s;
}

// grad_context[b][col]: the board's moves in order (one thread per (b, col)).
__global__ void fused_ctx_grad_kernel(const float* __restrict__ t, const int64_t* __restrict__ items,
                                      const float* __restrict__ g_out, int64_t batch, int64_t moves,
                                      float* __restrict__ g_ctx) {
  const int64_t n = batch * kCtx;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = q / kCtx;
    const int col = (int)(q - b * kCtx);
    float s = 0.f;
    for (int64_t m = 0; m < moves; ++m) {
      const int64_t i = b * moves + m;
      const Item it = decode(items[i]);
      if (!it.policy || !it.move || !in_range(it)) continue;
      const float w = col < 16 ? t[kContext + it.mv * 16 + col] : t[kAccMove + it.mv * 32 + (col - 16)];
      s = __fadd_rn(s, __fmul_rn(g_out[i], w));
    }
    g_ctx[q] = s;
  }
}

__global__ void table_fwd_kernel(const float* __restrict__ table, int64_t table_len, const int64_t* __restrict__ idx,
                                 int64_t outputs, int terms, float* __restrict__ out, uint32_t* status) {
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < outputs; o += (int64_t)gridDim.x * blockDim.x) {
    float s = -0.f;  // the additive identity Rust's f32 Sum starts from
    for (int k = 0; k < terms; ++k) {
      const int64_t j = idx[o * terms + k];
      if (j < 0 || j >= table_len) {
        atomicOr(status, CNNUE_STATUS_BAD_INDEX);
        continue;
      }
      s = __fadd_rn(s, table[j]);
    }
    out[o] = s;
  }
}

// Contribution (o, k) adds grad_out[o] to entry idx[o * terms + k].  Out of
// range indices are flagged and dropped; so are contributions whose value is
// exactly zero (masked move slots), which change no sum: partial sums here
// start at +0 and never hold -0, and x + (+-0) == x for every other x.
__global__ void index_keys_kernel(const int64_t* __restrict__ idx, const float* __restrict__ grad_out, int terms,
                                  int64_t n, int64_t table_len, uint32_t* __restrict__ keys, uint32_t* status) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = idx[i];
    const bool ok = j >= 0 && j < table_len;
    if (!ok) atomicOr(status, CNNUE_STATUS_BAD_INDEX);
    keys[i] = ok && grad_out[i / terms] != 0.f ? (uint32_t)j : (uint32_t)table_len;  // else dropped
  }
}

// Compact packed batch -> the policy lookups' index arrays (src/az.rs:763-859).
constexpr int64_t kSparseTable = 2396815, kSparseMain = 2086LL * 14 * 81;
constexpr int64_t kTacticalExact = 2086LL * 7 * 64, kTacticalSize = kTacticalExact + 7 * 64;

__global__ void expand_indices_kernel(const int64_t* __restrict__ items, const uint8_t* __restrict__ signature,
                                      const uint8_t* __restrict__ buckets, int64_t batch, int64_t moves,
                                      int64_t* __restrict__ sparse, int64_t* __restrict__ tactical,
                                      float* __restrict__ mask) {
  const int64_t n = batch * moves;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const Item it = decode(items[i]);
    if (mask) mask[i] = it.policy ? 0.f : -1.0e9f;
    int64_t sp[7], ta[2];
    const bool live = it.policy && it.move && in_range(it) && it.from / 90 < 7;
    if (live) {
      const uint32_t b = buckets[i / moves];
      const int us = b & 15, them = b >> 4, pair = us * 9 + them;
      const int piece = it.from / 90, from = it.from % 90, to = it.to % 90;
      const int64_t mv = it.mv;
      // policy_king_distance_buckets (src/az.rs:841-859)
      const int king = 89 - ((7 + them / 3) * 9 + 3 + them % 3);
      const int before = abs(from / 9 - king / 9) + abs(from % 9 - king % 9);
      const int after = abs(to / 9 - king / 9) + abs(to % 9 - king % 9);
      const int approach = min(max(before - after, -2), 2) + 2, distance = min(after, 5);
      const int64_t move_piece = 2086LL * 14, move_king = 2086LL * 81, dist_off = move_piece + move_king + 14 * 81;
      sp[0] = ((mv * 14 + piece) * 9 + us) * 9 + them;
      sp[1] = kSparseMain + mv * 15 + (it.capture ? it.cap / 90 : 14);
      sp[2] = kSparseTable + mv * 14 + piece;
      sp[3] = kSparseTable + move_piece + mv * 81 + pair;
      sp[4] = kSparseTable + move_piece + move_king + piece * 81 + pair;
      sp[5] = kSparseTable + dist_off + piece * 6 + distance;
      sp[6] = kSparseTable + dist_off + 14 * 6 + piece * 5 + approach;
      const int64_t sig = signature[i] & 63;
      ta[0] = (mv * 7 + piece) * 64 + sig;
      ta[1] = kTacticalExact + piece * 64 + sig;
    } else {
#pragma unroll
      for (int k = 0; k < 7; ++k) sp[k] = kSparseTable - 1;
      ta[0] = ta[1] = kTacticalSize;
    }
#pragma unroll
    for (int k = 0; k < 7; ++k) sparse[i * 7 + k] = sp[k];
    tactical[i * 2] = ta[0];
    tactical[i * 2 + 1] = ta[1];
  }
}

inline unsigned grid_for(int64_t n) { return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 16)); }

}  // namespace
}  // namespace pol
}  // namespace cnnue

using namespace cnnue;
using namespace cnnue::pol;

extern "C" {

int cnnue_policy_fused_fwd(const float* d_tables, const float* d_context, const int64_t* d_items, int64_t batch,
                           int64_t moves, float* d_out, uint32_t* d_status, void* stream) {
  if (batch < 0 || moves < 0 || (batch * moves > 0 && (!d_tables || !d_context || !d_items || !d_out || !d_status)))
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer or negative size");
  if (batch * moves == 0) return CNNUE_OK;
  if ((uintptr_t)d_tables & 15u) return set_error(CNNUE_ERR_INVALID_ARG, "d_tables must be 16-byte aligned");
  const int64_t blocks = std::min<int64_t>((batch + kFwdWarps - 1) / kFwdWarps, 148 * 16);
  fused_fwd_kernel<<<(unsigned)blocks, 32 * kFwdWarps, 0, (cudaStream_t)stream>>>(d_tables, d_context, d_items,
                                                                                 batch, moves, d_out, d_status);
  return check_launch_error("fused_fwd_kernel");
}

size_t cnnue_policy_fused_bwd_workspace_bytes(int64_t batch, int64_t moves) {
  const int64_t n = std::max<int64_t>(batch * moves, 0);
  const int64_t chunks = std::max<int64_t>((n + kConsChunk - 1) / kConsChunk, 1);
  return sizeof(WorkspaceHeader) + align_up((size_t)std::max<int64_t>(3 * n, 1) * 4, 256) +
         align_up((size_t)std::max<int64_t>(n, 1) * 4, 256) + align_up((size_t)chunks * 32 * 4, 256) +
         std::max(scat::workspace_bytes(3 * n, 64), scat::workspace_bytes(n, 49));
}

int cnnue_policy_fused_bwd(const float* d_tables, const float* d_context, const int64_t* d_items,
                           const float* d_grad_out, int64_t batch, int64_t moves, float* d_grad_tables,
                           float* d_grad_context, void* ws, size_t ws_bytes, void* stream) {
  if (batch < 0 || moves < 0 || !ws || !d_grad_tables ||
      (batch * moves > 0 && (!d_tables || !d_context || !d_items || !d_grad_out || !d_grad_context)))
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer or negative size");
  if (ws_bytes < cnnue_policy_fused_bwd_workspace_bytes(batch, moves))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu < %zu bytes", ws_bytes,
                     cnnue_policy_fused_bwd_workspace_bytes(batch, moves));
  const int64_t n = batch * moves;
  if (3 * n >= (int64_t)UINT32_MAX) return set_error(CNNUE_ERR_INVALID_ARG, "batch x moves too large");
  cudaStream_t s = (cudaStream_t)stream;
  CNNUE_CUDA_TRY(cudaMemsetAsync(ws, 0, sizeof(WorkspaceHeader), s));
  CNNUE_CUDA_TRY(cudaMemsetAsync(d_grad_tables, 0, sizeof(float) * kTableLen, s));
  if (n == 0) return CNNUE_OK;
  uint32_t* status = &((WorkspaceHeader*)ws)->status;
  char* p = (char*)ws + sizeof(WorkspaceHeader);
  uint32_t* fkeys = (uint32_t*)p;
  p += align_up((size_t)(3 * n) * 4, 256);
  uint32_t* mkeys = (uint32_t*)p;
  p += align_up((size_t)n * 4, 256);
  const int64_t chunks = (n + kConsChunk - 1) / kConsChunk;
  float* cons_partial = (float*)p;
  p += align_up((size_t)chunks * 32 * 4, 256);
  fused_feature_keys_kernel<<<grid_for(3 * n), 256, 0, s>>>(d_items, n, fkeys, status);
  if (int st = check_launch_error("fused_feature_keys_kernel")) return st;
  fused_move_keys_kernel<<<grid_for(n), 256, 0, s>>>(d_items, n, mkeys);
  if (int st = check_launch_error("fused_move_keys_kernel")) return st;
  fused_ctx_grad_kernel<<<grid_for(batch * kCtx), 256, 0, s>>>(d_tables, d_items, d_grad_out, batch, moves,
                                                              d_grad_context);
  if (int st = check_launch_error("fused_ctx_grad_kernel")) return st;
  cons_chunk_kernel<<<grid_for(chunks * 32), 256, 0, s>>>(d_tables, d_items, d_grad_out, n, chunks, cons_partial,
                                                          d_grad_tables);
  if (int st = check_launch_error("cons_chunk_kernel")) return st;
  if (chunks > 1) {
    cons_final_kernel<<<32, 32, 0, s>>>(cons_partial, chunks, d_grad_tables);
    if (int st = check_launch_error("cons_final_kernel")) return st;
  }
  // the two row sorts share the scatter workspace (stream order separates them)
  if (int st = scat::launch_scatter_rows(fkeys, FeatureVal{d_tables, d_items, d_grad_out}, FeatureOut{d_grad_tables},
                                         64, 3 * n, kFeatureKeys, p, s))
    return st;
  return scat::launch_scatter_rows(mkeys, MoveVal{d_tables, d_context, d_items, d_grad_out, moves},
                                   MoveOut{d_grad_tables}, 49, n, kMoveKeys, p, s);
}

int cnnue_policy_table_fwd(const float* d_table, int64_t table_len, const int64_t* d_indices, int64_t outputs,
                           int terms, float* d_out, uint32_t* d_status, void* stream) {
  if (outputs < 0 || terms <= 0 || table_len <= 0 ||
      (outputs > 0 && (!d_table || !d_indices || !d_out || !d_status)))
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer or bad size");
  if (outputs == 0) return CNNUE_OK;
  table_fwd_kernel<<<grid_for(outputs), 256, 0, (cudaStream_t)stream>>>(d_table, table_len, d_indices, outputs,
                                                                        terms, d_out, d_status);
  return check_launch_error("table_fwd_kernel");
}

size_t cnnue_policy_table_bwd_workspace_bytes(int64_t outputs, int terms) {
  const int64_t n = std::max<int64_t>(outputs, 0) * std::max(terms, 1);
  return sizeof(WorkspaceHeader) + align_up((size_t)n * 4, 256) + scat::workspace_bytes(n);
}

int cnnue_policy_table_bwd(const int64_t* d_indices, const float* d_grad_out, int64_t outputs, int terms,
                           int64_t table_len, float* d_grad_table, void* ws, size_t ws_bytes, void* stream) {
  if (outputs < 0 || terms <= 0 || table_len <= 0 || table_len >= (int64_t)UINT32_MAX || !ws || !d_grad_table ||
      (outputs > 0 && (!d_indices || !d_grad_out)))
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer or bad size");
  if (ws_bytes < cnnue_policy_table_bwd_workspace_bytes(outputs, terms))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu < %zu bytes", ws_bytes,
                     cnnue_policy_table_bwd_workspace_bytes(outputs, terms));
  const int64_t n = outputs * terms;
  if (n >= (int64_t)UINT32_MAX) return set_error(CNNUE_ERR_INVALID_ARG, "too many indices");
  cudaStream_t s = (cudaStream_t)stream;
  CNNUE_CUDA_TRY(cudaMemsetAsync(ws, 0, sizeof(WorkspaceHeader), s));
  uint32_t* status = &((WorkspaceHeader*)ws)->status;
  uint32_t* keys = (uint32_t*)((char*)ws + sizeof(WorkspaceHeader));
  void* scratch = (char*)keys + align_up((size_t)n * 4, 256);
  if (n > 0) {
    index_keys_kernel<<<grid_for(n), 256, 0, s>>>(d_indices, d_grad_out, terms, n, table_len, keys, status);
    if (int st = check_launch_error("index_keys_kernel")) return st;
  }
  return scat::launch_scatter_add(keys, d_grad_out, (uint32_t)terms, n, table_len, d_grad_table, scratch, s);
}

int cnnue_az_expand_policy_indices(const int64_t* d_items, const uint8_t* d_signature, const uint8_t* d_king_buckets,
                                   int64_t batch, int64_t moves, int64_t* d_sparse, int64_t* d_tactical,
                                   float* d_mask, void* stream) {
  if (batch < 0 || moves < 0 ||
      (batch * moves > 0 && (!d_items || !d_signature || !d_king_buckets || !d_sparse || !d_tactical)))
    return set_error(CNNUE_ERR_INVALID_ARG, "null buffer or negative size");
  if (batch * moves == 0) return CNNUE_OK;
  expand_indices_kernel<<<grid_for(batch * moves), 256, 0, (cudaStream_t)stream>>>(
      d_items, d_signature, d_king_buckets, batch, moves, d_sparse, d_tactical, d_mask);
  return check_launch_error("expand_indices_kernel");
}

}  // extern "C"
