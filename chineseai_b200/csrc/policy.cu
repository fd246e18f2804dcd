// policy.cu - the AZ-NNUE policy-head training ops (Candle custom ops of the
// reference): fused_policy (src/az/fused_policy.rs) and the sparse / tactical
// table lookups (src/az/fused_sparse_policy.rs), forward and backward.
//
// Forward kernels keep the CPU twins' operation order (one product and one
// add per term, no fused multiply-add), so outputs are bit-identical to them.
// Backward passes are atomic-free: every scalar contribution to the table
// gradient becomes a (table entry, value) pair, summed per entry in
// contribution order by the deterministic scatter (scatter.cuh); the context
// gradient of a board is summed over its moves in order by one thread per
// (board, context column).
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
constexpr int kMaxContrib = 1 + 4 * 32 + 16 + 4 * 32;  // table contributions of one item

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

__global__ void fused_fwd_kernel(const float* __restrict__ t, const float* __restrict__ ctx,
                                 const int64_t* __restrict__ items, int64_t batch, int64_t moves,
                                 float* __restrict__ out, uint32_t* status) {
  const int64_t n = batch * moves;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
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
    float v = t[kBias + it.mv];
    if (it.move) {
      const float* c = ctx + (i / moves) * kCtx;
      for (int h = 0; h < 32; ++h) {
        float delta = __fsub_rn(t[it.to * 32 + h], t[it.from * 32 + h]);
        if (it.capture) delta = __fsub_rn(delta, t[it.cap * 32 + h]);
        v = __fadd_rn(v, __fmul_rn(delta, t[kConsequence + h]));
      }
      for (int h = 0; h < 16; ++h) v = __fadd_rn(v, __fmul_rn(c[h], t[kContext + it.mv * 16 + h]));
      for (int h = 0; h < 32; ++h) {
        float after = __fsub_rn(__fadd_rn(c[16 + h], t[kAccFeature + it.to * 32 + h]), t[kAccFeature + it.from * 32 + h]);
        if (it.capture) after = __fsub_rn(after, t[kAccFeature + it.cap * 32 + h]);
        v = __fadd_rn(v, __fmul_rn(after, t[kAccMove + it.mv * 32 + h]));
      }
    }
    out[i] = v;
  }
}

// Table contributions of item i, kMaxContrib slots (unused slots get key
// kTableLen, dropped by the scatter as "no table entry").
__global__ void fused_contrib_kernel(const float* __restrict__ t, const float* __restrict__ ctx,
                                     const int64_t* __restrict__ items, const float* __restrict__ g_out,
                                     int64_t batch, int64_t moves, uint32_t* __restrict__ keys,
                                     float* __restrict__ vals, uint32_t* status) {
  const int64_t n = batch * moves;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    uint32_t* k = keys + i * kMaxContrib;
    float* v = vals + i * kMaxContrib;
    int c = 0;
    const Item it = decode(items[i]);
    const bool ok = it.policy && in_range(it);
    if (it.policy && !ok) atomicOr(status, CNNUE_STATUS_BAD_INDEX);
    if (ok) {
      const float g = g_out[i];
      k[c] = kBias + it.mv;
      v[c++] = g;
      if (it.move) {
        const float* cx = ctx + (i / moves) * kCtx;
        for (int h = 0; h < 32; ++h) {
          const float w = t[kConsequence + h];
          float delta = __fsub_rn(t[it.to * 32 + h], t[it.from * 32 + h]);
          const float gw = __fmul_rn(g, w);
          k[c] = it.to * 32 + h;
          v[c++] = gw;
          k[c] = it.from * 32 + h;
          v[c++] = -gw;
          if (it.capture) {
            delta = __fsub_rn(delta, t[it.cap * 32 + h]);
            k[c] = it.cap * 32 + h;
            v[c++] = -gw;
          }
          k[c] = kConsequence + h;
          v[c++] = __fmul_rn(g, delta);
        }
        for (int h = 0; h < 16; ++h) {
          k[c] = kContext + it.mv * 16 + h;
          v[c++] = __fmul_rn(g, cx[h]);
        }
        for (int h = 0; h < 32; ++h) {
          const uint32_t mf = kAccMove + it.mv * 32 + h;
          const float w = t[mf];
          float after = __fsub_rn(__fadd_rn(cx[16 + h], t[kAccFeature + it.to * 32 + h]), t[kAccFeature + it.from * 32 + h]);
          const float gw = __fmul_rn(g, w);
          k[c] = kAccFeature + it.to * 32 + h;
          v[c++] = gw;
          k[c] = kAccFeature + it.from * 32 + h;
          v[c++] = -gw;
          if (it.capture) {
            after = __fsub_rn(after, t[kAccFeature + it.cap * 32 + h]);
            k[c] = kAccFeature + it.cap * 32 + h;
            v[c++] = -gw;
          }
          k[c] = mf;
          v[c++] = __fmul_rn(g, after);
        }
      }
    }
    for (; c < kMaxContrib; ++c) {
      k[c] = kTableLen;
      v[c] = 0.f;
    }
  }
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

__global__ void index_keys_kernel(const int64_t* __restrict__ idx, int64_t n, int64_t table_len,
                                  uint32_t* __restrict__ keys, uint32_t* status) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = idx[i];
    const bool ok = j >= 0 && j < table_len;
    if (!ok) atomicOr(status, CNNUE_STATUS_BAD_INDEX);
    keys[i] = ok ? (uint32_t)j : (uint32_t)table_len;  // out of range: dropped by the scatter
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
  fused_fwd_kernel<<<grid_for(batch * moves), 256, 0, (cudaStream_t)stream>>>(d_tables, d_context, d_items, batch,
                                                                              moves, d_out, d_status);
  return check_launch_error("fused_fwd_kernel");
}

size_t cnnue_policy_fused_bwd_workspace_bytes(int64_t batch, int64_t moves) {
  const int64_t n = std::max<int64_t>(batch * moves, 0) * kMaxContrib;
  return sizeof(WorkspaceHeader) + align_up((size_t)n * 4, 256) * 2 + scat::workspace_bytes(n);
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
  const int64_t n = batch * moves * kMaxContrib;
  if (n >= (int64_t)UINT32_MAX) return set_error(CNNUE_ERR_INVALID_ARG, "batch x moves too large");
  cudaStream_t s = (cudaStream_t)stream;
  CNNUE_CUDA_TRY(cudaMemsetAsync(ws, 0, sizeof(WorkspaceHeader), s));
  uint32_t* status = &((WorkspaceHeader*)ws)->status;
  char* p = (char*)ws + sizeof(WorkspaceHeader);
  uint32_t* keys = (uint32_t*)p;
  p += align_up((size_t)n * 4, 256);
  float* vals = (float*)p;
  p += align_up((size_t)n * 4, 256);
  if (batch * moves > 0) {
    fused_contrib_kernel<<<grid_for(batch * moves), 256, 0, s>>>(d_tables, d_context, d_items, d_grad_out, batch,
                                                                moves, keys, vals, status);
    if (int st = check_launch_error("fused_contrib_kernel")) return st;
    fused_ctx_grad_kernel<<<grid_for(batch * kCtx), 256, 0, s>>>(d_tables, d_items, d_grad_out, batch, moves,
                                                                d_grad_context);
    if (int st = check_launch_error("fused_ctx_grad_kernel")) return st;
  }
  // unused slots carry key kTableLen, which the scatter drops
  return scat::launch_scatter_add(keys, vals, 1, n, kTableLen, d_grad_tables, p, s);
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
    index_keys_kernel<<<grid_for(n), 256, 0, s>>>(d_indices, n, table_len, keys, status);
    if (int st = check_launch_error("index_keys_kernel")) return st;
  }
  return scat::launch_scatter_add(keys, d_grad_out, (uint32_t)terms, n, table_len, d_grad_table, scratch, s);
}

}  // extern "C"
