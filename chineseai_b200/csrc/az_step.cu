// az_step.cu - the AZ-NNUE training step as native kernels: forward of
// AzCandleModel (src/az/candle_model.rs:46-147), the loss of
// compute_batch_loss (src/az/train_gpu_candle.rs:221-305), and the backward
// of every one of the 22 weight tensors, in a fixed number of launches
// whatever the batch (no autograd graph, no library GEMM).
//
// Stream layout of one step (cnnue_azt_step):
//   main:  zero the gradient | forward (trunk per board + accumulator
//          features) | policy logits + both losses + the logit gradients
//          (per board) | trunk backward (per board) | wait for the side
//          stream | table gradient block sums | cross-block run sums |
//          weight-gradient tiles + feature-row gradient + metrics
//   side:  one key per table contribution of the batch | one joint LSD radix
//          sort of all of them (scatter.cuh)
// The batch alone decides which table rows a step touches, so the sort runs
// beside the forward and the per-board backward.
//
// Every table gradient (feature pool rows, threat rows, policy move rows,
// policy feature rows, sparse and tactical scalars) is one sort problem in
// a joint key space.  The sorted contributions are summed in aligned blocks
// of 64 positions, one warp per block, each stretch of equal keys in sorted
// (= contribution) order; runs that cross a block boundary add their block
// partials in block order afterwards.  Dense weight gradients are
// reductions over the batch's boards, computed as tiles with a fixed split
// of the boards and a fixed order of the split partials.  No atomics touch
// a value, so a step is deterministic run to run.
#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "scatter.cuh"

namespace cnnue {
namespace azt {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr uint32_t kPad = 0xffffffffu;
constexpr int kTrunkRows = CNNUE_AZ_TRUNK_ROWS;  // 1545
constexpr int kInput = CNNUE_AZ_INPUT;           // 1260
constexpr int kVH = CNNUE_AZ_VALUE_HEAD;         // 96
constexpr int kRule = CNNUE_AZ_RULE_CONTEXT;     // 7
constexpr int kVocab = CNNUE_AZ_THREAT_VOCAB;    // 57702
constexpr int kTR = CNNUE_AZ_THREAT_RANK;        // 64
constexpr int kPair = 2 * kTR;                   // 128: [act, act^2]
constexpr int kMoves = CNNUE_AZ_DENSE_MOVES;     // 2086
constexpr int kCtx = CNNUE_POLICY_CONTEXT;       // 48 = 16 move context + 32 accumulator
constexpr int kAcc = 32;                         // accumulator rank
constexpr int kPsp = 32;                         // consequence columns of the feature rows
constexpr int64_t kSparseLen = 2596273;          // sparse table + sparse factors
constexpr int64_t kTactLen = 934977;             // tactical table + its constant zero
constexpr float kMaskDrop = -1.0e8f;             // masked (the packer writes -1e9)

// Joint key space of the table gradients.
constexpr uint32_t kKeyPool = 0;
constexpr uint32_t kKeyThreat = kKeyPool + kTrunkRows;
constexpr uint32_t kKeyMove = kKeyThreat + kVocab;
constexpr uint32_t kKeyFeat = kKeyMove + kMoves;
constexpr uint32_t kKeyRowsEnd = kKeyFeat + kInput;  // keys below: row problems
constexpr uint32_t kKeySparse = kKeyRowsEnd;
constexpr uint32_t kKeyTact = kKeySparse + (uint32_t)kSparseLen;
constexpr uint32_t kKeyDrop = kKeyTact + (uint32_t)kTactLen;
constexpr int kMoveW = 16 + kAcc + 1;  // move row: move context, accumulator move, bias
constexpr int kRowStride = 64;         // floats per stored move / feature gradient row
constexpr int kMultBits = 11;          // trunk payload: board << 11 | multiplicity (<= 5 x 256)
constexpr uint32_t kNegBit = 1u << 31; // feature payload: the row enters subtracted
constexpr int kFeatW = kPsp + kAcc;    // feature row: consequence rows, accumulator features

constexpr int kWarps = 8;  // warps per block of every per-board kernel

// The 17 parameter leaves of the flat buffer (tensors 0-4 form the trunk
// table, 19-20 the sparse table).
enum Leaf {
  L_FT, L_RULE, L_HB, L_VHH, L_VHB, L_VHO, L_TE, L_VTO, L_PTC, L_MB, L_CONS, L_PCH, L_MC, L_PAH, L_AM, L_SPARSE,
  L_TACT, kLeaves
};
static_assert(kLeaves == CNNUE_AZT_LEAVES, "leaf count");
static_assert(kAcc == 32 && kVH == 96, "the forward's 32-output products");

struct Params {
  const float* p[kLeaves];
};
struct Grads {
  float* g[kLeaves];
};

struct Batch {
  int64_t B, F, M, T;
  const uint32_t* fi;   // [B][F]
  const uint32_t* ti;   // [B][T]
  const int64_t* pi;    // [B][M]
  const int64_t* sp;    // [B][M][7]
  const int64_t* tc;    // [B][M][2]
  const float* tgt;     // [B][M]
  const float* mask;    // [B][M]
  const float* wdl;     // [B][3]
  const float* values;  // [B]
  const float* rule;    // [B][7]
  const float* pw;      // [B]
  const float* vw;      // [B]
  const float* phase;   // [B][3]
};

// Contribution index bases of the joint sort.
struct Bases {
  uint32_t pool, threat, move, feat, sparse, tact, n;
};
__host__ __device__ inline Bases bases(int64_t B, int64_t F, int64_t M, int64_t T) {
  Bases b;
  b.pool = 0;
  b.threat = (uint32_t)(B * F * 6);
  b.move = b.threat + (uint32_t)(B * T);
  b.feat = b.move + (uint32_t)(B * M);
  b.sparse = b.feat + (uint32_t)(B * M * 3);
  b.tact = b.sparse + (uint32_t)(B * M * 7);
  b.n = b.tact + (uint32_t)(B * M * 2);
  return b;
}

// Per-board and per-step buffers of the workspace.
struct Act {
  float *bp, *hid, *rms, *vh, *ta, *ctx, *vl, *af;      // forward
  float *dl, *dvl, *dctx, *cons, *rec;                  // loss
  float *mrow, *frow;                                   // per move: its move-row and feature-row gradients
  uint32_t *pay;                                        // [n] payload of every contribution slot
  float *dbp, *dpre, *dta, *dvh;                        // backward
  float *pspaf;                                         // [1260][64] feature-row gradients
  float *part, *tile_part;                              // segment partials (head, tail per block), tile partials
  uint32_t *keys, *counters, *tile_cnt;
  int row_w;                                            // partial row width max(H, 64)
  uint32_t part_slots;                                  // 2 x blocks of the largest sort
  uint32_t* status;
};

// A failed self-check: counters[2] gets the first check's code, counters[3..4]
// its operands; the status word gets CNNUE_STATUS_INTERNAL; the access is
// skipped by the caller.
__device__ __noinline__ void check_failed(const Act& A, uint32_t code, uint32_t a, uint32_t b) {
  if (atomicCAS(A.counters + 2, 0u, code) == 0u) {
    A.counters[3] = a;
    A.counters[4] = b;
  }
  atomicOr(A.status, CNNUE_STATUS_INTERNAL);
}

// ---- policy items (src/az/fused_policy.rs:10-35) -----------------------------
struct Item {
  bool policy, move, capture;
  uint32_t mv, from, to, cap;
};
__device__ __forceinline__ Item decode(int64_t packed_s) {
  const uint64_t p = (uint64_t)packed_s;
  Item it;
  it.policy = (p >> 47) & 1u;
  it.move = (p >> 45) & 1u;
  it.capture = (p >> 46) & 1u;
  it.mv = (uint32_t)(p & 0xfffu);
  it.from = (uint32_t)((p >> 12) & 0x7ffu);
  it.to = (uint32_t)((p >> 23) & 0x7ffu);
  it.cap = (uint32_t)((p >> 34) & 0x7ffu);
  return it;
}
__device__ __forceinline__ bool in_range(const Item& it) {
  return it.mv < (uint32_t)kMoves &&
         (!it.move || (it.from < (uint32_t)kInput && it.to < (uint32_t)kInput &&
                       (!it.capture || it.cap < (uint32_t)kInput)));
}

// Trunk feature item -> its six rows (fused_feature_pool.rs:389-403); 0 for
// padding, -1 when a row falls outside the table.
__device__ __forceinline__ int pool_rows(uint32_t packed, uint32_t rows[6]) {
  if (packed == kPad) return 0;
  const uint32_t feature = packed & 0x7ffu, us = (packed >> 11) & 0xfu, them = (packed >> 15) & 0xfu;
  const uint32_t piece = feature / 90u, square = feature - piece * 90u;
  rows[0] = feature;
  rows[1] = 1260u + piece;
  rows[2] = 1274u + square / 9u;
  rows[3] = 1284u + square % 9u;
  rows[4] = 1293u + us * 14u + piece;
  rows[5] = 1293u + (9u + them) * 14u + piece;
  bool ok = true;
#pragma unroll
  for (int r = 0; r < 6; ++r) ok &= rows[r] < (uint32_t)kTrunkRows;
  return ok ? 6 : -1;
}

// ---- warp helpers ----------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
  return v;
}
// v[o] holds each lane's partial of output o (o < 32); afterwards v[0] of
// lane l is the sum over lanes of output l (31 shuffles for 32 outputs).
__device__ __forceinline__ void reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool up = lane & off;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = up ? v[i] : v[i + off];
      const float keep = up ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(kFull, send, off);
    }
  }
}

// A lane's columns of an H = 32 * NC row: chunks of V consecutive columns,
// chunk q at V * lane + 32 * V * q (16-byte loads when NC % 4 == 0).
template <int NC>
struct Lay {
  static constexpr int V = NC % 4 == 0 ? 4 : (NC % 2 == 0 ? 2 : 1);
  static constexpr int Q = NC / V;
  static __device__ __forceinline__ int col(int lane, int q) { return V * lane + 32 * V * q; }
};
template <int NC>
__device__ __forceinline__ void ld_row(const float* __restrict__ row, int lane, float (&x)[NC]) {
  using L = Lay<NC>;
#pragma unroll
  for (int q = 0; q < L::Q; ++q) {
    const float* p = row + L::col(lane, q);
    if constexpr (L::V == 4) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(p));
      x[4 * q] = t.x, x[4 * q + 1] = t.y, x[4 * q + 2] = t.z, x[4 * q + 3] = t.w;
    } else if constexpr (L::V == 2) {
      const float2 t = __ldg(reinterpret_cast<const float2*>(p));
      x[2 * q] = t.x, x[2 * q + 1] = t.y;
    } else {
      x[q] = __ldg(p);
    }
  }
}
// The same for rows written earlier in this kernel's grid or by this step
// (plain loads, no read-only path).
template <int NC>
__device__ __forceinline__ void ld_row_rw(const float* row, int lane, float (&x)[NC]) {
  using L = Lay<NC>;
#pragma unroll
  for (int q = 0; q < L::Q; ++q) {
    const float* p = row + L::col(lane, q);
    if constexpr (L::V == 4) {
      const float4 t = *reinterpret_cast<const float4*>(p);
      x[4 * q] = t.x, x[4 * q + 1] = t.y, x[4 * q + 2] = t.z, x[4 * q + 3] = t.w;
    } else if constexpr (L::V == 2) {
      const float2 t = *reinterpret_cast<const float2*>(p);
      x[2 * q] = t.x, x[2 * q + 1] = t.y;
    } else {
      x[q] = *p;
    }
  }
}
template <int NC>
__device__ __forceinline__ void st_row(float* row, int lane, const float (&x)[NC]) {
  using L = Lay<NC>;
#pragma unroll
  for (int q = 0; q < L::Q; ++q) {
    float* p = row + L::col(lane, q);
    if constexpr (L::V == 4) {
      *reinterpret_cast<float4*>(p) = make_float4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3]);
    } else if constexpr (L::V == 2) {
      *reinterpret_cast<float2*>(p) = make_float2(x[2 * q], x[2 * q + 1]);
    } else {
      *p = x[q];
    }
  }
}
// This lane's partial of dot(W row, x).
template <int NC>
__device__ __forceinline__ float dot_row(const float* __restrict__ wrow, int lane, const float (&x)[NC]) {
  float w[NC];
  ld_row<NC>(wrow, lane, w);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NC; ++i) s = fmaf(w[i], x[i], s);
  return s;
}
// x += a * W row.
template <int NC>
__device__ __forceinline__ void axpy_row(const float* __restrict__ wrow, int lane, float a, float (&x)[NC]) {
  float w[NC];
  ld_row<NC>(wrow, lane, w);
#pragma unroll
  for (int i = 0; i < NC; ++i) x[i] = fmaf(a, w[i], x[i]);
}
// The 32 outputs of W[32][H] . x; lane l gets output l.
template <int NC>
__device__ __forceinline__ float matvec32(const float* __restrict__ W, int H, const float (&x)[NC], int lane) {
  float v[32];
#pragma unroll
  for (int o = 0; o < 32; ++o) v[o] = dot_row<NC>(W + (size_t)o * H, lane, x);
  reduce_scatter32(v, lane);
  return v[0];
}

// ---- keys of every table contribution (side stream) -----------------------------
// Trunk-table contributions, per board (one warp): one per feature item (its
// feature row) and one per distinct derived row (piece, rank, file and king
// rows, 285 in all) with the number of the board's items that hit it as a
// multiplicity - the board gradient times that count.  The trunk section
// holds B x F feature slots, then 5F derived slots per board (a board hits
// at most 5F derived rows).  Then one thread per further contribution slot
// (threat rows, and per policy move its move row, feature rows and lookups).
// A contribution that cannot change a table gradient gets kKeyDrop:
// padding items and threats, moves without the policy bit (torch.where
// passes them no gradient), feature rows of moves without the move bit or
// of an absent capture, and the sparse / tactical lookups of padded moves
// (no policy bit, masked, zero target: their softmax probability underflows
// to exactly 0, so their logit gradient is exactly 0).  Indices outside
// their tables set CNNUE_STATUS_BAD_INDEX and are dropped.  counters[0]
// gets the number of row-problem contributions kept, counters[1] the number
// of scalar-table ones (each sort drops the others in its first pass).  Each slot also
// gets its payload, carried through the sort: where its value row lives -
// board << kMultBits | multiplicity (trunk), board (threat), move (move row,
// scalar tables), move | kNegBit for a subtracted feature row.
constexpr int kDerived = kTrunkRows - kInput;  // 285

__global__ void __launch_bounds__(256) keygen_kernel(Batch bt, Bases cb, uint32_t* __restrict__ keys,
                                                     uint32_t* __restrict__ pay, uint32_t* __restrict__ counters,
                                                     uint32_t* __restrict__ status, int pool_blocks) {
  __shared__ uint32_t hist[kWarps][kDerived];
  __shared__ uint32_t part[2][kWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t rows_kept = 0, scalars_kept = 0;
  bool bad = false;
  if ((int)blockIdx.x < pool_blocks) {
    const int64_t b = (int64_t)blockIdx.x * kWarps + warp;
    if (b < bt.B) {
      uint32_t* h = hist[warp];
      for (int i = lane; i < kDerived; i += 32) h[i] = 0;
      __syncwarp();
      for (int64_t i = lane; i < bt.F; i += 32) {
        uint32_t rows[6];
        const int r = pool_rows(bt.fi[b * bt.F + i], rows);
        bad |= r < 0;
        keys[cb.pool + b * bt.F + i] = r > 0 ? kKeyPool + rows[0] : kKeyDrop;
        pay[cb.pool + b * bt.F + i] = (uint32_t)b << kMultBits | 1u;
        if (r > 0) {
          ++rows_kept;
#pragma unroll
          for (int q = 1; q < 6; ++q) atomicAdd(&h[rows[q] - kInput], 1u);  // counts: order-free
        }
      }
      __syncwarp();
      const int64_t slots = 5 * bt.F;
      const int64_t dkey = cb.pool + bt.B * bt.F + b * slots;
      uint32_t used = 0;
      for (int bin0 = 0; bin0 < kDerived; bin0 += 32) {
        const int bin = bin0 + lane;
        const uint32_t c = bin < kDerived ? h[bin] : 0u;
        const uint32_t m = __ballot_sync(kFull, c > 0);
        if (c > 0) {
          const uint32_t pos = used + __popc(m & ((1u << lane) - 1u));
          if (pos < slots) {
            keys[dkey + pos] = kKeyPool + kInput + bin;
            pay[dkey + pos] = (uint32_t)b << kMultBits | c;
          } else {
            atomicOr(status, CNNUE_STATUS_INTERNAL);
          }
        }
        used += __popc(m);
      }
      for (int64_t k = used + lane; k < slots; k += 32) keys[dkey + k] = kKeyDrop;
      if (lane == 0) rows_kept += used;
    }
  } else {
    // one thread per contribution slot after the trunk section: threat
    // slots, then per move its move row, 3 feature rows, 7 sparse and 2
    // tactical lookups (each section contiguous: coalesced reads and writes)
    const int64_t first = cb.threat, total = (int64_t)cb.n - first;
    const int64_t stride = (int64_t)(gridDim.x - pool_blocks) * blockDim.x;
    for (int64_t t = (int64_t)(blockIdx.x - pool_blocks) * blockDim.x + threadIdx.x; t < total; t += stride) {
      const uint32_t slot = (uint32_t)(first + t);
      uint32_t key = kKeyDrop, py = 0;
      bool row = false;
      if (slot < cb.move) {
        const uint32_t idx = bt.ti[t];
        const bool ok = idx < (uint32_t)kVocab;
        bad |= !ok && idx != kPad;
        key = ok ? kKeyThreat + idx : kKeyDrop;
        py = (uint32_t)(t / bt.T);
        row = true;
      } else if (slot < cb.sparse) {
        const bool is_move = slot < cb.feat;
        const uint32_t u = is_move ? slot - cb.move : (slot - cb.feat) / 3u;
        const uint32_t role = is_move ? 0u : (slot - cb.feat) - 3u * u;
        const Item it = decode(bt.pi[u]);
        const bool ok = in_range(it);
        bad |= is_move && it.policy && !ok;
        const bool on = it.policy && ok;
        if (is_move) {
          key = on ? kKeyMove + it.mv : kKeyDrop;
          py = u;
        } else {
          const bool feat = on && it.move && (role < 2 || it.capture);
          key = feat ? kKeyFeat + (role == 0 ? it.to : role == 1 ? it.from : it.cap) : kKeyDrop;
          py = role == 0 ? u : u | kNegBit;
        }
        row = true;
      } else {
        const bool sparse = slot < cb.tact;
        const uint32_t r = sparse ? slot - cb.sparse : slot - cb.tact;
        const uint32_t u = sparse ? r / 7u : r >> 1;
        const int64_t sx = sparse ? bt.sp[r] : bt.tc[r];
        const bool sok = sx >= 0 && sx < (sparse ? kSparseLen : kTactLen);
        bad |= !sok;
        const Item it = decode(bt.pi[u]);
        const bool drop = !it.policy && bt.mask[u] <= kMaskDrop && bt.tgt[u] == 0.f;
        key = sok && !drop ? (sparse ? kKeySparse : kKeyTact) + (uint32_t)sx : kKeyDrop;
        py = u;
      }
      keys[slot] = key;
      pay[slot] = py;
      const bool kept = key < kKeyDrop;
      rows_kept += row && kept;
      scalars_kept += !row && kept;
    }
  }
  // block totals (counts: order-free)
  uint32_t v0 = rows_kept, v1 = scalars_kept;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    v0 += __shfl_xor_sync(kFull, v0, o);
    v1 += __shfl_xor_sync(kFull, v1, o);
  }
  if (lane == 0) part[0][warp] = v0, part[1][warp] = v1;
  if (__any_sync(kFull, bad) && lane == 0) atomicOr(status, CNNUE_STATUS_BAD_INDEX);
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t s0 = 0, s1 = 0;
    for (int w = 0; w < kWarps; ++w) s0 += part[0][w], s1 += part[1][w];
    if (s0) atomicAdd(counters, s0);
    if (s1) atomicAdd(counters + 1, s1);
  }
}

// ---- forward -------------------------------------------------------------------------
// Blocks [0, B): one block of kBW warps per board -
//   warp 0 lists the board's trunk rows (feature rows, and the distinct
//   derived rows with multiplicities from a shared histogram) while warps
//   1.. accumulate the threat rows; all warps then split the trunk rows;
//   board_pre = pool + hidden bias, sparse_hidden = relu(board_pre + rule .
//   R), hidden = RMS-normed (every warp), then one 32-output product per
//   warp: warp 0 the accumulator context W_acc . board_pre and the move
//   context W_pc . hidden + W_ptc . pair, warps 1-3 the value head groups;
//   warp 0 finishes with the value logits W_o . value head + W_to . pair
//   (pair = [act, act^2], act = clamp(threat, 0, 1));
// blocks after them: one warp per input row r < 1260 - the accumulator
// features af[r] = W_acc . trunk_table[r] (32 values).
constexpr int kBW = 4;  // warps per board in the forward and policy kernels
static_assert(kBW == 1 + kVH / 32, "one value-head group per warp after warp 0");

// Shared floats of the forward's block: partial sums (kBW x H), threat partials
// (kBW x 64), the value head (96), the derived-row histogram (kDerived + 1,
// even) and up to F + kDerived (row, multiplicity) pairs.
__host__ __device__ inline int64_t fwd_smem_words(int64_t F, int64_t H) {
  return kBW * H + kBW * kTR + kVH + kDerived + 1 + 2 * (F + kDerived);
}

template <int NC>
__global__ void __launch_bounds__(32 * kBW) fwd_kernel(Params P, Batch bt, Act A, int trunk_blocks,
                                                       uint32_t* __restrict__ status) {
  constexpr int H = 32 * NC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if ((int)blockIdx.x >= trunk_blocks) {
    const int r = ((int)blockIdx.x - trunk_blocks) * kBW + warp;
    if (r >= kInput) return;
    float x[NC];
    ld_row<NC>(P.p[L_FT] + (size_t)r * H, lane, x);
    A.af[(size_t)r * kAcc + lane] = matvec32<NC>(P.p[L_PAH], H, x, lane);
    return;
  }
  const int64_t b = blockIdx.x;
  extern __shared__ uint32_t fsm[];
  float* part = reinterpret_cast<float*>(fsm);  // [kBW][H]
  float* tpart = part + kBW * H;                // [kBW][64]
  float* vhs = tpart + kBW * kTR;               // [96]
  uint32_t* hist = reinterpret_cast<uint32_t*>(vhs + kVH);
  uint2* list = reinterpret_cast<uint2*>(hist + kDerived + 1);  // 8-byte aligned: every offset before is even
  __shared__ uint32_t s_nlist;
  __shared__ int s_flags;
  if (threadIdx.x == 0) s_flags = 0;
  bool bad = false, bad_list = false;
  if (warp == 0) {
    for (int i = lane; i < kDerived; i += 32) hist[i] = 0;
    __syncwarp();
    uint32_t n_list = 0;
    for (int64_t i0 = 0; i0 < bt.F; i0 += 32) {
      uint32_t rows[6];
      const int r = i0 + lane < bt.F ? pool_rows(bt.fi[b * bt.F + i0 + lane], rows) : 0;
      bad |= r < 0;
      const uint32_t m = __ballot_sync(kFull, r > 0);
      if (r > 0) {
        list[n_list + __popc(m & ((1u << lane) - 1u))] = make_uint2(rows[0], __float_as_uint(1.f));
#pragma unroll
        for (int q = 1; q < 6; ++q) atomicAdd(&hist[rows[q] - kInput], 1u);
      }
      n_list += __popc(m);
    }
    __syncwarp();
    for (int bin0 = 0; bin0 < kDerived; bin0 += 32) {
      const int bin = bin0 + lane;
      const uint32_t c = bin < kDerived ? hist[bin] : 0u;
      const uint32_t m = __ballot_sync(kFull, c > 0);
      const uint32_t pos = n_list + __popc(m & ((1u << lane) - 1u));
      if (c > 0 && pos < (uint32_t)(bt.F + kDerived)) list[pos] = make_uint2(kInput + bin, __float_as_uint((float)c));
      bad_list |= c > 0 && pos >= (uint32_t)(bt.F + kDerived);
      n_list += __popc(m);
    }
    if (lane == 0) s_nlist = n_list < (uint32_t)(bt.F + kDerived) ? n_list : (uint32_t)(bt.F + kDerived);
    reinterpret_cast<float2*>(tpart)[lane] = make_float2(0.f, 0.f);
  } else {
    // threat rows: chunks of 32 indices (one per lane) dealt round-robin to
    // warps 1.., rows loaded eight at a time; lane owns columns 2 lane, 2 lane + 1
    float t0 = 0.f, t1 = 0.f;
    for (int64_t i0 = (int64_t)(warp - 1) * 32; i0 < bt.T; i0 += (int64_t)(kBW - 1) * 32) {
      const uint32_t mine = i0 + lane < bt.T ? bt.ti[b * bt.T + i0 + lane] : kPad;
      bad |= mine >= (uint32_t)kVocab && mine != kPad;
      const int cnt = (int)(bt.T - i0 < 32 ? bt.T - i0 : 32);
      for (int j0 = 0; j0 < cnt; j0 += 8) {
        float2 v[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const uint32_t idx = __shfl_sync(kFull, mine, (j0 + t) & 31);
          v[t] = j0 + t < cnt && idx < (uint32_t)kVocab
                     ? __ldg(reinterpret_cast<const float2*>(P.p[L_TE] + (size_t)idx * kTR) + lane)
                     : make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          t0 += v[t].x;
          t1 += v[t].y;
        }
      }
    }
    reinterpret_cast<float2*>(tpart + warp * kTR)[lane] = make_float2(t0, t1);
  }
  __syncthreads();
  // trunk rows: batches of eight dealt round-robin to the warps
  const uint32_t n_list = s_nlist;
  constexpr int kB = NC > 4 ? 4 : 8;
  float acc[NC];
#pragma unroll
  for (int i = 0; i < NC; ++i) acc[i] = 0.f;
  for (uint32_t j0 = (uint32_t)warp * kB; j0 < n_list; j0 += kBW * kB) {
    float x[kB][NC], mult[kB];
#pragma unroll
    for (int t = 0; t < kB; ++t) {
      const bool ok = j0 + t < n_list;
      const uint2 e = ok ? list[j0 + t] : make_uint2(0u, 0u);
      mult[t] = __uint_as_float(e.y);
      ld_row<NC>(P.p[L_FT] + (size_t)e.x * H, lane, x[t]);
    }
#pragma unroll
    for (int t = 0; t < kB; ++t)
      if (j0 + t < n_list)
#pragma unroll
        for (int c = 0; c < NC; ++c) acc[c] = fmaf(mult[t], x[t][c], acc[c]);
  }
  st_row<NC>(part + warp * H, lane, acc);
  __syncthreads();
  // every warp: board_pre (partials added in warp order), rule, relu, RMS
  float bias[NC], bp[NC], h[NC];
  ld_row<NC>(P.p[L_HB], lane, bias);
#pragma unroll
  for (int c = 0; c < NC; ++c) bp[c] = 0.f;
#pragma unroll
  for (int w = 0; w < kBW; ++w) {
    float x[NC];
    ld_row_rw<NC>(part + w * H, lane, x);
#pragma unroll
    for (int c = 0; c < NC; ++c) bp[c] += x[c];
  }
#pragma unroll
  for (int c = 0; c < NC; ++c) bp[c] += bias[c];
  float pre[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) pre[c] = 0.f;
#pragma unroll
  for (int k = 0; k < kRule; ++k) axpy_row<NC>(P.p[L_RULE] + (size_t)k * H, lane, __ldg(bt.rule + b * kRule + k), pre);
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    h[c] = fmaxf(bp[c] + pre[c], 0.f);
    ss = fmaf(h[c], h[c], ss);
  }
  const float rms = sqrtf(warp_sum(ss) / (float)H + 1.0e-6f);
#pragma unroll
  for (int c = 0; c < NC; ++c) h[c] = h[c] / rms;
  float t0 = 0.f, t1 = 0.f;
#pragma unroll
  for (int w = 0; w < kBW; ++w) {
    const float2 v = reinterpret_cast<const float2*>(tpart + w * kTR)[lane];
    t0 += v.x;
    t1 += v.y;
  }
  const float a0 = fminf(fmaxf(t0, 0.f), 1.f), a1 = fminf(fmaxf(t1, 0.f), 1.f);
  const float pr[4] = {a0, a1, a0 * a0, a1 * a1};  // pair columns 2l, 2l+1, 64+2l, 65+2l
  const int pc[4] = {2 * lane, 2 * lane + 1, kTR + 2 * lane, kTR + 2 * lane + 1};
  if (warp > 0) {
    const int g = warp - 1;
    const float vh =
        fmaxf(matvec32<NC>(P.p[L_VHH] + (size_t)32 * g * H, H, h, lane) + __ldg(P.p[L_VHB] + 32 * g + lane), 0.f);
    vhs[32 * g + lane] = vh;
    A.vh[b * kVH + 32 * g + lane] = vh;
  } else {
    const float acc_ctx = matvec32<NC>(P.p[L_PAH], H, bp, lane);
    // move context (16): hidden and pair terms in one reduce-scatter
    float v[32];
#pragma unroll
    for (int o = 0; o < 32; ++o) {
      float sm = 0.f;
      if (o < 16) {
        sm = dot_row<NC>(P.p[L_PCH] + (size_t)o * H, lane, h);
#pragma unroll
        for (int q = 0; q < 4; ++q) sm = fmaf(pr[q], __ldg(P.p[L_PTC] + o * kPair + pc[q]), sm);
      }
      v[o] = sm;
    }
    reduce_scatter32(v, lane);
    if (lane < 16) A.ctx[b * kCtx + lane] = v[0];
    A.ctx[b * kCtx + 16 + lane] = acc_ctx;
    st_row<NC>(A.bp + b * H, lane, bp);
    st_row<NC>(A.hid + b * H, lane, h);
    if (lane == 0) A.rms[b] = rms;
    reinterpret_cast<float2*>(A.ta + b * kTR)[lane] = make_float2(t0, t1);
  }
  if (__any_sync(kFull, bad) && lane == 0) atomicOr(&s_flags, 1);
  if (__any_sync(kFull, bad_list) && lane == 0) atomicOr(&s_flags, 2);
  __syncthreads();
  if (warp == 0) {
    // value logits from the value head (shared) and the pair
    float vl[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      float sm = 0.f;
#pragma unroll
      for (int g = 0; g < 3; ++g) sm = fmaf(vhs[32 * g + lane], __ldg(P.p[L_VHO] + k * kVH + 32 * g + lane), sm);
#pragma unroll
      for (int q = 0; q < 4; ++q) sm = fmaf(pr[q], __ldg(P.p[L_VTO] + k * kPair + pc[q]), sm);
      vl[k] = warp_sum(sm);
    }
    if (lane < 3) A.vl[b * 4 + lane] = lane == 0 ? vl[0] : (lane == 1 ? vl[1] : vl[2]);
    if (lane == 0 && (s_flags & 1)) atomicOr(status, CNNUE_STATUS_BAD_INDEX);
    if (lane == 0 && (s_flags & 2)) atomicOr(status, CNNUE_STATUS_INTERNAL);
  }
}

// ---- policy logits, losses, logit gradients ------------------------------------------
// One block of kBW warps per board, thread t taking moves t, t + 32 kBW, ...
// (block reductions add the warps' results in warp order).  A move's logit is
// (policy bit set) bias[mv] + move_bit * (consequence . (psp[to] - psp[from]
// - capture * psp[cap]) + ctx16 . move_context[mv] + (ctx32 + af[to] -
// af[from] - capture * af[cap]) . accumulator_move[mv]), else 0, plus its 7
// sparse and 2 tactical lookups (fused_policy.rs:178-241,
// fused_sparse_policy.rs:8-34); psp = trunk_table[:, :32].  Then, per board
// (compute_batch_loss): log-softmax of logits + mask, policy CE = -sum t *
// log p, dlogit = pw_scale * w_b / B * (p * sum t - t); value log-softmax,
// CE against the WDL target, value = p_win - p_loss, dvalue_logit likewise.
// The board's move-context gradient (48) and its share of the consequence
// weights' gradient (32) are summed over its moves here.
__device__ __forceinline__ float4 ld4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 sub4(float4 a, float4 b) {
  return make_float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w);
}

struct LossScale {
  float value, policy;  // max(weight, 0) / B
};

// Block sum (or max) of one value per thread: warp butterflies, then the
// warps' results in warp order; every thread gets the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = red[0];
#pragma unroll
  for (int w = 1; w < kBW; ++w) t += red[w];
  return t;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = red[0];
#pragma unroll
  for (int w = 1; w < kBW; ++w) t = fmaxf(t, red[w]);
  return t;
}

__global__ void __launch_bounds__(32 * kBW, 4) policy_kernel(Params P, Batch bt, Act A, int H, LossScale ls,
                                                          uint32_t* __restrict__ status) {
  extern __shared__ float smem[];
  __shared__ float cons[kPsp];
  __shared__ float sctx[kCtx];
  __shared__ float red[kBW];
  __shared__ float gred[kBW][96];
  __shared__ int s_bad;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* z = smem;  // the board's logits, then probabilities
  const int64_t b = blockIdx.x;
  if (threadIdx.x < kPsp) cons[threadIdx.x] = __ldg(P.p[L_CONS] + threadIdx.x);
  if (threadIdx.x < kCtx) sctx[threadIdx.x] = A.ctx[b * kCtx + threadIdx.x];
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  const float* c = sctx;
  const float* ft = P.p[L_FT];
  bool bad = false;
  float zmax = -INFINITY;
  for (int64_t m = threadIdx.x; m < bt.M; m += 32 * kBW) {
    const int64_t u = b * bt.M + m;
    const Item it = decode(bt.pi[u]);
    float v = 0.f;
    if (it.policy) {
      if (!in_range(it)) {
        bad = true;
      } else {
        v = __ldg(P.p[L_MB] + it.mv);
        if (it.move) {
          const float* rt = ft + (size_t)it.to * H;
          const float* rf = ft + (size_t)it.from * H;
          const float* rc = ft + (size_t)it.cap * H;
          float s = 0.f;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float4 d = sub4(ld4(rt + 4 * q), ld4(rf + 4 * q));
            if (it.capture) d = sub4(d, ld4(rc + 4 * q));
            s = fmaf(d.x, cons[4 * q], s);
            s = fmaf(d.y, cons[4 * q + 1], s);
            s = fmaf(d.z, cons[4 * q + 2], s);
            s = fmaf(d.w, cons[4 * q + 3], s);
          }
          const float* mc = P.p[L_MC] + (size_t)it.mv * 16;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 w = ld4(mc + 4 * q);
            s = fmaf(c[4 * q], w.x, s);
            s = fmaf(c[4 * q + 1], w.y, s);
            s = fmaf(c[4 * q + 2], w.z, s);
            s = fmaf(c[4 * q + 3], w.w, s);
          }
          const float* at = A.af + (size_t)it.to * kAcc;
          const float* af = A.af + (size_t)it.from * kAcc;
          const float* ac = A.af + (size_t)it.cap * kAcc;
          const float* am = P.p[L_AM] + (size_t)it.mv * kAcc;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float4 x = sub4(*reinterpret_cast<const float4*>(at + 4 * q), *reinterpret_cast<const float4*>(af + 4 * q));
            if (it.capture) x = sub4(x, *reinterpret_cast<const float4*>(ac + 4 * q));
            const float4 w = ld4(am + 4 * q);
            s = fmaf(c[16 + 4 * q] + x.x, w.x, s);
            s = fmaf(c[17 + 4 * q] + x.y, w.y, s);
            s = fmaf(c[18 + 4 * q] + x.z, w.z, s);
            s = fmaf(c[19 + 4 * q] + x.w, w.w, s);
          }
          v += s;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 7; ++j) {
      const int64_t s = bt.sp[u * 7 + j];
      if (s >= 0 && s < kSparseLen) v += __ldg(P.p[L_SPARSE] + s);
      else bad = true;
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int64_t s = bt.tc[u * 2 + j];
      if (s >= 0 && s < kTactLen) v += __ldg(P.p[L_TACT] + s);
      else bad = true;
    }
    const float zz = v + bt.mask[u];
    z[m] = zz;
    zmax = fmaxf(zmax, zz);
  }
  zmax = block_max(zmax, red);
  float se = 0.f;
  for (int64_t m = threadIdx.x; m < bt.M; m += 32 * kBW) se += expf(z[m] - zmax);
  const float lse = zmax + logf(block_sum(se, red));
  float ce = 0.f, tsum = 0.f;
  for (int64_t m = threadIdx.x; m < bt.M; m += 32 * kBW) {
    const float lp = z[m] - lse, t = bt.tgt[b * bt.M + m];
    ce -= t * lp;
    tsum += t;
    z[m] = expf(lp);
  }
  ce = block_sum(ce, red);
  tsum = block_sum(tsum, red);
  const float scale_p = ls.policy * __ldg(bt.pw + b);
  // logit gradients and the board's move-context / consequence sums
  float g16[32], g32[32], gc[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) g16[j] = g32[j] = gc[j] = 0.f;
  for (int64_t m = threadIdx.x; m < bt.M; m += 32 * kBW) {
    const int64_t u = b * bt.M + m;
    const float dl = scale_p * (z[m] * tsum - bt.tgt[u]);
    A.dl[u] = dl;
    const Item it = decode(bt.pi[u]);
    if (!it.policy || !in_range(it)) continue;
    // the move's gradient rows, read by the table sums: move row [dl ctx16,
    // dl (ctx32 + af delta), dl], feature row [dl consequence, dl acc move]
    float* mrow = A.mrow + (size_t)u * kRowStride;
    mrow[kMoveW - 1] = dl;
    if (!it.move) {
#pragma unroll
      for (int q = 0; q < 12; ++q) reinterpret_cast<float4*>(mrow)[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      continue;
    }
    float* frow = A.frow + (size_t)u * kRowStride;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      reinterpret_cast<float4*>(mrow)[q] =
          make_float4(dl * c[4 * q], dl * c[4 * q + 1], dl * c[4 * q + 2], dl * c[4 * q + 3]);
    const float* at = A.af + (size_t)it.to * kAcc;
    const float* af = A.af + (size_t)it.from * kAcc;
    const float* ac = A.af + (size_t)it.cap * kAcc;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 x = sub4(*reinterpret_cast<const float4*>(at + 4 * q), *reinterpret_cast<const float4*>(af + 4 * q));
      if (it.capture) x = sub4(x, *reinterpret_cast<const float4*>(ac + 4 * q));
      reinterpret_cast<float4*>(mrow + 16)[q] =
          make_float4(dl * (c[16 + 4 * q] + x.x), dl * (c[17 + 4 * q] + x.y), dl * (c[18 + 4 * q] + x.z),
                      dl * (c[19 + 4 * q] + x.w));
      reinterpret_cast<float4*>(frow)[q] =
          make_float4(dl * cons[4 * q], dl * cons[4 * q + 1], dl * cons[4 * q + 2], dl * cons[4 * q + 3]);
    }
    const float* mc = P.p[L_MC] + (size_t)it.mv * 16;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 w = ld4(mc + 4 * q);
      g16[4 * q] = fmaf(dl, w.x, g16[4 * q]);
      g16[4 * q + 1] = fmaf(dl, w.y, g16[4 * q + 1]);
      g16[4 * q + 2] = fmaf(dl, w.z, g16[4 * q + 2]);
      g16[4 * q + 3] = fmaf(dl, w.w, g16[4 * q + 3]);
    }
    const float* am = P.p[L_AM] + (size_t)it.mv * kAcc;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 w = ld4(am + 4 * q);
      g32[4 * q] = fmaf(dl, w.x, g32[4 * q]);
      g32[4 * q + 1] = fmaf(dl, w.y, g32[4 * q + 1]);
      g32[4 * q + 2] = fmaf(dl, w.z, g32[4 * q + 2]);
      g32[4 * q + 3] = fmaf(dl, w.w, g32[4 * q + 3]);
      reinterpret_cast<float4*>(frow + kPsp)[q] = make_float4(dl * w.x, dl * w.y, dl * w.z, dl * w.w);
    }
    const float* rt = ft + (size_t)it.to * H;
    const float* rf = ft + (size_t)it.from * H;
    const float* rc = ft + (size_t)it.cap * H;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 d = sub4(ld4(rt + 4 * q), ld4(rf + 4 * q));
      if (it.capture) d = sub4(d, ld4(rc + 4 * q));
      gc[4 * q] = fmaf(dl, d.x, gc[4 * q]);
      gc[4 * q + 1] = fmaf(dl, d.y, gc[4 * q + 1]);
      gc[4 * q + 2] = fmaf(dl, d.z, gc[4 * q + 2]);
      gc[4 * q + 3] = fmaf(dl, d.w, gc[4 * q + 3]);
    }
  }
  reduce_scatter32(g16, lane);
  reduce_scatter32(g32, lane);
  reduce_scatter32(gc, lane);
  gred[warp][lane] = g16[0];
  gred[warp][32 + lane] = g32[0];
  gred[warp][64 + lane] = gc[0];
  if (__any_sync(kFull, bad) && lane == 0) s_bad = 1;
  __syncthreads();
  if (warp == 0) {
    float x[3];
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      x[q] = gred[0][32 * q + lane];
#pragma unroll
      for (int w = 1; w < kBW; ++w) x[q] += gred[w][32 * q + lane];
    }
    if (lane < 16) A.dctx[b * kCtx + lane] = x[0];
    A.dctx[b * kCtx + 16 + lane] = x[1];
    A.cons[b * kPsp + lane] = x[2];
    if (lane == 0 && s_bad) atomicOr(status, CNNUE_STATUS_BAD_INDEX);
  }
  // value head loss (thread 0)
  if (threadIdx.x == 0) {
    const float l0 = A.vl[b * 4], l1 = A.vl[b * 4 + 1], l2 = A.vl[b * 4 + 2];
    const float mx = fmaxf(l0, fmaxf(l1, l2));
    const float lse3 = mx + logf(expf(l0 - mx) + expf(l1 - mx) + expf(l2 - mx));
    const float lp[3] = {l0 - lse3, l1 - lse3, l2 - lse3};
    const float w0 = bt.wdl[b * 3], w1 = bt.wdl[b * 3 + 1], w2 = bt.wdl[b * 3 + 2];
    const float vce = -(w0 * lp[0] + w1 * lp[1] + w2 * lp[2]);
    const float p0 = expf(lp[0]), p1 = expf(lp[1]), p2 = expf(lp[2]);
    const float wsum = w0 + w1 + w2;
    const float sv = ls.value * __ldg(bt.vw + b);
    A.dvl[b * 4] = sv * (p0 * wsum - w0);
    A.dvl[b * 4 + 1] = sv * (p1 * wsum - w1);
    A.dvl[b * 4 + 2] = sv * (p2 * wsum - w2);
    A.dvl[b * 4 + 3] = 0.f;
    float* r = A.rec + b * 8;
    r[0] = vce * __ldg(bt.vw + b);
    r[1] = ce * __ldg(bt.pw + b);
    r[2] = vce;
    r[3] = ce;
    r[4] = p0 - p2;  // value = p . (1, 0, -1)
  }
}

// ---- trunk backward (one warp per board) -------------------------------------------
// From dvalue_logits (3) and the move-context gradient (48):
//   dvh = W_o^T dvl (where value head > 0), dpair = W_to^T dvl + W_ptc^T dctx16,
//   dthreat = (dpair[:64] + 2 act dpair[64:]) where 0 <= threat <= 1,
//   dhidden = W_v^T dvh + W_pc^T dctx16,
//   dsparse = (dhidden - hidden * mean(dhidden * hidden)) / rms where > 0,
//   dboard = dsparse + W_acc^T dctx32.
template <int NC>
__global__ void __launch_bounds__(32 * kWarps) bwd_kernel(Params P, Batch bt, Act A) {
  constexpr int H = 32 * NC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t b = (int64_t)blockIdx.x * kWarps + warp;
  if (b >= bt.B) return;
  const float dv0 = A.dvl[b * 4], dv1 = A.dvl[b * 4 + 1], dv2 = A.dvl[b * 4 + 2];
  const float c16 = lane < 16 ? A.dctx[b * kCtx + lane] : 0.f;
  const float c32 = A.dctx[b * kCtx + 16 + lane];
  // value head pre-activation gradient: lane owns outputs lane, 32 + lane, 64 + lane
  float dvh[3];
#pragma unroll
  for (int g = 0; g < 3; ++g) {
    const int o = 32 * g + lane;
    const float t = dv0 * __ldg(P.p[L_VHO] + o) + dv1 * __ldg(P.p[L_VHO] + kVH + o) +
                    dv2 * __ldg(P.p[L_VHO] + 2 * kVH + o);
    dvh[g] = A.vh[b * kVH + o] > 0.f ? t : 0.f;
    A.dvh[b * kVH + o] = dvh[g];
  }
  // threat: lane owns columns 2 lane, 2 lane + 1 of act (pair 2l, 2l+1, 64+2l, 65+2l)
  const float2 ta = reinterpret_cast<const float2*>(A.ta + b * kTR)[lane];
  const int pc[4] = {2 * lane, 2 * lane + 1, kTR + 2 * lane, kTR + 2 * lane + 1};
  float dp[4];
#pragma unroll
  for (int q = 0; q < 4; ++q)
    dp[q] = dv0 * __ldg(P.p[L_VTO] + pc[q]) + dv1 * __ldg(P.p[L_VTO] + kPair + pc[q]) +
            dv2 * __ldg(P.p[L_VTO] + 2 * kPair + pc[q]);
#pragma unroll
  for (int o = 0; o < 16; ++o) {
    const float co = __shfl_sync(kFull, c16, o);
#pragma unroll
    for (int q = 0; q < 4; ++q) dp[q] = fmaf(co, __ldg(P.p[L_PTC] + o * kPair + pc[q]), dp[q]);
  }
  const float a0 = fminf(fmaxf(ta.x, 0.f), 1.f), a1 = fminf(fmaxf(ta.y, 0.f), 1.f);
  const float d0 = dp[0] + 2.f * a0 * dp[2], d1 = dp[1] + 2.f * a1 * dp[3];
  reinterpret_cast<float2*>(A.dta + b * kTR)[lane] =
      make_float2(ta.x >= 0.f && ta.x <= 1.f ? d0 : 0.f, ta.y >= 0.f && ta.y <= 1.f ? d1 : 0.f);
  // hidden
  float dh[NC];
#pragma unroll
  for (int i = 0; i < NC; ++i) dh[i] = 0.f;
#pragma unroll
  for (int g = 0; g < 3; ++g)
#pragma unroll 8
    for (int j = 0; j < 32; ++j)
      axpy_row<NC>(P.p[L_VHH] + (size_t)(32 * g + j) * H, lane, __shfl_sync(kFull, dvh[g], j), dh);
#pragma unroll
  for (int o = 0; o < 16; ++o) axpy_row<NC>(P.p[L_PCH] + (size_t)o * H, lane, __shfl_sync(kFull, c16, o), dh);
  float h[NC];
  ld_row_rw<NC>(A.hid + b * H, lane, h);
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < NC; ++i) dot = fmaf(dh[i], h[i], dot);
  const float mean = warp_sum(dot) / (float)H;
  const float rms = A.rms[b];
  float dpre[NC], dbp[NC];
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    dpre[i] = h[i] > 0.f ? (dh[i] - h[i] * mean) / rms : 0.f;
    dbp[i] = dpre[i];
  }
#pragma unroll 8
  for (int j = 0; j < kAcc; ++j) axpy_row<NC>(P.p[L_PAH] + (size_t)j * H, lane, __shfl_sync(kFull, c32, j), dbp);
  st_row<NC>(A.dpre + b * H, lane, dpre);
  st_row<NC>(A.dbp + b * H, lane, dbp);
}

// ---- table gradients: segment sums over the joint sort ---------------------------------
// The sorted contributions are cut into aligned blocks of kSeg positions; a
// segment is a maximal stretch of equal keys inside one block.  One warp per
// block sums its segments in position (= contribution) order: a segment that
// is its key's whole run writes the gradient row (or scalar) directly; a
// segment continuing from the previous block leaves its partial in the
// block's head slot, one that only continues into the next block in the tail
// slot.  The combine kernel then gives every run crossing a block boundary to
// one warp, which adds the run's tail partial and the head partials of the
// following blocks in block order.  Every contribution's value is a row (or
// scalar) already in memory, found from the payload it carries through the
// sort: the board gradient times a multiplicity (trunk rows), the threat
// gradient, the move's move row or signed feature row, or dlogit.
constexpr int kSeg = 64;

// Two sorted arrays (row keys, scalar-table keys: disjoint key ranges, so a
// run never spans both); their blocks are enumerated one after the other.
struct Sorted {
  const uint32_t* keys[2];    // [n_live] sorted keys
  const uint32_t* pay[2];     // [n_live] payload of each sorted slot
  const uint32_t* n_live[2];  // device words: contributions kept
  uint32_t n_max[2];          // contribution slots (bounds n_live)
  uint32_t slot_base[2];      // first partial slot of each array's blocks
};

// The value row of a contribution: src[c] * mult for c < W (W = 0: none).
struct Src {
  const float* src;
  float mult;
  int W;
};
__device__ __forceinline__ Src source(const Act& A, const Batch& bt, uint32_t key, uint32_t pay, int H) {
  const uint32_t nbm = (uint32_t)(bt.B * bt.M);
  if (key < kKeyMove) {
    const bool trunk = key < kKeyThreat;
    const uint32_t b = trunk ? pay >> kMultBits : pay;
    if (b >= (uint32_t)bt.B) {
      check_failed(A, trunk ? 6 : 7, key, pay);
      return {A.dl, 0.f, 0};
    }
    return trunk ? Src{A.dbp + (size_t)b * H, (float)(pay & ((1u << kMultBits) - 1u)), H}
                 : Src{A.dta + (size_t)b * kTR, 1.f, kTR};
  }
  const uint32_t u = key < kKeyRowsEnd ? pay & ~kNegBit : pay;
  if (u >= nbm || key >= kKeyDrop) {
    check_failed(A, 8, key, pay);
    return {A.dl, 0.f, 0};
  }
  if (key < kKeyFeat) return {A.mrow + (size_t)u * kRowStride, 1.f, kMoveW};
  if (key < kKeyRowsEnd) return {A.frow + (size_t)u * kRowStride, (pay & kNegBit) ? -1.f : 1.f, kFeatW};
  return {A.dl + u, 1.f, 1};
}
__device__ __forceinline__ int key_width(uint32_t key, int H) {
  return key < kKeyThreat ? H : key < kKeyMove ? kTR : key < kKeyFeat ? kMoveW : key < kKeyRowsEnd ? kFeatW : 1;
}
__device__ __forceinline__ float* key_dest(const Grads& G, const Act& A, uint32_t key, int c, int H) {
  if (key < kKeyThreat) return G.g[L_FT] + (size_t)(key - kKeyPool) * H + c;
  if (key < kKeyMove) return G.g[L_TE] + (size_t)(key - kKeyThreat) * kTR + c;
  if (key < kKeyFeat) {
    const uint32_t mv = key - kKeyMove;
    return c < 16 ? G.g[L_MC] + (size_t)mv * 16 + c
                  : c < 16 + kAcc ? G.g[L_AM] + (size_t)mv * kAcc + (c - 16) : G.g[L_MB] + mv;
  }
  if (key < kKeyRowsEnd) return A.pspaf + (size_t)(key - kKeyFeat) * kFeatW + c;
  return key < kKeyTact ? G.g[L_SPARSE] + (key - kKeySparse) : G.g[L_TACT] + (key - kKeyTact);
}

template <int NC>
__global__ void __launch_bounds__(256, 3) seg_kernel(Grads G, Act A, Batch bt, Sorted s, int H) {
  constexpr int KW = NC > 2 ? NC : 2;   // column chunks of the widest row: max(H, 64) / 32
  constexpr int BT = NC > 4 ? 4 : 8;    // positions whose loads are in flight together
  const int lane = threadIdx.x & 31;
  const uint32_t n0 = min(*s.n_live[0], s.n_max[0]), n1 = min(*s.n_live[1], s.n_max[1]);
  const uint32_t nb0 = (n0 + kSeg - 1) / kSeg, nb1 = (n1 + kSeg - 1) / kSeg;
  const uint32_t gw = (uint32_t)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const uint32_t n_warps = (uint32_t)((gridDim.x * blockDim.x) >> 5);
  for (uint32_t g = gw; g < nb0 + nb1; g += n_warps) {
    const int sg = g < nb0 ? 0 : 1;
    const uint32_t blk = sg ? g - nb0 : g, n = sg ? n1 : n0;
    const uint32_t* keys = s.keys[sg];
    const uint32_t* pays = s.pay[sg];
    const uint32_t slot = s.slot_base[sg] + 2 * blk;
    const uint32_t base = blk * kSeg;
    const int cnt = n - base < (uint32_t)kSeg ? (int)(n - base) : kSeg;
    const uint32_t k_lo = lane < cnt ? keys[base + lane] : kKeyDrop;
    const uint32_t k_hi = 32 + lane < cnt ? keys[base + 32 + lane] : kKeyDrop;
    const uint32_t p_lo = lane < cnt ? pays[base + lane] : 0u;
    const uint32_t p_hi = 32 + lane < cnt ? pays[base + 32 + lane] : 0u;
    const uint32_t first = __shfl_sync(kFull, k_lo, 0);
    if (first >= kKeyDrop) continue;  // keys ascend: the block is all dropped
    const uint32_t prev = base > 0 ? keys[base - 1] : 0xffffffffu;
    const uint32_t next = base + cnt < n ? keys[base + cnt] : 0xffffffffu;
    if (slot + 1 >= A.part_slots) {
      if (lane == 0) check_failed(A, 11, blk, A.part_slots);
      continue;
    }
    float* head_slot = A.part + (size_t)slot * A.row_w;
    float* tail_slot = head_slot + A.row_w;
    if (first >= kKeyRowsEnd) {
      // scalar block: each lane loads its two positions, then one pass in order
      float v_lo = 0.f, v_hi = 0.f;
      if (k_lo < kKeyDrop) {
        const Src q = source(A, bt, k_lo, p_lo, H);
        if (q.W) v_lo = *q.src;
      }
      if (k_hi < kKeyDrop) {
        const Src q = source(A, bt, k_hi, p_hi, H);
        if (q.W) v_hi = *q.src;
      }
      // segmented inclusive scans over the lanes (a fixed shuffle tree), one
      // per half of the block; every shuffle runs on all lanes
      const uint32_t lt = (1u << lane) - 1u, me = 1u << lane;
      const uint32_t klo_up = __shfl_up_sync(kFull, k_lo, 1), khi_up = __shfl_up_sync(kFull, k_hi, 1);
      const uint32_t klo_dn = __shfl_down_sync(kFull, k_lo, 1), khi_dn = __shfl_down_sync(kFull, k_hi, 1);
      const uint32_t khi_0 = __shfl_sync(kFull, k_hi, 0), klo_31 = __shfl_sync(kFull, k_lo, 31);
      const uint32_t bal_lo = __ballot_sync(kFull, lane == 0 || klo_up != k_lo);
      const uint32_t bal_hi = __ballot_sync(kFull, lane == 0 || khi_up != k_hi);
      const int seg_lo = 31 - __clz(bal_lo & (lt | me)), seg_hi = 31 - __clz(bal_hi & (lt | me));
      float x_lo = v_lo, x_hi = v_hi;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y_lo = __shfl_up_sync(kFull, x_lo, o), y_hi = __shfl_up_sync(kFull, x_hi, o);
        if (lane - o >= seg_lo) x_lo += y_lo;
        if (lane - o >= seg_hi) x_hi += y_hi;
      }
      // the high half's first segment continues the low half's last one
      const float carry = __shfl_sync(kFull, x_lo, 31);
      const int first_hi_end = (bal_hi & ~1u) ? __ffs(bal_hi & ~1u) - 2 : 31;
      if (cnt > 32 && khi_0 == klo_31 && lane <= first_hi_end) x_hi += carry;
      const uint32_t kfirst = __shfl_sync(kFull, k_lo, 0);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int j = 32 * half + lane;
        const uint32_t key = half ? k_hi : k_lo;
        const uint32_t kn = half ? khi_dn : (lane < 31 ? klo_dn : khi_0);
        const bool end = j < cnt && key < kKeyDrop && (j == cnt - 1 || kn != key);
        if (!end) continue;
        const float x = half ? x_hi : x_lo;
        const bool head = key == kfirst && prev == key;  // keys ascend: such a segment starts the block
        const bool tail = j == cnt - 1 && next == key;
        if (head) *head_slot = x;
        else if (tail) *tail_slot = x;
        else *key_dest(G, A, key, 0, H) = x;
      }
      continue;
    }
    float acc[KW];
#pragma unroll
    for (int k = 0; k < KW; ++k) acc[k] = 0.f;
    int seg_start = 0;
    bool done = false;
    for (int j0 = 0; j0 < cnt && !done; j0 += BT) {
      uint32_t kk[BT + 1];
#pragma unroll
      for (int t = 0; t <= BT; ++t) {
        const int j = j0 + t;
        const uint32_t k = __shfl_sync(kFull, (j & 32) ? k_hi : k_lo, j & 31);
        kk[t] = j < cnt ? k : next;
      }
      float v[BT][KW];
#pragma unroll
      for (int t = 0; t < BT; ++t) {
        const int j = j0 + t;
        const uint32_t py = __shfl_sync(kFull, (j & 32) ? p_hi : p_lo, j & 31);
        const Src q = j < cnt && kk[t] < kKeyDrop ? source(A, bt, kk[t], py, H) : Src{A.dl, 0.f, 0};
#pragma unroll
        for (int k = 0; k < KW; ++k) {
          const int c = lane + 32 * k;
          v[t][k] = c < q.W ? q.mult * q.src[c] : 0.f;
        }
      }
#pragma unroll
      for (int t = 0; t < BT; ++t) {
        const int j = j0 + t;
        const uint32_t key = kk[t];
        if (j >= cnt || key >= kKeyDrop) {
          done = true;
          break;
        }
#pragma unroll
        for (int k = 0; k < KW; ++k) acc[k] += v[t][k];
        if (j + 1 < cnt && kk[t + 1] == key) continue;
        // the segment [seg_start, j] ends here
        const bool head = seg_start == 0 && prev == key;
        const bool tail = j == cnt - 1 && next == key;
        const int W = key_width(key, H);
        float* out = head ? head_slot : tail_slot;
#pragma unroll
        for (int k = 0; k < KW; ++k) {
          const int c = lane + 32 * k;
          if (c < W) {
            if (head || tail) out[c] = acc[k];
            else *key_dest(G, A, key, c, H) = acc[k];
          }
          acc[k] = 0.f;
        }
        seg_start = j + 1;
      }
    }
  }
}

// Runs crossing block boundaries, one warp per block: the block holding a
// run's tail slot (the run began in it) finds the run's last block (32
// blocks probed per step) and adds the tail partial and the following
// blocks' head partials in block order.
template <int NC>
__global__ void __launch_bounds__(256) combine_kernel(Grads G, Act A, Sorted s, int H) {
  constexpr int KW = NC > 2 ? NC : 2;
  const int lane = threadIdx.x & 31;
  const uint32_t n0 = min(*s.n_live[0], s.n_max[0]), n1 = min(*s.n_live[1], s.n_max[1]);
  const uint32_t nb0 = (n0 + kSeg - 1) / kSeg, nb1 = (n1 + kSeg - 1) / kSeg;
  const uint32_t gw = (uint32_t)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const uint32_t n_warps = (uint32_t)((gridDim.x * blockDim.x) >> 5);
  for (uint32_t g = gw; g < nb0 + nb1; g += n_warps) {
    const int sg = g < nb0 ? 0 : 1;
    const uint32_t ob = sg ? g - nb0 : g, n_blocks = sg ? nb1 : nb0;
    const uint32_t* keys = s.keys[sg];
    const uint32_t sb = s.slot_base[sg];
    if (ob + 1 >= n_blocks) continue;  // a full block with a successor
    const uint32_t base = ob * kSeg;
    const uint32_t key = keys[base + kSeg - 1], kn = keys[base + kSeg], k0 = keys[base];
    const uint32_t kp = base > 0 ? keys[base - 1] : 0xffffffffu;
    if (key >= kKeyDrop || kn != key) continue;
    if (k0 == key && kp == key) continue;  // the run began in an earlier block
    // last block q of the run: the run continues into block q + 1 while that
    // block starts with the key
    uint32_t q = ob + 1;
    for (int round = 0; round < (1 << 20); ++round) {
      const uint32_t probe = q + 1 + (uint32_t)lane;
      const bool cont = probe < n_blocks && keys[probe * kSeg] == key;
      const uint32_t bal = __ballot_sync(kFull, cont);
      const int lead = bal == kFull ? 32 : __ffs(~bal) - 1;
      q += (uint32_t)lead;
      if (lead < 32) break;
    }
    const int W = sb + 2 * q + 1 < A.part_slots ? key_width(key, H) : 0;
    if (W == 0 && lane == 0) check_failed(A, 12, q, A.part_slots);
    float sum[KW];
#pragma unroll
    for (int k = 0; k < KW; ++k) {
      const int c = lane + 32 * k;
      sum[k] = c < W ? A.part[(size_t)(sb + 2 * ob + 1) * A.row_w + c] : 0.f;
    }
    uint32_t b = ob + 1;
    for (; b + 4 <= q + 1; b += 4) {
      float x[4][KW];
#pragma unroll
      for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int k = 0; k < KW; ++k) {
          const int c = lane + 32 * k;
          x[t][k] = c < W ? A.part[(size_t)(sb + 2 * (b + t)) * A.row_w + c] : 0.f;
        }
#pragma unroll
      for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int k = 0; k < KW; ++k) sum[k] += x[t][k];
    }
    for (; b <= q; ++b)
#pragma unroll
      for (int k = 0; k < KW; ++k) {
        const int c = lane + 32 * k;
        if (c < W) sum[k] += A.part[(size_t)(sb + 2 * b) * A.row_w + c];
      }
#pragma unroll
    for (int k = 0; k < KW; ++k) {
      const int c = lane + 32 * k;
      if (c < W) *key_dest(G, A, key, c, H) = sum[k];
    }
  }
}

// ---- dense weight gradients, feature-row gradient, metrics ----------------------------
// A reduction problem: out[o][c] = sum over k of A(k, o) X(k, c), k over the
// boards, then (optionally) over K2 further rows of a second pair.  Tiles of
// 16 x 64 outputs, the k range split kSplits ways; the split partials are
// added in split order by whichever block of the tile finishes last.
constexpr int kTO = 16, kTC = 64, kTK = 32, kSplits = 8, kMaxProb = 12;

struct RedProb {
  const float* a;  // A(k, o) = a[k * lda + o]; nullptr: A = 1
  int lda, O;
  const float* x;  // X(k, c) = x[k * ldx + c]; xpair: x is the threat accumulator, X = pair columns
  int ldx, C, xpair;
  const float* a2;  // rows k >= K of the second pair
  int lda2;
  const float* x2;
  int ldx2, K2;
  float* out;
  int tiles_c, tile0;
};
struct RedTable {
  RedProb p[kMaxProb];
  int n_prob, n_tiles, K;
  int tile_base;  // this table's first tile in the partial and counter arrays
};

__device__ __forceinline__ float pair_of(const float* ta, int c) {
  const float a = fminf(fmaxf(ta[c & (kTR - 1)], 0.f), 1.f);
  return c < kTR ? a : a * a;
}

__device__ void tile_block(const RedTable& T, Act& A, int tile, int split) {
  __shared__ float As[kTK][kTO];
  __shared__ float Xs[kTK][kTC];
  __shared__ bool last;
  int pi = 0;
  while (pi + 1 < T.n_prob && T.p[pi + 1].tile0 <= tile) ++pi;
  const RedProb& q = T.p[pi];
  const int t = tile - q.tile0, o0 = (t / q.tiles_c) * kTO, c0 = (t % q.tiles_c) * kTC;
  const int K = T.K + q.K2;
  const int chunk = (K + kSplits * kTK - 1) / (kSplits * kTK) * kTK;
  const int k_beg = split * chunk, k_end = min(K, k_beg + chunk);
  const int tid = threadIdx.x, to = tid / 16, tc = (tid % 16) * 4;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  // one chunk of kTK rows of A (16 columns) and X (64 columns) per step; the
  // next chunk's loads are issued into registers before this one's products
  constexpr int kAL = kTK * kTO / 256, kXL = kTK * kTC / 256;  // loads per thread: 2, 8
  float ra[kAL], rx[kXL];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int l = 0; l < kAL; ++l) {
      const int i = tid + 256 * l, kk = i / kTO, oo = i % kTO, k = k0 + kk, o = o0 + oo;
      float v = 0.f;
      if (k < k_end && o < q.O) {
        if (k < T.K) v = q.a ? q.a[(size_t)k * q.lda + o] : 1.f;
        else v = q.a2[(size_t)(k - T.K) * q.lda2 + o];
      }
      ra[l] = v;
    }
#pragma unroll
    for (int l = 0; l < kXL; ++l) {
      const int i = tid + 256 * l, kk = i / kTC, cc = i % kTC, k = k0 + kk, c = c0 + cc;
      float v = 0.f;
      if (k < k_end && c < q.C) {
        if (k < T.K) v = q.xpair ? pair_of(q.x + (size_t)k * kTR, c) : q.x[(size_t)k * q.ldx + c];
        else v = q.x2[(size_t)(k - T.K) * q.ldx2 + c];
      }
      rx[l] = v;
    }
  };
  if (k_beg < k_end) fetch(k_beg);
  for (int k0 = k_beg; k0 < k_end; k0 += kTK) {
#pragma unroll
    for (int l = 0; l < kAL; ++l) {
      const int i = tid + 256 * l;
      As[i / kTO][i % kTO] = ra[l];
    }
#pragma unroll
    for (int l = 0; l < kXL; ++l) {
      const int i = tid + 256 * l;
      Xs[i / kTC][i % kTC] = rx[l];
    }
    __syncthreads();
    if (k0 + kTK < k_end) fetch(k0 + kTK);
#pragma unroll 8
    for (int kk = 0; kk < kTK; ++kk) {
      const float a = As[kk][to];
#pragma unroll
      for (int v = 0; v < 4; ++v) acc[v] = fmaf(a, Xs[kk][tc + v], acc[v]);
    }
    __syncthreads();
  }
  const int gt = T.tile_base + tile;  // the tile's slot among all of the step's tiles
  float* part = A.tile_part + ((size_t)gt * kSplits + split) * (kTO * kTC) + tid * 4;
  *reinterpret_cast<float4*>(part) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(A.tile_cnt + gt, 1u) == kSplits - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  float sum[4] = {0.f, 0.f, 0.f, 0.f};
  for (int sp = 0; sp < kSplits; ++sp) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(A.tile_part + ((size_t)gt * kSplits + sp) * (kTO * kTC) +
                                                           tid * 4));
    sum[0] += v.x, sum[1] += v.y, sum[2] += v.z, sum[3] += v.w;
  }
  const int o = o0 + to;
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const int c = c0 + tc + v;
    if (o < q.O && c < q.C) q.out[(size_t)o * q.C + c] = sum[v];
  }
  if (tid == 0) A.tile_cnt[gt] = 0;  // ready for the next step
}

// The 30 metrics of compute_batch_loss (train_gpu_candle.rs:271-300), summed
// over the boards in a fixed order, then the status word's four bits as 0/1
// and the word itself: out[0..35).
__device__ void metrics_block(const Batch& bt, const Act& A, LossScale raw, const uint32_t* status, float* out) {
  constexpr int kN = 2 + 2 + 6 + 21;  // weighted CEs, CEs, per-sample sums, phase
  __shared__ float red[256][kN + 1];
  float s[kN];
#pragma unroll
  for (int i = 0; i < kN; ++i) s[i] = 0.f;
  for (int64_t b = threadIdx.x; b < bt.B; b += 256) {
    const float* r = A.rec + b * 8;
    const float v = r[4], t = bt.values[b], err = v - t;
    const float per[6] = {v, v * v, t, t * t, v * t, err * err};
    s[0] += r[0], s[1] += r[1], s[2] += r[2], s[3] += r[3];
#pragma unroll
    for (int k = 0; k < 6; ++k) s[4 + k] += per[k];
#pragma unroll
    for (int ph = 0; ph < 3; ++ph) {
      const float m = bt.phase[b * 3 + ph];
      s[10 + ph * 7] += m;
#pragma unroll
      for (int k = 0; k < 6; ++k) s[10 + ph * 7 + 1 + k] += m * per[k];
    }
  }
#pragma unroll
  for (int i = 0; i < kN; ++i) red[threadIdx.x][i] = s[i];
  __syncthreads();
  for (int w = 128; w >= 1; w >>= 1) {
    if ((int)threadIdx.x < w)
      for (int i = 0; i < kN; ++i) red[threadIdx.x][i] += red[threadIdx.x + w][i];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float* t = red[0];
    out[0] = t[0] * raw.value + t[1] * raw.policy;  // loss sum (not divided by the batch)
    out[1] = t[2];
    out[2] = t[3];
    for (int k = 0; k < 6; ++k) out[3 + k] = t[4 + k];
    for (int k = 0; k < 21; ++k) out[9 + k] = t[10 + k];
    const uint32_t word = *(volatile const uint32_t*)status;
    for (int k = 0; k < 4; ++k) out[30 + k] = (word >> k) & 1u ? 1.f : 0.f;
    out[34] = (float)word;
  }
}

// Blocks [0, n_tiles * kSplits): weight-gradient tiles; then (feature_rows)
// the feature-row gradient grad_trunk[r][c] += dpsp[r][c] (c < 32) + sum_j
// daf[r][j] W_acc[j][c] for r < 1260 (one thread per element) and the
// metrics block.  The tiles that need only the per-board backward run as one
// launch beside the table sums; the accumulator weights' tile (it also needs
// the feature rows' gradients), the feature rows and the metrics after them.
__global__ void __launch_bounds__(256) final_kernel(RedTable T, Params P, Grads G, Act A, Batch bt, int H,
                                                    LossScale raw, const uint32_t* status, float* metrics,
                                                    int feature_rows) {
  const int tile_blocks = T.n_tiles * kSplits;
  const int64_t feat_elems = (int64_t)kInput * H;
  const int feat_blocks = feature_rows ? (int)((feat_elems + 255) / 256) : 0;
  if ((int)blockIdx.x < tile_blocks) {
    tile_block(T, A, blockIdx.x / kSplits, blockIdx.x % kSplits);
    return;
  }
  const int fb = (int)blockIdx.x - tile_blocks;
  if (fb < feat_blocks) {
    const int64_t i = (int64_t)fb * 256 + threadIdx.x;
    if (i >= feat_elems) return;
    const int r = (int)(i / H), c = (int)(i % H);
    const float* d = A.pspaf + (size_t)r * kFeatW;
    float v = c < kPsp ? d[c] : 0.f;
#pragma unroll 8
    for (int j = 0; j < kAcc; ++j) v = fmaf(d[kPsp + j], __ldg(P.p[L_PAH] + (size_t)j * H + c), v);
    G.g[L_FT][i] += v;
    return;
  }
  metrics_block(bt, A, raw, status, metrics);
}

// ---- host -----------------------------------------------------------------------------
constexpr size_t kSmallCounters = 64;   // u32: counters[0] = kept row contributions
constexpr size_t kTileCounters = 256;   // u32: one per weight tile (<= 97 at H = 512)

int64_t leaf_size(int leaf, int64_t H) {
  switch (leaf) {
    case L_FT: return (int64_t)kTrunkRows * H;
    case L_RULE: return (int64_t)kRule * H;
    case L_HB: return H;
    case L_VHH: return (int64_t)kVH * H;
    case L_VHB: return kVH;
    case L_VHO: return 3 * kVH;
    case L_TE: return (int64_t)kVocab * kTR;
    case L_VTO: return 3 * kPair;
    case L_PTC: return 16 * kPair;
    case L_MB: return kMoves;
    case L_CONS: return kPsp;
    case L_PCH: return 16 * H;
    case L_MC: return (int64_t)kMoves * 16;
    case L_PAH: return (int64_t)kAcc * H;
    case L_AM: return (int64_t)kMoves * kAcc;
    case L_SPARSE: return kSparseLen;
    default: return kTactLen;
  }
}

struct Plan {
  size_t small, keys, sort, sort2, part, tile_part;
  size_t bp, hid, rms, vh, ta, ctx, vl, af, dl, mrow, frow, pay, dvl, dctx, cons, rec, dbp, dpre, dta, dvh;
  size_t small_bytes, total;
  int row_w, max_tiles;
};

int tiles_for(int64_t O, int64_t C) { return (int)(((O + kTO - 1) / kTO) * ((C + kTC - 1) / kTC)); }
int max_tiles(int64_t H) {
  return tiles_for(kRule, H) + tiles_for(1, H) + tiles_for(kVH, H) + tiles_for(1, kVH) + tiles_for(3, kVH) +
         tiles_for(3, kPair) + tiles_for(16, kPair) + tiles_for(16, H) + tiles_for(kAcc, H) + tiles_for(1, kPsp);
}

Plan make_plan(int64_t H, int64_t B, int64_t F, int64_t M, int64_t T) {
  Plan p{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += align_up(bytes, 256);
    return o;
  };
  const Bases cb = bases(B, F, M, T);
  const int64_t n = cb.n;
  p.row_w = (int)std::max<int64_t>(H, kTR);
  p.max_tiles = max_tiles(H);
  p.small_bytes = (kSmallCounters + kTileCounters) * 4 + (size_t)kInput * kFeatW * 4;
  p.small = take(p.small_bytes);
  p.keys = take((size_t)n * 4);
  const int64_t n_rows = cb.sparse, n_scalars = n - cb.sparse;  // the two sorts' slots
  p.sort = take(scat::sort_bytes(n_rows));
  p.sort2 = take(scat::sort_bytes(n_scalars));
  p.part = take((size_t)2 * ((n_rows + kSeg - 1) / kSeg + (n_scalars + kSeg - 1) / kSeg) * p.row_w * 4);
  p.tile_part = take((size_t)p.max_tiles * kSplits * kTO * kTC * 4);
  p.bp = take((size_t)B * H * 4);
  p.hid = take((size_t)B * H * 4);
  p.rms = take((size_t)B * 4);
  p.vh = take((size_t)B * kVH * 4);
  p.ta = take((size_t)B * kTR * 4);
  p.ctx = take((size_t)B * kCtx * 4);
  p.vl = take((size_t)B * 4 * 4);
  p.af = take((size_t)kInput * kAcc * 4);
  p.dl = take((size_t)B * M * 4);
  p.mrow = take((size_t)B * M * kRowStride * 4);
  p.frow = take((size_t)B * M * kRowStride * 4);
  p.pay = take((size_t)n * 4);
  p.dvl = take((size_t)B * 4 * 4);
  p.dctx = take((size_t)B * kCtx * 4);
  p.cons = take((size_t)B * kPsp * 4);
  p.rec = take((size_t)B * 8 * 4);
  p.dbp = take((size_t)B * H * 4);
  p.dpre = take((size_t)B * H * 4);
  p.dta = take((size_t)B * kTR * 4);
  p.dvh = take((size_t)B * kVH * 4);
  p.total = off;
  return p;
}

bool dims_ok(int64_t H, int64_t B, int64_t F, int64_t M, int64_t T) {
  if (!(H == 32 || H == 64 || H == 128 || H == 256 || H == 512)) return false;
  if (B < 1 || F < 1 || M < 1 || T < 1 || M > 1024 || F > 256) return false;
  const double n = (double)B * (6.0 * F + T + 13.0 * M);
  return n < 2147483647.0 && B < (1 << (32 - kMultBits));
}

void add_prob(RedTable& T, const float* a, int lda, int O, const float* x, int ldx, int C, int xpair, float* out,
              const float* a2 = nullptr, int lda2 = 0, const float* x2 = nullptr, int ldx2 = 0, int K2 = 0) {
  RedProb& q = T.p[T.n_prob++];
  q.a = a, q.lda = lda, q.O = O;
  q.x = x, q.ldx = ldx, q.C = C, q.xpair = xpair;
  q.a2 = a2, q.lda2 = lda2, q.x2 = x2, q.ldx2 = ldx2, q.K2 = K2;
  q.out = out;
  q.tiles_c = (C + kTC - 1) / kTC;
  q.tile0 = T.n_tiles;
  T.n_tiles += tiles_for(O, C);
}

// The step's streams and events (one stream, no events, without an engine).
struct Streams {
  cudaStream_t main, side, side2;
  cudaEvent_t join, join2, bwd, join3, comb, join4;
  bool forked;
};
// The optional AdamW of a single-GPU step: the table leaves' ranges (final
// after the table sums) and the dense leaves' (final after the last kernel).
struct Optim {
  float *params, *m, *v;
  const float* grads;
  cnnue_adamw_state* state;
  AdamWRanges table, dense;
};

template <int NC>
int launch_main(const Params& P, const Grads& G, Act& A, const Batch& bt, const Bases& cb, const Sorted& srt,
                LossScale ls, LossScale raw, uint32_t* status, float* metrics, const Streams& st,
                const Optim* opt) {
  constexpr int H = 32 * NC;
  const cudaStream_t s = st.main;
  const int board_blocks = (int)((bt.B + kWarps - 1) / kWarps);
  const int af_blocks = (kInput + kBW - 1) / kBW;
  fwd_kernel<NC><<<(unsigned)bt.B + af_blocks, 32 * kBW, (size_t)fwd_smem_words(bt.F, H) * 4, s>>>(
      P, bt, A, (int)bt.B, status);
  if (int e = check_launch_error("azt forward")) return e;
  policy_kernel<<<(unsigned)bt.B, 32 * kBW, (size_t)bt.M * 4, s>>>(P, bt, A, H, ls, status);
  if (int e = check_launch_error("azt policy")) return e;
  bwd_kernel<NC><<<board_blocks, 32 * kWarps, 0, s>>>(P, bt, A);
  if (int e = check_launch_error("azt backward")) return e;
  // dense weight gradients: all but the accumulator weights need only the
  // per-board backward, so they run beside the table sums
  RedTable Te{}, Tl{};
  Te.K = Tl.K = (int)bt.B;
  add_prob(Te, bt.rule, kRule, kRule, A.dpre, H, H, 0, G.g[L_RULE]);
  add_prob(Te, nullptr, 0, 1, A.dbp, H, H, 0, G.g[L_HB]);
  add_prob(Te, A.dvh, kVH, kVH, A.hid, H, H, 0, G.g[L_VHH]);
  add_prob(Te, nullptr, 0, 1, A.dvh, kVH, kVH, 0, G.g[L_VHB]);
  add_prob(Te, A.dvl, 4, 3, A.vh, kVH, kVH, 0, G.g[L_VHO]);
  add_prob(Te, A.dvl, 4, 3, A.ta, kTR, kPair, 1, G.g[L_VTO]);
  add_prob(Te, A.dctx, kCtx, 16, A.ta, kTR, kPair, 1, G.g[L_PTC]);
  add_prob(Te, A.dctx, kCtx, 16, A.hid, H, H, 0, G.g[L_PCH]);
  add_prob(Te, nullptr, 0, 1, A.cons, kPsp, kPsp, 0, G.g[L_CONS]);
  Tl.tile_base = Te.n_tiles;
  add_prob(Tl, A.dctx + 16, kCtx, kAcc, A.bp, H, H, 0, G.g[L_PAH], A.pspaf + kPsp, kFeatW, P.p[L_FT], H, kInput);
  const cudaStream_t early = st.forked ? st.side : s;
  if (st.forked) {
    CNNUE_CUDA_TRY(cudaEventRecord(st.bwd, s));
    CNNUE_CUDA_TRY(cudaStreamWaitEvent(st.side, st.bwd, 0));
  }
  final_kernel<<<Te.n_tiles * kSplits, 256, 0, early>>>(Te, P, G, A, bt, H, raw, status, metrics, 0);
  if (int e = check_launch_error("azt dense gradients")) return e;
  if (st.forked) {
    CNNUE_CUDA_TRY(cudaEventRecord(st.join3, st.side));
    CNNUE_CUDA_TRY(cudaStreamWaitEvent(s, st.join, 0));
    CNNUE_CUDA_TRY(cudaStreamWaitEvent(s, st.join2, 0));
  }
  const int64_t seg_blocks = ((int64_t)srt.n_max[0] + kSeg - 1) / kSeg + ((int64_t)srt.n_max[1] + kSeg - 1) / kSeg;
  const unsigned seg_grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((seg_blocks + 7) / 8, 148 * 32));
  seg_kernel<NC><<<seg_grid, 256, 0, s>>>(G, A, bt, srt, H);
  if (int e = check_launch_error("azt segment sums")) return e;
  combine_kernel<NC><<<seg_grid, 256, 0, s>>>(G, A, srt, H);
  if (int e = check_launch_error("azt run combine")) return e;
  if (opt) {
    // the table leaves' gradients are final: their AdamW runs beside the rest
    if (int e = adamw_prepare(opt->state, s)) return e;
    const cudaStream_t tab = st.forked ? st.side2 : s;
    if (st.forked) {
      CNNUE_CUDA_TRY(cudaEventRecord(st.comb, s));
      CNNUE_CUDA_TRY(cudaStreamWaitEvent(st.side2, st.comb, 0));
    }
    if (int e = adamw_ranges(opt->params, opt->m, opt->v, opt->grads, opt->table, opt->state, tab)) return e;
    if (st.forked) CNNUE_CUDA_TRY(cudaEventRecord(st.join4, st.side2));
  }
  const int feat_blocks = (int)(((int64_t)kInput * H + 255) / 256);
  final_kernel<<<Tl.n_tiles * kSplits + feat_blocks + 1, 256, 0, s>>>(Tl, P, G, A, bt, H, raw, status, metrics, 1);
  if (int e = check_launch_error("azt final")) return e;
  if (st.forked) CNNUE_CUDA_TRY(cudaStreamWaitEvent(s, st.join3, 0));
  if (opt) {
    if (int e = adamw_ranges(opt->params, opt->m, opt->v, opt->grads, opt->dense, opt->state, s)) return e;
    if (st.forked) CNNUE_CUDA_TRY(cudaStreamWaitEvent(s, st.join4, 0));
  }
  return CNNUE_OK;
}

}  // namespace
}  // namespace azt
}  // namespace cnnue

struct cnnue_azt {
  int device;
  cudaStream_t side, side2;  // the row-key sort then the early dense gradients; the scalar-key sort then AdamW
  cudaEvent_t fork, keys, join, join2, bwd, join3, comb, join4;
};

using namespace cnnue;
using namespace cnnue::azt;

extern "C" {

int cnnue_azt_create(int device, cnnue_azt** out) {
  if (!out) return set_error(CNNUE_ERR_INVALID_ARG, "cnnue_azt_create: out is NULL");
  *out = nullptr;
  if (int st = use_device(device)) return st;
  cnnue_azt* e = new cnnue_azt{};
  e->device = device;
  cudaError_t err = cudaStreamCreateWithFlags(&e->side, cudaStreamNonBlocking);
  if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&e->side2, cudaStreamNonBlocking);
  for (cudaEvent_t* ev : {&e->fork, &e->keys, &e->join, &e->join2, &e->bwd, &e->join3, &e->comb, &e->join4})
    if (err == cudaSuccess) err = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
  if (err != cudaSuccess) {
    for (cudaEvent_t ev : {e->fork, e->keys, e->join, e->join2, e->bwd, e->join3, e->comb, e->join4})
      if (ev) cudaEventDestroy(ev);
    if (e->side2) cudaStreamDestroy(e->side2);
    if (e->side) cudaStreamDestroy(e->side);
    delete e;
    return cuda_error(err, "cnnue_azt_create");
  }
  *out = e;
  return CNNUE_OK;
}

int cnnue_azt_destroy(cnnue_azt* e) {
  if (!e) return CNNUE_OK;
  use_device(e->device);
  cudaStreamSynchronize(e->side);
  cudaStreamSynchronize(e->side2);
  for (cudaEvent_t ev : {e->fork, e->keys, e->join, e->join2, e->bwd, e->join3, e->comb, e->join4})
    cudaEventDestroy(ev);
  cudaStreamDestroy(e->side2);
  cudaStreamDestroy(e->side);
  delete e;
  return CNNUE_OK;
}

size_t cnnue_azt_workspace_bytes(int64_t hidden, int64_t batch, int64_t features, int64_t moves, int64_t threats) {
  if (!dims_ok(hidden, batch, features, moves, threats)) return 0;
  return make_plan(hidden, batch, features, moves, threats).total;
}

int cnnue_azt_step(cnnue_azt* e, const float* d_params, float* d_grads, int64_t n_grads, const int64_t* leaf_offsets,
                   int64_t hidden, const cnnue_azt_batch* batch, float value_weight, float policy_weight,
                   float* d_metrics, uint32_t* d_status, void* d_ws, size_t ws_bytes, const cnnue_azt_optim* optim,
                   void* stream) {
  if (!d_params || !d_grads || !leaf_offsets || !batch || !d_metrics || !d_status || !d_ws)
    return set_error(CNNUE_ERR_INVALID_ARG, "cnnue_azt_step: NULL argument");
  const cnnue_azt_batch& b = *batch;
  if (!dims_ok(hidden, b.batch, b.features, b.moves, b.threats))
    return set_error(CNNUE_ERR_INVALID_ARG,
                     "cnnue_azt_step: hidden must be 32, 64, 128, 256 or 512, dims >= 1, moves <= 1024, "
                     "features <= 256 "
                     "(hidden %lld, batch %lld, features %lld, moves %lld, threats %lld)",
                     (long long)hidden, (long long)b.batch, (long long)b.features, (long long)b.moves,
                     (long long)b.threats);
  if (!b.feature_items || !b.value_threat_indices || !b.policy_items || !b.policy_sparse_indices ||
      !b.policy_tactical_indices || !b.policy_targets || !b.policy_mask || !b.value_wdl || !b.values ||
      !b.rule_context || !b.policy_weights || !b.value_weights || !b.value_phase_masks)
    return set_error(CNNUE_ERR_INVALID_ARG, "cnnue_azt_step: every batch array is needed (expand compact batches)");
  if (((uintptr_t)d_params | (uintptr_t)d_grads) & 15)
    return set_error(CNNUE_ERR_INVALID_ARG, "cnnue_azt_step: parameters and gradients must be 16-byte aligned");
  for (int l = 0; l < kLeaves; ++l) {
    if (leaf_offsets[l] < 0 || (leaf_offsets[l] & 3) || leaf_offsets[l] + leaf_size(l, hidden) > n_grads)
      return set_error(CNNUE_ERR_INVALID_ARG, "cnnue_azt_step: leaf %d offset %lld (size %lld) outside the %lld "
                       "gradients or not a multiple of 4", l, (long long)leaf_offsets[l],
                       (long long)leaf_size(l, hidden), (long long)n_grads);
  }
  const Plan pl = make_plan(hidden, b.batch, b.features, b.moves, b.threats);
  if ((uintptr_t)d_ws & 255) return set_error(CNNUE_ERR_INVALID_ARG, "cnnue_azt_step: workspace not 256-byte aligned");
  if (ws_bytes < pl.total)
    return set_error(CNNUE_ERR_WORKSPACE, "cnnue_azt_step: workspace %zu bytes, need %zu", ws_bytes, pl.total);
  if (e) {
    if (int st = use_device(e->device)) return st;
  }
  cudaStream_t s = (cudaStream_t)stream;
  cudaStream_t side = e ? e->side : s;

  Params P;
  Grads G;
  for (int l = 0; l < kLeaves; ++l) {
    P.p[l] = d_params + leaf_offsets[l];
    G.g[l] = d_grads + leaf_offsets[l];
  }
  Batch bt{b.batch, b.features, b.moves, b.threats, b.feature_items, b.value_threat_indices, b.policy_items,
           b.policy_sparse_indices, b.policy_tactical_indices, b.policy_targets, b.policy_mask, b.value_wdl,
           b.values, b.rule_context, b.policy_weights, b.value_weights, b.value_phase_masks};
  char* w = (char*)d_ws;
  Act A{};
  A.counters = (uint32_t*)(w + pl.small);
  A.tile_cnt = A.counters + kSmallCounters;
  A.pspaf = (float*)(A.tile_cnt + kTileCounters);
  A.keys = (uint32_t*)(w + pl.keys);
  A.part = (float*)(w + pl.part);
  A.tile_part = (float*)(w + pl.tile_part);
  A.bp = (float*)(w + pl.bp), A.hid = (float*)(w + pl.hid), A.rms = (float*)(w + pl.rms);
  A.vh = (float*)(w + pl.vh), A.ta = (float*)(w + pl.ta), A.ctx = (float*)(w + pl.ctx);
  A.vl = (float*)(w + pl.vl), A.af = (float*)(w + pl.af), A.dl = (float*)(w + pl.dl);
  A.mrow = (float*)(w + pl.mrow), A.frow = (float*)(w + pl.frow), A.pay = (uint32_t*)(w + pl.pay);
  A.dvl = (float*)(w + pl.dvl), A.dctx = (float*)(w + pl.dctx), A.cons = (float*)(w + pl.cons);
  A.rec = (float*)(w + pl.rec), A.dbp = (float*)(w + pl.dbp), A.dpre = (float*)(w + pl.dpre);
  A.dta = (float*)(w + pl.dta), A.dvh = (float*)(w + pl.dvh);
  A.row_w = pl.row_w;
  A.status = d_status;
  const Bases cb = bases(b.batch, b.features, b.moves, b.threats);
  A.part_slots = (uint32_t)(2 * (((int64_t)cb.sparse + kSeg - 1) / kSeg + ((int64_t)cb.n - cb.sparse + kSeg - 1) / kSeg));
  const LossScale raw{std::max(value_weight, 0.f), std::max(policy_weight, 0.f)};
  const LossScale ls{raw.value / (float)b.batch, raw.policy / (float)b.batch};

  CNNUE_CUDA_TRY(cudaMemsetAsync(d_grads, 0, (size_t)n_grads * 4, s));
  CNNUE_CUDA_TRY(cudaMemsetAsync(w + pl.small, 0, pl.small_bytes, s));
  CNNUE_CUDA_TRY(cudaMemsetAsync(d_status, 0, 4, s));
  if (side != s) {
    CNNUE_CUDA_TRY(cudaEventRecord(e->fork, s));
    CNNUE_CUDA_TRY(cudaStreamWaitEvent(side, e->fork, 0));
  }
  // side: keys of every table contribution, one joint sort
  const int pool_blocks = (int)((b.batch + kWarps - 1) / kWarps);
  const int64_t slots = (int64_t)cb.n - cb.threat;  // threat and move slots: one thread each
  const int other_blocks = (int)std::max<int64_t>(1, std::min<int64_t>((slots + 255) / 256, 148 * 8));
  keygen_kernel<<<pool_blocks + other_blocks, 256, 0, side>>>(bt, cb, A.keys, A.pay, A.counters, d_status,
                                                             pool_blocks);
  if (int st = check_launch_error("azt keys")) return st;
  // the row keys (2 passes, 16 bits) on the side stream, the scalar-table
  // keys (3 passes) on the second one, both after the keys
  cudaStream_t side2 = e ? e->side2 : s;
  if (side != s) {
    CNNUE_CUDA_TRY(cudaEventRecord(e->keys, side));
    CNNUE_CUDA_TRY(cudaStreamWaitEvent(side2, e->keys, 0));
  }
  Sorted srt{};
  srt.n_live[0] = A.counters;
  srt.n_live[1] = A.counters + 1;
  srt.n_max[0] = cb.sparse;
  srt.n_max[1] = cb.n - cb.sparse;
  srt.slot_base[0] = 0;
  srt.slot_base[1] = (uint32_t)(2 * ((cb.sparse + kSeg - 1) / kSeg));
  if (int st = scat::radix_sort(A.keys, cb.sparse, kKeyRowsEnd, w + pl.sort, side, &srt.keys[0], &srt.pay[0],
                                A.counters, kKeyDrop, A.pay))
    return st;
  if (int st = scat::radix_sort(A.keys + cb.sparse, (int64_t)cb.n - cb.sparse, kKeyDrop, w + pl.sort2, side2,
                                &srt.keys[1], &srt.pay[1], A.counters + 1, kKeyDrop, A.pay + cb.sparse))
    return st;
  if (side != s) {
    CNNUE_CUDA_TRY(cudaEventRecord(e->join, side));
    CNNUE_CUDA_TRY(cudaEventRecord(e->join2, side2));
  }
  Streams streams{s, side, side2, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, side != s};
  if (e) {
    streams.join = e->join, streams.join2 = e->join2, streams.bwd = e->bwd;
    streams.join3 = e->join3, streams.comb = e->comb, streams.join4 = e->join4;
  }
  Optim opt{};
  if (optim) {
    if (!optim->params || !optim->m || !optim->v || !optim->state || optim->params != d_params)
      return set_error(CNNUE_ERR_INVALID_ARG, "cnnue_azt_step: optim needs params (= d_params), m, v and state");
    for (int l = 0; l + 1 < kLeaves; ++l)
      if (leaf_offsets[l + 1] < leaf_offsets[l] + leaf_size(l, hidden))
        return set_error(CNNUE_ERR_INVALID_ARG, "cnnue_azt_step: the optimizer needs the leaves in order");
    opt.params = optim->params, opt.m = optim->m, opt.v = optim->v, opt.state = optim->state;
    opt.grads = d_grads;
    const int64_t* o = leaf_offsets;
    auto add = [](AdamWRanges& r, int64_t b, int64_t e) {
      r.begin[r.n] = b;
      r.len4[r.n] = (e - b + 3) / 4;  // into the leaf's padding (zeros: AdamW keeps them)
      ++r.n;
    };
    // table leaves (final after the table sums) and the dense ones; the
    // tactical table's constant zero (its last element) is not a parameter
    add(opt.table, o[L_TE], o[L_VTO]);
    add(opt.table, o[L_MB], o[L_CONS]);
    add(opt.table, o[L_MC], o[L_PAH]);
    add(opt.table, o[L_AM], o[L_TACT] + kTactLen - 1);
    add(opt.dense, 0, o[L_TE]);
    add(opt.dense, o[L_VTO], o[L_MB]);
    add(opt.dense, o[L_CONS], o[L_MC]);
    add(opt.dense, o[L_PAH], o[L_AM]);
    if (o[L_FT] != 0 || ((o[L_TACT] + kTactLen - 1) & 3))
      return set_error(CNNUE_ERR_INVALID_ARG, "cnnue_azt_step: the optimizer needs the trunk table first and the "
                       "tactical table ending on a 4-element boundary");
  }
  const Optim* op = optim ? &opt : nullptr;
  switch (hidden) {
    case 32: return launch_main<1>(P, G, A, bt, cb, srt, ls, raw, d_status, d_metrics, streams, op);
    case 64: return launch_main<2>(P, G, A, bt, cb, srt, ls, raw, d_status, d_metrics, streams, op);
    case 128: return launch_main<4>(P, G, A, bt, cb, srt, ls, raw, d_status, d_metrics, streams, op);
    case 256: return launch_main<8>(P, G, A, bt, cb, srt, ls, raw, d_status, d_metrics, streams, op);
    default: return launch_main<16>(P, G, A, bt, cb, srt, ls, raw, d_status, d_metrics, streams, op);
  }
}

}  // extern "C"
