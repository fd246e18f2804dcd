/*
 * cnnue.h - C ABI of the B200 (sm_100a) NNUE evaluation library.
 *
 * Every entry point returns an int status (CNNUE_OK == 0).  Nothing aborts.
 * Device buffers are caller-owned device pointers; `stream` is a cudaStream_t
 * passed as void* (NULL = the legacy default stream).  Entry points that take
 * device buffers only enqueue work: kernel-side faults in the data (an index
 * out of range, non-monotone offsets) are recorded in a status word inside the
 * caller's workspace and reported by cnnue_read_status().  Entry points that
 * take host buffers synchronise the stream and return that status directly.
 *
 * The reference (mycve/chineseai, Rust) has no FFI.  Each function below names
 * the reference function or Candle custom op it replaces (path:line within the
 * reference project).  The quantised HalfKA evaluator (cnnue_q_*) and the fp32
 * HalfKA evaluator (cnnue_f32_*) implement the workload specification the
 * reference's evaluator API is measured on; their reference anchors are the
 * evaluator entry points whose role they take.
 */
#ifndef CNNUE_H
#define CNNUE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
enum {
  CNNUE_OK = 0,
  CNNUE_ERR_INVALID_ARG = 1,  /* null pointer, negative size, bad enum       */
  CNNUE_ERR_BAD_INDEX = 2,    /* a feature index >= the feature count        */
  CNNUE_ERR_BAD_OFFSETS = 3,  /* offsets not monotone or beyond the indices  */
  CNNUE_ERR_CUDA = 4,         /* a CUDA runtime call failed                  */
  CNNUE_ERR_WORKSPACE = 5,    /* workspace smaller than cnnue_*_workspace_bytes */
  CNNUE_ERR_FORMAT = 6,       /* weight file: wrong format tag or tensor size */
  CNNUE_ERR_IO = 7,           /* weight file cannot be read or written       */
  CNNUE_ERR_NO_DEVICE = 8,    /* no CUDA device / wrong device ordinal       */
  CNNUE_ERR_TIMEOUT = 9,      /* a bounded device-side wait gave up          */
  CNNUE_ERR_INTERNAL = 10     /* a kernel self-check failed                  */
};

/* Status bits written by kernels into the workspace status word. */
#define CNNUE_STATUS_BAD_INDEX 0x1u
#define CNNUE_STATUS_BAD_OFFSETS 0x2u
#define CNNUE_STATUS_TIMEOUT 0x4u     /* a bounded device-side wait gave up */
#define CNNUE_STATUS_INTERNAL 0x8u    /* a kernel self-check failed (access skipped) */

const char* cnnue_status_string(int status);
/* Detail of the last error raised on the calling thread ("" if none). */
const char* cnnue_last_error(void);
/* Library version, e.g. "0.1.0". */
const char* cnnue_version(void);

/* ---- dimensions of the quantised HalfKA network ------------------------ */
#define CNNUE_Q_FEATURES 11340   /* 9 king squares x 14 piece kinds x 90 squares */
#define CNNUE_Q_COLS 1024        /* int16 FT columns per perspective            */
#define CNNUE_Q_HALF 512         /* pairwise pack: column j pairs with j + 512  */
#define CNNUE_Q_PACKED 1024      /* 2 perspectives x 512 uint8                  */
#define CNNUE_Q_BUCKETS 16
#define CNNUE_Q_L1 16
#define CNNUE_Q_L2 32

/* Host-side weights of the quantised network (all row-major, contiguous).
 *   ft_weight [11340][1024] int16     ft_bias  [1024] int16
 *   l1_weight [16][16][1024] int8     l1_bias  [16][16] int32
 *   l2_weight [16][32][16] int8       l2_bias  [16][32] int32
 *   l3_weight [16][32] int8           l3_bias  [16] int32
 * One FT table serves both perspectives. */
typedef struct cnnue_q_weights {
  const int16_t* ft_weight;
  const int16_t* ft_bias;
  const int8_t* l1_weight;
  const int32_t* l1_bias;
  const int8_t* l2_weight;
  const int32_t* l2_bias;
  const int8_t* l3_weight;
  const int32_t* l3_bias;
} cnnue_q_weights;

typedef struct cnnue_q_model cnnue_q_model;

/* Uploads the weights to `device` and returns a model handle.
 * Replaces AzNnue::load / AzNnue::random as the evaluator constructor
 * (src/az.rs:1433-1529): the model owns its device copy of the weights and is
 * shared read-only by every caller thread. */
int cnnue_q_model_create(const cnnue_q_weights* weights, int device, cnnue_q_model** out);
int cnnue_q_model_destroy(cnnue_q_model* model);

/* Bytes of device workspace cnnue_q_forward / cnnue_q_update need for
 * `n_positions` positions: the status word, the bucket sort and the packed
 * activations (1 KB per position).  Workspaces are 256-byte aligned
 * (cudaMalloc'd memory is). */
size_t cnnue_q_workspace_bytes(int64_t n_positions);

/* Reads and clears the status word of a workspace after the work queued on
 * `stream` has finished (synchronises `stream`).  *status_out receives a
 * CNNUE_ERR_* code (CNNUE_OK when the kernels saw valid data). */
int cnnue_read_status(void* d_workspace, void* stream, int* status_out);

/* Full quantised forward of a batch: for every position and perspective the
 * FT gather-accumulate (int16 wraparound), the pairwise clipped-ReLU pack to
 * uint8, the bucket selection by the perspective-0 active count and the int8
 * bucket stack 1024->16->32->1.  Replaces the evaluator entry point
 * AzNnue::evaluate_with_scratch_output (src/az.rs:1562-1604) and its FT gather
 * input_embedding_linear_into_slice (src/az.rs:2049-2076).
 *   d_indices  [n_indices] uint16 feature indices (< 11340)
 *   d_offsets  [2*n_positions+1] uint32; perspective s of position p owns
 *              d_indices[d_offsets[2p+s] .. d_offsets[2p+s+1])
 *   d_scores   [n_positions] int32 output
 * Two stages, also callable separately: cnnue_q_bucket_sort (groups positions
 * by bucket into the workspace) and cnnue_q_forward_sorted (over the sorted
 * order: the gather + pack kernel, which writes every position's 1024 packed
 * bytes into the workspace, then the bucket-stack kernel). */
int cnnue_q_forward(const cnnue_q_model* model, const uint16_t* d_indices, uint32_t n_indices,
                    const uint32_t* d_offsets, int64_t n_positions, int32_t* d_scores,
                    void* d_workspace, size_t workspace_bytes, void* stream);
int cnnue_q_bucket_sort(const cnnue_q_model* model, const uint32_t* d_offsets, uint32_t n_indices,
                        int64_t n_positions, void* d_workspace, size_t workspace_bytes,
                        void* stream);
int cnnue_q_forward_sorted(const cnnue_q_model* model, const uint16_t* d_indices,
                           uint32_t n_indices, const uint32_t* d_offsets, int64_t n_positions,
                           int32_t* d_scores, void* d_workspace, size_t workspace_bytes,
                           void* stream);

/* Test hook of the bounded device-side waits (no counterpart in the
 * reference, whose only failure handling is the search's stop flag,
 * src/main.rs:2106-2114).  Runs cnnue_q_forward with every wait of the
 * evaluation kernel limited to wait_limit_ns (0 < limit <= 1 s) and with CTA
 * `stall_block` never announcing or copying its pipeline stage
 * `stall_stage`, so the consumers' wait on that stage runs out: the kernel
 * sets CNNUE_STATUS_TIMEOUT, stops issuing, lets the copies already in flight
 * land and ends.  The scores are then undefined; cnnue_read_status reports
 * CNNUE_ERR_TIMEOUT and clears the word, and the model stays usable.  A
 * stall_block past the grid or a stall_stage past the CTA's stages runs the
 * plain forward. */
int cnnue_q_forward_stall_test(const cnnue_q_model* model, const uint16_t* d_indices,
                               uint32_t n_indices, const uint32_t* d_offsets, int64_t n_positions,
                               int32_t* d_scores, void* d_workspace, size_t workspace_bytes,
                               uint32_t stall_block, uint32_t stall_stage, uint64_t wait_limit_ns,
                               void* stream);

/* Same as cnnue_q_forward with HOST buffers: copies the inputs to the device,
 * runs the forward and copies the scores back, then synchronises `stream`
 * and returns the kernels' status.  The model keeps device staging buffers
 * that grow to the largest batch seen (not thread-safe per model). */
int cnnue_q_forward_host(cnnue_q_model* model, const uint16_t* h_indices, uint32_t n_indices,
                         const uint32_t* h_offsets, int64_t n_positions, int32_t* h_scores,
                         void* stream);

/* Pipelined host-buffer evaluation.  Replaces, for batched callers, the
 * per-thread evaluation loop over AzNnue::evaluate_with_scratch_output
 * (src/az.rs:1562-1604) with its per-thread AzEvalScratch (src/az.rs:309-367):
 * the context is the per-thread scratch, the model stays shared read-only.
 *
 * A context holds two slots, each with its own CUDA stream and device staging
 * for batches of up to max_positions positions and max_indices indices;
 * cnnue_q_ctx_create allocates them, the calls allocate nothing.  Call k runs
 * on slot k % 2: it enqueues the host-to-device copies of its indices and
 * offsets, the bucket sort, the forward and the device-to-host copy of the
 * scores, and returns at once with a ticket, so batch k + 1's copies overlap
 * batch k's kernels.  cnnue_q_ctx_wait(ticket) blocks until that batch's
 * scores are in h_scores and returns its kernels' status in *status.  At most
 * two calls may be in flight: a third call before the oldest is waited for
 * returns CNNUE_ERR_INVALID_ARG.  The host buffers of a call must stay
 * untouched until its wait returns; page-locked (pinned) buffers make the
 * copies asynchronous, pageable ones still work but serialise the copies.
 * One context per thread; several contexts may share a model.
 * cnnue_q_ctx_next_stream gives the stream the next call will use (to order
 * other work, e.g. a cache flush, before it). */
typedef struct cnnue_q_stream_ctx cnnue_q_stream_ctx;
int cnnue_q_ctx_create(const cnnue_q_model* model, int64_t max_positions, uint32_t max_indices,
                       cnnue_q_stream_ctx** out);
int cnnue_q_ctx_destroy(cnnue_q_stream_ctx* ctx);
int cnnue_q_ctx_next_stream(const cnnue_q_stream_ctx* ctx, void** stream);
int cnnue_q_forward_host_async(cnnue_q_stream_ctx* ctx, const uint16_t* h_indices, uint32_t n_indices,
                               const uint32_t* h_offsets, int64_t n_positions, int32_t* h_scores,
                               uint64_t* ticket);
int cnnue_q_ctx_wait(cnnue_q_stream_ctx* ctx, uint64_t ticket, int* status);

/* No-allocation variant of cnnue_q_forward (no counterpart in the reference).
 *
 * For callers that cannot allocate device memory at evaluation time: a search
 * thread that must not stall on cudaMalloc (which can synchronise the whole
 * device), or a host process that hands all of its device memory to its own
 * pool at start-up and has nothing left to give a workspace.  Such a caller
 * passes only its inputs and outputs; the bucket-sort scratch lives in a
 * fixed array inside the library (CNNUE_Q_NOALLOC_SCRATCH_BYTES, about 417 KB,
 * held on every GPU that loads the library until the process exits).
 *
 *   - n_positions may be at most CNNUE_Q_NOALLOC_MAX_POSITIONS; larger batches
 *     are rejected with CNNUE_ERR_INVALID_ARG (split them, or use
 *     cnnue_q_forward with a workspace).
 *   - The first call on a device looks up the scratch array's device address
 *     (once per device, with that device current).  The address is kept for
 *     the life of the process: after cudaDeviceReset on that device the
 *     entry point must not be called again.
 *   - The call synchronises its stream to read the kernels' status, so it
 *     cannot be captured into a CUDA graph (use cnnue_q_forward with a
 *     workspace inside a capture).
 *   - Every call on a device shares the one scratch array, which keeps the
 *     previous call's contents; each call clears the part that must start at
 *     zero.  Calls whose GPU work overlaps (other threads, other streams)
 *     race on the scratch: serialise them.
 *   - The call waits for its stream and returns the kernels' status
 *     (CNNUE_ERR_BAD_INDEX / CNNUE_ERR_BAD_OFFSETS on bad data).
 *   - It calls no cudaMalloc, cudaFree or other allocating routine. */
#define CNNUE_Q_NOALLOC_MAX_POSITIONS 65536
#define CNNUE_Q_NOALLOC_SCRATCH_BYTES (512 + 65536 + 4 * 65536 + 65536 + 256 * 32 * 4)
int cnnue_q_forward_noalloc(const cnnue_q_model* model, const uint16_t* d_indices,
                            uint32_t n_indices, const uint32_t* d_offsets, int64_t n_positions,
                            int32_t* d_scores, void* stream);

/* Optional: also write the int16 accumulators [n_positions][2][1024] of the
 * forward (d_acc may be NULL).  Used to check the gather separately. */
int cnnue_q_forward_acc(const cnnue_q_model* model, const uint16_t* d_indices, uint32_t n_indices,
                        const uint32_t* d_offsets, int64_t n_positions, int32_t* d_scores,
                        int16_t* d_acc, void* d_workspace, size_t workspace_bytes, void* stream);

/* Incremental accumulator update followed by the same pack + bucket stack.
 * Replaces AzEvalAccumulator::apply_transition_for_perspective
 * (src/az.rs:439-485) for the quantised network: per perspective either
 * child = parent - sum(removed rows) + sum(added rows), or, when the
 * perspective's refresh flag is set (a king move), child = bias + sum(added
 * rows) with `added` holding the full active list.
 *   d_parent       [n][2][1024] int16      d_child [n][2][1024] int16 (out)
 *   d_flags        [2n] uint8, bit 0 = refresh perspective (p, s) at 2p+s
 *   d_rem_offsets  [2n+1] uint32 into d_rem (uint16)
 *   d_add_offsets  [2n+1] uint32 into d_add (uint16)
 *   d_count0       [n] uint8: the child's perspective-0 active count (bucket)
 *   d_scores       [n] int32 (out) */
int cnnue_q_update(const cnnue_q_model* model, const int16_t* d_parent, const uint8_t* d_flags,
                   const uint16_t* d_rem, uint32_t n_rem, const uint32_t* d_rem_offsets,
                   const uint16_t* d_add, uint32_t n_add, const uint32_t* d_add_offsets,
                   const uint8_t* d_count0, int64_t n_positions, int16_t* d_child,
                   int32_t* d_scores, void* d_workspace, size_t workspace_bytes, void* stream);

/* ---- fp32 HalfKA network ------------------------------------------------ */
#define CNNUE_F_FEATURES 11340
#define CNNUE_F_COLS 256         /* fp32 FT columns per perspective */
#define CNNUE_F_BUCKETS 8
/* ft_weight [11340][256], ft_bias [256], l1_weight [8][16][512], l1_bias [8][16],
 * l2_weight [8][32][16], l2_bias [8][32], l3_weight [8][32], l3_bias [8]. */
typedef struct cnnue_f_weights {
  const float* ft_weight;
  const float* ft_bias;
  const float* l1_weight;
  const float* l1_bias;
  const float* l2_weight;
  const float* l2_bias;
  const float* l3_weight;
  const float* l3_bias;
} cnnue_f_weights;

typedef struct cnnue_f_model cnnue_f_model;
int cnnue_f_model_create(const cnnue_f_weights* weights, int device, cnnue_f_model** out);
int cnnue_f_model_destroy(cnnue_f_model* model);
/* Workspace of cnnue_f_forward for n positions: the 512-byte header (status
 * word and the kernel's counters, cleared by each call), the clipped FT
 * outputs [n][512] fp32 and the per-bucket position lists [8][n]. */
size_t cnnue_f_workspace_bytes(int64_t n_positions);
/* fp32 forward: FT sum (bias + rows in index order), clipped ReLU [0,1] on the
 * concatenated 512, bucket = (n0-1)/4 (8 buckets), stack 512->16->32->1 with
 * clipped ReLU between layers.  Same index/offset layout as cnnue_q_forward.
 * Replaces the fp32 evaluator path input_embedding_linear_into_slice +
 * value head (src/az.rs:2049-2076, src/az.rs:2133-2157). */
int cnnue_f_forward(const cnnue_f_model* model, const uint16_t* d_indices, uint32_t n_indices,
                    const uint32_t* d_offsets, int64_t n_positions, float* d_out,
                    void* d_workspace, size_t workspace_bytes, void* stream);

/* ---- reference-native feature pool (AZ-NNUE trunk FT) ------------------- */
#define CNNUE_POOL_ROWS 1545     /* 1260 piece-square + 14 piece + 10 rank + 9 file + 252 king-piece */
#define CNNUE_POOL_PADDING 0xffffffffu

/* out[b][h] = sum over the non-padding items of row b of the six table rows of
 * the item (feature, 1260+piece, 1274+rank, 1284+file, 1293+us*14+piece,
 * 1293+(9+them)*14+piece), summed from 0 in item order, rows in that order.
 * Item = feature | us_bucket << 11 | them_bucket << 15, 0xffffffff = padding.
 * An item with a row past the table is skipped and CNNUE_STATUS_BAD_INDEX is
 * ORed into *d_status (a device word the caller zeroes and reads).
 * Replaces the Candle op feature_pool / kernel feature_pool_fwd
 * (src/az/fused_feature_pool.rs:22-49, :134-148, CPU twin :169-198). */
int cnnue_feature_pool_fwd(const float* d_tables, const uint32_t* d_items, int64_t batch,
                           int64_t item_count, int64_t hidden, float* d_out, uint32_t* d_status,
                           void* stream);

/* grad_tables[r][h] = sum of grad_out[b][h] over every (b, item, slot) whose
 * slot row is r, without atomics: a stable radix sort of the contributions by
 * row, then per-row sums in that order (rows with at most 256 contributions
 * are summed in exactly the reference CPU order; longer rows in
 * 256-contribution units combined in order).  Deterministic run to run, no
 * host synchronisation.  Every row of grad_tables is written.  The
 * workspace's first word is the status word (read it with cnnue_read_status).
 * Replaces FeaturePoolGrad / kernel feature_pool_grad
 * (src/az/fused_feature_pool.rs:51-76, :214-223, CPU twin :231-260). */
size_t cnnue_feature_pool_bwd_workspace_bytes(int64_t batch, int64_t item_count, int64_t hidden);
int cnnue_feature_pool_bwd(const uint32_t* d_items, const float* d_grad_out, int64_t batch,
                           int64_t item_count, int64_t hidden, float* d_grad_tables,
                           void* d_workspace, size_t workspace_bytes, void* stream);

/* Plain table pool: out[b][h] = sum of table[item][h] over the non-padding
 * items of row b, in item order (rows >= `rows` are skipped and flagged).
 * Replaces SparsePool / kernel sparse_pool_fwd
 * (src/az/fused_feature_pool.rs:78-92, CPU twin :284-309). */
int cnnue_sparse_pool_fwd(const float* d_table, int64_t rows, const uint32_t* d_items,
                          int64_t batch, int64_t item_count, int64_t hidden, float* d_out,
                          uint32_t* d_status, void* stream);
/* Atomic-free backward of the plain pool (same scheme as the feature pool up
 * to 16384 rows; larger tables such as the 57,702-row threat table use a
 * radix-sorted row scatter with the same order).  Synchronises the stream for
 * tables of more than 16384 rows.  Replaces SparsePoolGrad / kernel sparse_pool_grad
 * (src/az/fused_feature_pool.rs:94-106, CPU twin :342-370). */
size_t cnnue_sparse_pool_bwd_workspace_bytes(int64_t rows, int64_t batch, int64_t item_count,
                                             int64_t hidden);
int cnnue_sparse_pool_bwd(const uint32_t* d_items, const float* d_grad_out, int64_t rows,
                          int64_t batch, int64_t item_count, int64_t hidden, float* d_grad_table,
                          void* d_workspace, size_t workspace_bytes, void* stream);

/* ---- AZ-NNUE policy-head training ops ------------------------------------
 * fused_policy: one logit per (board, move slot) from the 182,886-float
 * policy table (sections: consequence rows [1260][32] at 0, consequence
 * weights [32] at 40320, move bias [2086] at 40352, move context [2086][16]
 * at 42438, accumulator feature rows [1260][32] at 75814, accumulator move
 * factors [2086][32] at 116134), the board context [B][48] (16 move-context
 * values, then 32 accumulator values) and i64 items [B][M] packed as
 * move | from << 12 | to << 23 | captured << 34 | move_valid << 45 |
 * capture_valid << 46 | policy_valid << 47 (src/az/fused_policy.rs:10-35,
 * :146-157).  Items without policy_valid give 0; an item whose move or
 * feature indices fall outside their sections gives 0 and ORs
 * CNNUE_STATUS_BAD_INDEX into *d_status.  Terms are added one product at a
 * time in the CPU twin's order, so logits equal it bit for bit.
 * Replaces FusedPolicy (src/az/fused_policy.rs:159-245, CPU twin :178-241). */
#define CNNUE_POLICY_TABLE_LEN 182886
#define CNNUE_POLICY_CONTEXT 48
int cnnue_policy_fused_fwd(const float* d_tables, const float* d_context, const int64_t* d_items,
                           int64_t batch, int64_t moves, float* d_out, uint32_t* d_status,
                           void* stream);
/* Backward of fused_policy: d_grad_tables [182886] and d_grad_context [B][48]
 * are overwritten.  No atomics: grad_context[b] adds its board's moves in
 * order; table entries are summed in item order through stable radix sorts of
 * the feature rows (to, from, captured) and move rows each item touches.  An
 * entry with at most 256 contributions equals the CPU twin bit for bit; the
 * 32 consequence weights (every move item contributes) do when the batch has
 * at most 256 items.  Longer sums run in ordered units of 256: deterministic.
 * Bad items are flagged in the workspace status.  Synchronises the stream
 * (the sorts' run counts are read back).
 * Replaces FusedPolicyGrad (src/az/fused_policy.rs:263-371, CPU twin :287-366,
 * CUDA kernel fused_policy_grad :73-126, which uses atomicAdd). */
size_t cnnue_policy_fused_bwd_workspace_bytes(int64_t batch, int64_t moves);
int cnnue_policy_fused_bwd(const float* d_tables, const float* d_context, const int64_t* d_items,
                           const float* d_grad_out, int64_t batch, int64_t moves, float* d_grad_tables,
                           float* d_grad_context, void* d_workspace, size_t workspace_bytes,
                           void* stream);

/* Sparse / tactical policy table lookup: out[o] = sum over k < terms of
 * table[indices[o * terms + k]] in order (terms = 7 for sparse_policy, 2 for
 * tactical_policy); an index outside [0, table_len) is skipped and flagged.
 * Replaces SparsePolicy (src/az/fused_sparse_policy.rs:56-110, CPU twin :86-107). */
int cnnue_policy_table_fwd(const float* d_table, int64_t table_len, const int64_t* d_indices,
                           int64_t outputs, int terms, float* d_out, uint32_t* d_status,
                           void* stream);
/* Its backward: d_grad_table[j] = sum of grad_out[o] over every (o, k) with
 * indices[o * terms + k] == j, in (o, k) order, without atomics (the same
 * sorted scatter as cnnue_policy_fused_bwd).  Replaces SparsePolicyGrad
 * (src/az/fused_sparse_policy.rs:112-175, CPU twin :138-165). */
size_t cnnue_policy_table_bwd_workspace_bytes(int64_t outputs, int terms);
int cnnue_policy_table_bwd(const int64_t* d_indices, const float* d_grad_out, int64_t outputs,
                           int terms, int64_t table_len, float* d_grad_table, void* d_workspace,
                           size_t workspace_bytes, void* stream);

/* ---- training step (data parallel), HalfKA network --------------------- */
/* One rank's step of the fp32-master / bf16-activation form of the quantised
 * network: FT 11340x1024 (bf16 shadow gathered, fp32 sums), pairwise product
 * pack x = clamp(a_j,0,1)*clamp(a_j+512,0,1), bucket stacks 1024->16->32->1
 * with clipped ReLU, loss = mean((sigmoid(score/400) - target)^2).
 * Flat fp32 parameter layout (CNNUE_T_PARAMS floats):
 *   ft [11340][1024] | ft_bias [1024] | w1 [16][16][1024] | b1 [16][16] |
 *   w2 [16][32][16] | b2 [16][32] | w3 [16][32] | b3 [16]
 * The bf16 shadow covers ft and ft_bias (CNNUE_T_SHADOW elements).
 * Replaces the reference trainer's batch step GpuTrainer::compute_batch_grads
 * (src/az/train_gpu_candle.rs:184-219), with the FT backward of
 * FeaturePoolGrad (src/az/fused_feature_pool.rs:51-76) done without atomics,
 * and AdamW::step (src/az/train_gpu_candle.rs:159) by plain Adam. */
#define CNNUE_T_FEATURES 11340
#define CNNUE_T_SHADOW (11340 * 1024 + 1024)
#define CNNUE_T_PARAMS (11340 * 1024 + 1024 + 16 * 16 * 1024 + 16 * 16 + 16 * 32 * 16 + 16 * 32 + 16 * 32 + 16)
size_t cnnue_t_param_count(void);
size_t cnnue_t_workspace_bytes(int64_t n_positions, uint32_t n_indices);
/* Writes the bf16 shadow of the FT weights and bias from the fp32 params. */
int cnnue_t_make_shadow(const float* d_params, uint16_t* d_shadow, void* stream);
/* Forward + backward of one rank's batch (CSR positions as cnnue_q_forward,
 * targets fp32 [n]).  Writes the gradient of the rank's mean loss for every
 * parameter into d_grads (flat layout; no accumulation across calls) and the
 * mean loss into d_loss[0].  Deterministic: no atomics on floats.  Kernel
 * status (bad index / offsets) lands in the workspace's first word. */
int cnnue_t_forward_backward(const float* d_params, const uint16_t* d_shadow,
                             const uint16_t* d_indices, uint32_t n_indices,
                             const uint32_t* d_offsets, int64_t n_positions, const float* d_target,
                             float* d_grads, float* d_loss, void* d_workspace,
                             size_t workspace_bytes, void* stream);
/* cnnue_t_forward_backward in three phases, so that a data-parallel caller
 * can exchange gradients while the FT gradient is still being reduced (the
 * backward of GpuTrainer::compute_batch_grads, src/az/train_gpu_candle.rs:
 * 166-219, split at its gradient boundaries):
 *   _begin: everything but the FT gradient - gather, head, loss terms, the
 *     stack gradients (W1..b3 of d_grads are final when it completes) and the
 *     preparation of the FT segmented reduction;
 *   _ft_grad_rows: the FT gradient rows [row_begin, row_end) of the table
 *     [11340 + 1][1024] (row 11340 is the FT bias); ranges may be issued in
 *     any order and split any way, results are the same;
 *   _finish: the mean loss into d_loss[0] and, when d_flag is not null, the
 *     kernels' status as a float flag (0 clean, 1 bad input) to reduce with
 *     the gradient. */
int cnnue_t_forward_backward_begin(const float* d_params, const uint16_t* d_shadow, const uint16_t* d_indices,
                                   uint32_t n_indices, const uint32_t* d_offsets, int64_t n_positions,
                                   const float* d_target, float* d_grads, void* d_workspace,
                                   size_t workspace_bytes, void* stream);
int cnnue_t_ft_grad_rows(int64_t n_positions, uint32_t n_indices, float* d_grads, void* d_workspace,
                         size_t workspace_bytes, int64_t row_begin, int64_t row_end, void* stream);
int cnnue_t_finish(int64_t n_positions, uint32_t n_indices, float* d_loss, void* d_workspace,
                   size_t workspace_bytes, float* d_flag, void* stream);

/* Adam step over all parameters with gradient grad * grad_scale (e.g. 1/world
 * after a sum all-reduce); refreshes the bf16 shadow.  step counts from 1.
 * When d_skip is not null and *d_skip != 0 (a status flag summed over the
 * ranks) nothing is updated. */
int cnnue_t_adam(float* d_params, float* d_m, float* d_v, const float* d_grads, uint16_t* d_shadow,
                 float grad_scale, float lr, float beta1, float beta2, float eps, int step,
                 const float* d_skip, void* stream);
/* The same Adam step over the parameters [begin, end) only (flat
 * indices; the shadow is refreshed for those below the FT end): a data-
 * parallel rank's shard after a reduce-scatter of the gradient. */
int cnnue_t_adam_range(float* d_params, float* d_m, float* d_v, const float* d_grads, uint16_t* d_shadow,
                       int64_t begin, int64_t end, float grad_scale, float lr, float beta1, float beta2, float eps,
                       int step, const float* d_skip, void* stream);

/* AdamW step over n fp32 parameters (flat buffer) with moments m, v, as
 * candle-nn's AdamW::step (the AZ trainer's optimizer, lr / betas / eps /
 * weight decay as src/az/train_gpu_candle.rs:113-122), operation for
 * operation in fp32: m' = m*b1 + g*(1-b1); v' = v*b2 + g*g*(1-b2);
 * p' = p*(1 - lr*wd) - lr * (m'/(1-b1^t)) / (sqrt(v'/(1-b2^t)) + eps).
 * step counts from 1.  One pass, no atomics. */
int cnnue_adamw(float* d_params, float* d_m, float* d_v, const float* d_grads, int64_t n, double lr,
                double beta1, double beta2, double eps, double weight_decay, int64_t step,
                void* stream);
/* The same step with its hyper-parameters and step counter in device memory
 * (so a captured CUDA graph replays it step after step): the call advances
 * d_state->step by one on the device, then applies AdamW with the new step.
 * The host may rewrite lr (set_learning_rate) between replays. */
typedef struct cnnue_adamw_state {
  double lr, beta1, beta2, eps, weight_decay;
  int64_t step;        /* steps taken; 0 before the first */
  float scalars[9];    /* written by the device: this step's fp32 factors */
  float pad[3];        /* pad[0]: 1 when the last device step was skipped */
} cnnue_adamw_state;
int cnnue_adamw_device(float* d_params, float* d_m, float* d_v, const float* d_grads, int64_t n,
                       cnnue_adamw_state* d_state, void* stream);
/* The device-state step for a data-parallel exchange: every gradient is
 * multiplied by grad_scale first (1/world after a sum all-reduce), and when
 * any of d_skip[0..n_skip) is nonzero (status bits summed over the ranks)
 * the step is skipped on the device - nothing changes and the step counter
 * stays; d_state->pad[0] then reads 1 (0 after a step taken). */
int cnnue_adamw_device_scaled(float* d_params, float* d_m, float* d_v, const float* d_grads, int64_t n,
                              cnnue_adamw_state* d_state, float grad_scale, const float* d_skip, int n_skip,
                              void* stream);

/* ---- reference-native AZ-NNUE evaluator (src/az.rs, src/nnue.rs) -------- */
/* Squares are rank * 9 + file with rank 0 the first rank of a FEN (Black's
 * back rank), as src/xiangqi/geom.rs:28-30.  A board is int8_t[90]: 0 empty,
 * +(kind+1) Red, -(kind+1) Black, kind = General 0, Advisor 1, Elephant 2,
 * Horse 3, Rook 4, Cannon 5, Soldier 6 (piece_kind_index,
 * src/xiangqi/types.rs:206-216).  Perspective / side: 0 Red, 1 Black.
 * An item packs one piece of one perspective as feature | us_bucket << 11 |
 * them_bucket << 15 (pack_feature, src/az/fused_feature_pool.rs:130-132):
 * feature = (own ? 0 : 7 + kind) * 90 + canonical square (sq for Red,
 * 89 - sq for Black), buckets = the king-palace buckets of both generals
 * (src/az.rs:168-203), 4 when a general is absent. */
#define CNNUE_AZ_SQUARES 90
#define CNNUE_AZ_INPUT 1260          /* 14 piece kinds x 90 squares            */
#define CNNUE_AZ_TRUNK_ROWS 1545     /* input 1260 + piece 14 + rank 10 + file 9 + king-piece 252 */
#define CNNUE_AZ_VALUE_HEAD 96
#define CNNUE_AZ_RULE_CONTEXT 7
#define CNNUE_AZ_WDL 3
#define CNNUE_AZ_TENSORS 22
#define CNNUE_AZ_MAX_HIDDEN 512
#define CNNUE_AZ_NO_ITEM 0xffffffffu
#define CNNUE_AZ_FORMAT_VERSION 20.0f /* az_model_format_version (src/version.rs:5) */

/* FEN board field and side (src/xiangqi/mod.rs:163-207): ranks split by '/',
 * digits skip files, letters k a b/e n/h r c p, uppercase Red; side "w"/"r"
 * Red, "b" Black, missing = Red.  CNNUE_ERR_FORMAT on a malformed FEN. */
int cnnue_az_board_from_fen(const char* fen, int8_t* board, int* side);
/* Items of one perspective in board-scan order (fill_sparse_features_az,
 * src/nnue.rs:31-43, with refresh_perspective's perspective,
 * src/az.rs:413-426).  items holds 90; *count gets the piece count. */
int cnnue_az_features(const int8_t* board, int perspective, uint32_t* items, int* count);
/* What apply_transition_for_perspective (src/az.rs:439-485) adds and removes
 * for the move from -> to on `board` (the position before the move): if the
 * perspective's (us, them) bucket pair changes, *refresh = 1 and items/count
 * get the child's features; else *refresh = 0 and delta = {moved piece at
 * from, captured piece at to or CNNUE_AZ_NO_ITEM, moved piece at to}. */
int cnnue_az_move_items(const int8_t* board, int from, int to, int perspective, uint32_t* delta,
                        uint8_t* refresh, uint32_t* items, int* count);

/* Threat features of the side to move (value_threat_logits' accumulation,
 * src/az.rs:2078-2101): for every piece attacking an occupied square
 * (Position::visit_occupied_attacks, src/xiangqi/mod.rs:286-389, sources in
 * square order) the index of value_threat_index (src/az.rs:718-742) into the
 * 57,702-row threat table; relations outside threat_relation_map
 * (src/az.rs:577-661) are skipped.  features holds CNNUE_AZ_THREAT_MAX. */
#define CNNUE_AZ_THREAT_VOCAB 57702
#define CNNUE_AZ_THREAT_RANK 64
#define CNNUE_AZ_THREAT_MAX 256
int cnnue_az_threat_features(const int8_t* board, int perspective, uint32_t* features, int* count);
/* Size of the enumerated threat vocabulary (57,702 when the enumeration is
 * the reference's; the reference asserts the same count). */
int cnnue_az_threat_vocab(void);

/* ---- AZ-NNUE training batch packer ---------------------------------------
 * Training samples (the AzTrainingSample fields the packer reads) in CSR
 * form: features (canonical side-to-move piece-square features, as stored
 * by the self-play writer) per sample, its move_indices (dense move space;
 * >= 2086 are skipped) with their policy targets alongside, value_wdl [n][3],
 * value [n], rule_context [n][7], policy_weight [n], value_weight [n], ply [n]. */
typedef struct cnnue_az_samples {
  int64_t n;
  const uint16_t* features;
  const uint32_t* feature_offsets; /* [n + 1] */
  const uint16_t* move_indices;
  const float* policy;
  const uint32_t* move_offsets;    /* [n + 1] */
  const float* value_wdl;
  const float* value;
  const float* rule_context;
  const float* policy_weight;
  const float* value_weight;
  const uint32_t* ply;
} cnnue_az_samples;
/* The packed batch (PackedBatch, src/az/dataloader.rs:92-111): row-major
 * arrays with the batch's own strides F = max_features, M = max_policy_moves,
 * T = max_value_threats (each at least 1):
 *   feature_items u32 [B][F] (pack_feature items, 0xffffffff padding),
 *   value_threat_indices u32 [B][T], policy_items i64 [B][M] (fused_policy
 *   items, 0 padding), policy_sparse_indices i64 [B][M][7] (padding 2396814),
 *   policy_tactical_indices i64 [B][M][2] (padding 934976), policy_targets
 *   f32 [B][M] (normalised), policy_mask f32 [B][M] (0 or -1e9), value_wdl
 *   f32 [B][3] (normalised), values f32 [B] (clamped to [-1,1]), rule_context
 *   f32 [B][7], policy_weights / value_weights f32 [B], value_phase_masks f32
 *   [B][3] (ply < 40, < 120, else). */
typedef struct cnnue_az_packed {
  int64_t batch, max_features, max_policy_moves, max_value_threats; /* written by the packer */
  uint32_t* feature_items;
  uint32_t* value_threat_indices;
  int64_t* policy_items;
  int64_t* policy_sparse_indices;
  int64_t* policy_tactical_indices;
  float* policy_targets;
  float* policy_mask;
  float* value_wdl;
  float* values;
  float* rule_context;
  float* policy_weights;
  float* value_weights;
  float* value_phase_masks;
  /* compact form (policy_sparse_indices, policy_tactical_indices and
   * policy_mask all NULL): per move the 6-bit tactical signature (0 for moves
   * without an own piece on the source), per row us_bucket | them_bucket << 4;
   * cnnue_az_expand_policy_indices rebuilds the index arrays on the device */
  uint8_t* policy_signature;       /* [B][M] */
  uint8_t* king_buckets;           /* [B] */
} cnnue_az_packed;
/* Packs the samples rows[0..batch) (rows NULL = 0..batch) on n_threads host
 * threads (<= 0: up to 16).  The output arrays must hold the capacities
 * cap_features / cap_moves / cap_threats per row; the dims actually used are
 * written to out first, and CNNUE_ERR_WORKSPACE is returned (nothing else
 * written) when a capacity is too small.  With fixed_strides the capacities
 * themselves are the strides (extra columns hold the padding values), so
 * every batch has the same shapes.  Replaces PackedBatch::from_indices
 * (src/az/dataloader.rs:113-336). */
int cnnue_az_pack_batch(const cnnue_az_samples* samples, const int64_t* rows, int64_t batch,
                        int64_t cap_features, int64_t cap_moves, int64_t cap_threats, int fixed_strides,
                        cnnue_az_packed* out, int n_threads);

/* Device half of the compact packed batch: the sparse [B][M][7] and
 * tactical [B][M][2] index arrays of the policy lookups rebuilt from the
 * policy items (move, source and destination squares, pieces, flags), the
 * per-move signatures and the per-row king buckets - equal to what
 * cnnue_az_pack_batch writes in full form (policy_sparse_main_index /
 * _capture_index / _factor_indices, policy_tactical_indices,
 * src/az.rs:763-859).  d_mask (optional) gets 0 for policy-valid items and
 * -1e9 elsewhere (the packer's policy_mask). */
int cnnue_az_expand_policy_indices(const int64_t* d_items, const uint8_t* d_signature,
                                   const uint8_t* d_king_buckets, int64_t batch, int64_t moves,
                                   int64_t* d_sparse, int64_t* d_tactical, float* d_mask, void* stream);

/* ---- native AZ-NNUE training step --------------------------------------
 * One train_batch_single (src/az/train_gpu_candle.rs:145-160) without its
 * optimizer step: AzCandleModel::forward (src/az/candle_model.rs:46-147),
 * compute_batch_loss (train_gpu_candle.rs:221-305) and the gradients of all
 * 22 weight tensors, as a fixed set of kernels (no autograd graph).  The
 * parameters and their gradients live in flat fp32 buffers of 17 leaves in
 * this order: trunk table [1545][H] (tensors 0-4), rule_context_hidden
 * [7][H], hidden_bias [H], value_head_hidden [96][H], value_head_bias [96],
 * value_head_output [3][96], value_threat_embedding [57702][64],
 * value_threat_output [3][128], policy_threat_context [16][128],
 * policy_move_bias [2086], policy_consequence_output [32],
 * policy_context_hidden [16][H], policy_move_context [2086][16],
 * policy_accumulator_hidden [32][H], policy_accumulator_move [2086][32],
 * sparse table [2596273] (tensors 19-20), tactical table [934976] followed
 * by its constant zero; leaf_offsets[17] are element offsets, multiples of
 * 4.  The gradients are summed into nothing: d_grads[0..n_grads) is zeroed
 * first.  The batch is the packed batch in full form (device pointers;
 * expand a compact one with cnnue_az_expand_policy_indices first).
 * d_metrics[35] gets the 30 statistics of AzTrainStats (loss sum, value CE
 * sum, policy CE sum, the six value sums, the 3 x 7 phase table), the four
 * status bits as 0/1 floats and the status word as a float (a layout that
 * sums meaningfully over data-parallel ranks: d_metrics may point into the
 * tail of the gradient buffer that is all-reduced); d_status is cleared, then collects
 * CNNUE_STATUS_BAD_INDEX for indices outside their tables (those lookups
 * read 0 and pass no gradient).  hidden: 32, 64, 128, 256 or 512; moves <=
 * 1024.  Deterministic: the same inputs give the same bits, run to run.
 * The engine holds a second stream on which the batch's table indices are
 * sorted while the forward runs; a step may be captured in a CUDA graph
 * (the engine's stream joins the capture).  One engine per thread. */
#define CNNUE_AZT_LEAVES 17
typedef struct cnnue_azt_batch {
  int64_t batch, features, moves, threats; /* B, F, M, T */
  const uint32_t* feature_items;           /* [B][F] */
  const uint32_t* value_threat_indices;    /* [B][T] */
  const int64_t* policy_items;             /* [B][M] */
  const int64_t* policy_sparse_indices;    /* [B][M][7] */
  const int64_t* policy_tactical_indices;  /* [B][M][2] */
  const float* policy_targets;             /* [B][M] */
  const float* policy_mask;                /* [B][M] */
  const float* value_wdl;                  /* [B][3] */
  const float* values;                     /* [B] */
  const float* rule_context;               /* [B][7] */
  const float* policy_weights;             /* [B] */
  const float* value_weights;              /* [B] */
  const float* value_phase_masks;          /* [B][3] */
} cnnue_azt_batch;
typedef struct cnnue_azt cnnue_azt;
int cnnue_azt_create(int device, cnnue_azt** out);
int cnnue_azt_destroy(cnnue_azt* engine);
/* Workspace of one step (0 for unsupported dims); 256-byte aligned. */
size_t cnnue_azt_workspace_bytes(int64_t hidden, int64_t batch, int64_t features, int64_t moves, int64_t threats);
/* Optional AdamW inside the step (single GPU): params must be d_params (then
 * updated in place), m / v the moments in the same layout, state the device
 * state of cnnue_adamw_device; the leaves must be in the order above from
 * offset 0.  The table leaves are updated while the dense gradients finish. */
typedef struct cnnue_azt_optim {
  float* params;
  float* m;
  float* v;
  cnnue_adamw_state* state;
} cnnue_azt_optim;
int cnnue_azt_step(cnnue_azt* engine, const float* d_params, float* d_grads, int64_t n_grads,
                   const int64_t* leaf_offsets, int64_t hidden, const cnnue_azt_batch* batch, float value_weight,
                   float policy_weight, float* d_metrics, uint32_t* d_status, void* d_ws, size_t ws_bytes,
                   const cnnue_azt_optim* optim, void* stream);

/* Per-move records for the policy logits (the per-move inputs of
 * evaluate_prepared_hidden_with_context, src/az.rs:1766-1887), side to move
 * `side`.  moves[2i], moves[2i+1] = from, to squares (absolute).  info[2i] =
 * dense move index of the canonical move (12 bits, 0xfff when not in the
 * dense space) | moved piece index << 12 | captured piece index << 16 (15 =
 * none) | tactical signature << 20 (bits: from attacked by the opponent, to
 * attacked, from defended, to defended, capture, gives check:
 * attacked_squares_mask, src/xiangqi/mod.rs:391-484, and
 * gives_check_after_move_fast, :763-1012); info[2i+1] = canonical from |
 * canonical to << 7 | us bucket << 14 | them bucket << 18. */
int cnnue_az_policy_moves(const int8_t* board, int side, const uint8_t* moves, int n_moves, uint32_t* info);

/* Host weights: the 22 fp32 tensors of az_weight_tensors! (src/az.rs:241-278)
 * in that order, row-major. */
typedef struct cnnue_az_weights cnnue_az_weights;
/* Name and element count of tensor `index` at hidden size `hidden`. */
int cnnue_az_tensor_info(int index, int64_t hidden, const char** name, int64_t* count);
/* AzNnue::random(hidden, seed) (src/az.rs:1339-1431): the same SplitMix64
 * draws in the same order, so the tensors equal the reference's. */
int cnnue_az_weights_random(int64_t hidden, uint64_t seed, cnnue_az_weights** out);
/* AzNnue::load / save (src/az.rs:1437-1529, validate :2453-2499): a
 * safetensors file of F32 tensors named as az_weight_tensors! plus
 * az_model_format_version = [20.0].  CNNUE_ERR_IO if the file cannot be read
 * or written, CNNUE_ERR_FORMAT for a bad header, a missing tensor, another
 * dtype, a wrong format tag or a length mismatch (the hidden size comes from
 * hidden_bias). */
int cnnue_az_weights_load(const char* path, cnnue_az_weights** out);
int cnnue_az_weights_save(const cnnue_az_weights* weights, const char* path);
int cnnue_az_weights_destroy(cnnue_az_weights* weights);
int64_t cnnue_az_weights_hidden(const cnnue_az_weights* weights);
/* Host view of tensor `index` (writable; a model created later sees edits). */
int cnnue_az_weights_tensor(cnnue_az_weights* weights, int index, float** data, int64_t* count);

/* Quantised tables (rebuild_policy_accumulator_quantization,
 * rebuild_value_threat_quantization, rebuild_policy_tactical,
 * src/az.rs:2201-2342).  cnnue_az_weights_random and _load build them, as
 * AzNnue::random and ::load do; after editing tensors call
 * cnnue_az_quantize again.  Symmetric per-tensor int8: scale = max(max|x| /
 * 127, 1e-12), q = clamp(round(x / scale), -127, 127), round half away from
 * zero.  The policy feature rows are the 1546 rows (1260 input, 14 piece,
 * 10 rank, 9 file, 252 king-piece, 1 hidden_bias) projected on the 32 rows of
 * policy_accumulator_hidden with the reference's x86-64 AVX2/FMA dot product
 * summation order (dot_product, src/az.rs:2730-2766, :2880-2922), so the
 * tables are bit-identical to the reference's on that platform. */
#define CNNUE_AZ_Q_POLICY_FEATURE 0  /* int8  [1546][32]   */
#define CNNUE_AZ_Q_POLICY_MOVE 1     /* int8  [2086][32]   */
#define CNNUE_AZ_Q_POLICY_SPARSE 2   /* int8  [2396815], sparse factors folded in */
#define CNNUE_AZ_Q_VALUE_THREAT 3    /* int8  [57702][64]  */
#define CNNUE_AZ_Q_MOVED_DELTA 4     /* int32 [2086][14]   */
#define CNNUE_AZ_Q_CAPTURE 5         /* int32 [2086][14]   */
#define CNNUE_AZ_DENSE_MOVES 2086
#define CNNUE_AZ_POLICY_RANK 32
#define CNNUE_AZ_POLICY_ROWS 1546
int cnnue_az_quantize(cnnue_az_weights* weights);
/* Host view of quantised table `which`; *scale gets its scale (1 for the
 * int32 caches).  Element size: 1 byte for the int8 tables, 4 for int32. */
int cnnue_az_quant_table(const cnnue_az_weights* weights, int which, const void** data, int64_t* count,
                         float* scale);
/* value_threat_active, policy_tactical_active (src/az.rs:2202-2206, :2223-2225). */
int cnnue_az_quant_flags(const cnnue_az_weights* weights, int* value_threat_active,
                         int* policy_tactical_active);
/* The dense policy move space (move_map, src/az.rs:3261-3285): the 2086
 * from * 90 + to pairs of is_valid_policy_move (:3206-3237) in from-major
 * order; sparse_to_dense[8100] gets the inverse, 0xffff for invalid pairs.
 * Either pointer may be NULL. */
int cnnue_az_dense_moves(uint16_t* dense_to_sparse, uint16_t* sparse_to_dense);

/* Device copy of the trunk (the 5 input tables concatenated as [1545][H],
 * hidden_bias, rule_context_hidden) and the value head.  Hidden sizes 1..127
 * and multiples of 4 up to 512. */
typedef struct cnnue_az_model cnnue_az_model;
int cnnue_az_model_create(const cnnue_az_weights* weights, int device, cnnue_az_model** out);
int cnnue_az_model_destroy(cnnue_az_model* model);
/* The CUDA device ordinal the model lives on (-1 for a null model). */
int cnnue_az_model_device(const cnnue_az_model* model);
/* Workspace of the AZ entry points (the status word). */
size_t cnnue_az_workspace_bytes(void);

/* Accumulator refresh of n_lists item lists (CSR: offsets[n_lists+1] into
 * d_items): acc[l] = hidden_bias, + the input row of every item in list
 * order, + for every item its piece, rank, file, king-piece(us) and
 * king-piece(them) rows, one fp32 add per row per column in exactly that
 * order (input_embedding_linear_into_slice, src/az.rs:2049-2076, and
 * add_factorized_structure_into, :1920-2042), so the result is bit-identical
 * to the reference.  acc is [n_lists][H]; the two perspectives of a node are
 * two consecutive lists ([2][H], AzEvalAccumulator::refresh, src/az.rs:384-411).
 * An item with feature >= 1260 or a bucket > 8 is skipped and flagged
 * CNNUE_STATUS_BAD_INDEX; bad offsets are flagged CNNUE_STATUS_BAD_OFFSETS. */
int cnnue_az_refresh(const cnnue_az_model* model, const uint32_t* d_items, uint32_t n_items,
                     const uint32_t* d_offsets, int64_t n_lists, float* d_acc, void* d_workspace,
                     size_t workspace_bytes, void* stream);
/* Incremental accumulator update per list (apply_transition_for_perspective,
 * src/az.rs:439-485; add_canonical_piece_contribution, :509-566): if
 * d_refresh[l] & 1, child[l] = the refresh of list l of d_items/d_offsets;
 * else child[l] = parent[l] - 6 rows(delta[3l]) - 6 rows(delta[3l+1], unless
 * CNNUE_AZ_NO_ITEM) + 6 rows(delta[3l+2]), each item's rows in the order
 * input, piece, rank, file, king(us), king(them): bit-identical to the
 * reference.  d_items may be NULL when no list refreshes. */
int cnnue_az_transition(const cnnue_az_model* model, const float* d_parent, const uint32_t* d_delta,
                        const uint8_t* d_refresh, const uint32_t* d_items, uint32_t n_items,
                        const uint32_t* d_offsets, int64_t n_lists, float* d_child,
                        void* d_workspace, size_t workspace_bytes, void* stream);
/* Value of n positions from side-to-move accumulators: x = acc (+ the rule
 * context rows scaled by d_rule[p][k] for non-zero entries,
 * add_rule_context_to_hidden src/az.rs:1903-1918), ReLU, RMSNorm with eps
 * 1e-6 (src/az.rs:3020-3040, :3110-3126), value head 96 ReLU units, 3 logits
 * (+ d_threat[p][k] when not NULL), softmax, q = W - L
 * (value_wdl_from_hidden_into, src/az.rs:2133-2157; softmax_fixed3,
 * :2563-2575).  With d_side == NULL d_acc is [n][H]; else it is [n][2][H]
 * (both perspectives of a node) and position p reads perspective d_side[p].
 * d_rule ([n][7]) and d_threat ([n][3]) may be NULL.  Writes d_wdl [n][3]
 * and d_q [n] (AzEvalOutput). */
int cnnue_az_value(const cnnue_az_model* model, const float* d_acc, const uint8_t* d_side,
                   const float* d_rule, const float* d_threat, int64_t n, float* d_wdl, float* d_q,
                   void* stream);

/* Threat logits [n][3] of n positions (value_threat_logits, src/az.rs:
 * 2078-2120): acc[64] = wrapping int16 sum of the CNNUE_AZ_Q_VALUE_THREAT rows
 * of the position's threat features (CSR: offsets[n+1] into d_features),
 * act = clamp(acc * scale, 0, 1), logits = value_threat_output . (act ||
 * act^2) in the reference's dot-product order: bit-identical.  Feed them to
 * cnnue_az_value as d_threat when value_threat_active (else the reference
 * adds zeros).  A feature >= 57,702 is skipped and flagged BAD_INDEX. */
int cnnue_az_threat_logits(const cnnue_az_model* model, const uint32_t* d_features, uint32_t n_features,
                           const uint32_t* d_offsets, int64_t n, float* d_logits, void* d_workspace,
                           size_t workspace_bytes, void* stream);

/* The evaluator entry point evaluate_incremental_with_scratch_output
 * (src/az.rs:1606-1652) for n positions: side-to-move hidden from d_acc (+
 * rule context), ReLU, RMSNorm, value head with the threat logits of
 * d_threat_features (CSR; used when the model's value_threat_active is set)
 * -> d_wdl [n][3], d_q [n]; then, when d_move_info is given, the policy
 * logits of the listed moves (records of cnnue_az_policy_moves, CSR by
 * d_move_offsets) from the side-to-move policy accumulators d_policy_acc
 * (int16 [n][32], or [n][2][32] with d_side) -> d_logits [n_moves]
 * (evaluate_prepared_hidden_with_scratch + _with_context, src/az.rs:
 * 1738-1887: move bias + piece-square consequence + context . move context
 * + quantised accumulator + folded sparse table + tactical table, summed in
 * that order).  The workspace holds the normalised hidden and the threat
 * activations between the kernels. */
size_t cnnue_az_evaluate_workspace_bytes(const cnnue_az_model* model, int64_t n);
int cnnue_az_evaluate(const cnnue_az_model* model, const float* d_acc, const uint8_t* d_side,
                      const float* d_rule, const uint32_t* d_threat_features, uint32_t n_threat_features,
                      const uint32_t* d_threat_offsets, const int16_t* d_policy_acc,
                      const uint32_t* d_move_info, uint32_t n_moves, const uint32_t* d_move_offsets,
                      int64_t n, float* d_wdl, float* d_q, float* d_logits, void* d_workspace,
                      size_t workspace_bytes, void* stream);

/* int16 policy accumulators [n_lists][32] (quantized_policy_accumulator,
 * src/az.rs:2344-2365): the bias row, then for every item its 6 rows of the
 * CNNUE_AZ_Q_POLICY_FEATURE table (input, piece, rank, file, king(us),
 * king(them)), each row add saturating to int16 in that order
 * (add_quantized_policy_row, :2439-2451): bit-identical to the reference.
 * Same lists, status and skipping rules as cnnue_az_refresh. */
int cnnue_az_policy_refresh(const cnnue_az_model* model, const uint32_t* d_items, uint32_t n_items,
                            const uint32_t* d_offsets, int64_t n_lists, int16_t* d_acc,
                            void* d_workspace, size_t workspace_bytes, void* stream);
/* apply_quantized_policy_transition (src/az.rs:2367-2409): parent minus the
 * rows of delta[3l] and delta[3l+1], plus those of delta[3l+2], saturating per
 * row, or the refresh of list l where d_refresh[l] & 1.  child may be parent. */
int cnnue_az_policy_transition(const cnnue_az_model* model, const int16_t* d_parent,
                               const uint32_t* d_delta, const uint8_t* d_refresh,
                               const uint32_t* d_items, uint32_t n_items, const uint32_t* d_offsets,
                               int64_t n_lists, int16_t* d_child, void* d_workspace,
                               size_t workspace_bytes, void* stream);

/* ---- AlphaZero policy/value ResNet for MCTS leaf batches ---------------- */
/* No counterpart in the reference's code (its evaluator is the AZ-NNUE
 * above); this is the dense network of the workload specification, evaluated
 * where the reference evaluates leaves (AzNnue::evaluate_with_scratch_output,
 * src/az.rs:1562-1604; MCTS leaf batches, src/az/alphazero.rs:388-521).
 * Input planes bf16 [B][15][10][9]: 14 piece planes and a side-to-move plane.
 * Trunk: conv 3x3 15->128 + bias, ReLU; 10 residual blocks h = ReLU(conv1(x)
 * + b1), x = ReLU(conv2(h) + b2 + x) (BN folded into weights and biases);
 * activations stored as bf16 after every layer, sums in fp32 on the tensor
 * cores.  Policy: ReLU(conv1x1 128->2 + b), flattened channel-major (c * 90 +
 * square), FC 180->2086, softmax.  Value: ReLU(conv1x1 128->1 + b), FC
 * 90->256 + ReLU, FC 256->1, tanh.  Heads in fp32. */
#define CNNUE_RN_PLANES 15
#define CNNUE_RN_CHANNELS 128
#define CNNUE_RN_BLOCKS 10
#define CNNUE_RN_MOVES 2086
typedef struct cnnue_rn_weights {   /* host fp32, PyTorch layouts; conv weights
                                       are rounded to bf16 on upload */
  const float* stem_w;         /* [128][15][3][3]            */
  const float* stem_b;         /* [128]                      */
  const float* block_w;        /* [10][2][128][128][3][3]    */
  const float* block_b;        /* [10][2][128]               */
  const float* policy_conv_w;  /* [2][128]                   */
  const float* policy_conv_b;  /* [2]                        */
  const float* policy_fc_w;    /* [2086][180]                */
  const float* policy_fc_b;    /* [2086]                     */
  const float* value_conv_w;   /* [128]                      */
  const float* value_conv_b;   /* [1]                        */
  const float* value_fc1_w;    /* [256][90]                  */
  const float* value_fc1_b;    /* [256]                      */
  const float* value_fc2_w;    /* [256]                      */
  const float* value_fc2_b;    /* [1]                        */
} cnnue_rn_weights;
typedef struct cnnue_rn_model cnnue_rn_model;
int cnnue_rn_model_create(const cnnue_rn_weights* weights, int device, cnnue_rn_model** out);
int cnnue_rn_model_destroy(cnnue_rn_model* model);
size_t cnnue_rn_workspace_bytes(int64_t batch);
/* d_planes bf16 bits [B][15][90]; writes d_probs [B][2086] (softmax),
 * d_logits [B][2086] (may be NULL) and d_value [B] (tanh).  A bounded wait
 * that gives up is reported through the workspace status word. */
int cnnue_rn_forward(const cnnue_rn_model* model, const uint16_t* d_planes, int64_t batch, float* d_probs,
                     float* d_logits, float* d_value, void* d_workspace, size_t workspace_bytes,
                     void* stream);
/* Conv kernel choice: 2 (default) the halo kernel (activations in a padded,
 * 8-board-interleaved layout where every 3x3 tap is a whole-atom row shift of
 * one shared-memory halo tile), 1 the persistent square-major kernel (one CTA
 * per SM, two 128-row tiles per K block sharing each weight tile,
 * double-buffered TMEM), 0 the one-tile-per-CTA kernel.  All compute the same
 * convolution. */
int cnnue_rn_set_conv_kernel(cnnue_rn_model* model, int kind);

/* ---- deterministic synthetic workloads (host) --------------------------- */
/* SplitMix64 as the reference defines it (src/az.rs:3146-3176): the state is
 * replaced by the mixed output at every draw. */
uint64_t cnnue_splitmix64_next(uint64_t* state);

/* Positions: per position and perspective a count n uniform in
 * [min_active, max_active] and n unique indices uniform in [0, n_features),
 * sorted ascending.  Writes at most 2*n_positions*max_active indices and
 * 2*n_positions+1 offsets; returns the index count through *n_indices. */
int cnnue_synth_positions(uint64_t seed, int64_t n_positions, uint32_t n_features,
                          uint32_t min_active, uint32_t max_active, uint16_t* h_indices,
                          uint32_t* h_offsets, uint32_t* n_indices);
/* Quantised weights from seed: FT uniform in [-127,127], FT bias in [-64,64],
 * stack weights uniform in [-64,64], stack biases in [-64,64]; the arrays
 * must have the sizes of cnnue_q_weights. */
int cnnue_synth_q_weights(uint64_t seed, int16_t* ft_weight, int16_t* ft_bias, int8_t* l1_weight,
                          int32_t* l1_bias, int8_t* l2_weight, int32_t* l2_bias,
                          int8_t* l3_weight, int32_t* l3_bias);
/* fp32 weights: FT N(0, 0.01), FT bias 0, stack N(0, 0.05), stack biases 0
 * (Box-Muller over the SplitMix64 stream). */
int cnnue_synth_f_weights(uint64_t seed, float* ft_weight, float* ft_bias, float* l1_weight,
                          float* l1_bias, float* l2_weight, float* l2_bias, float* l3_weight,
                          float* l3_bias);
/* Incremental-update workload: parents uniform in [-2000,2000]; per
 * perspective 1-2 removed and 1-3 added indices, or with probability 1/20 a
 * refresh with 2-32 fresh unique sorted indices; child perspective-0 count.
 * Capacities: h_rem 4n, h_add 64n. */
/* ResNet weights (sizes of cnnue_rn_weights, writable arrays): conv weights
 * He-normal N(0, sqrt(2 / fan_in)), the second conv of each block scaled by
 * 1/4 (a small residual branch keeps activations bounded through 10 blocks),
 * conv biases N(0, 0.02), FC weights N(0, sqrt(1 / fan_in)), FC biases
 * N(0, 0.02); every value rounded to a bf16 value. */
int cnnue_synth_rn_weights(uint64_t seed, float* stem_w, float* stem_b, float* block_w, float* block_b,
                           float* policy_conv_w, float* policy_conv_b, float* policy_fc_w,
                           float* policy_fc_b, float* value_conv_w, float* value_conv_b,
                           float* value_fc1_w, float* value_fc1_b, float* value_fc2_w,
                           float* value_fc2_b);
/* Input planes bf16 bits [B][15][90]: per board k uniform in [0,32] pieces on
 * distinct squares, each of a kind uniform over the 14 piece planes; plane 14
 * all ones with probability 1/2 (side to move). */
int cnnue_synth_rn_planes(uint64_t seed, int64_t batch, uint16_t* planes);
int cnnue_synth_q_update(uint64_t seed, int64_t n_positions, int16_t* h_parent, uint8_t* h_flags,
                         uint16_t* h_rem, uint32_t* h_rem_offsets, uint32_t* n_rem,
                         uint16_t* h_add, uint32_t* h_add_offsets, uint32_t* n_add,
                         uint8_t* h_count0);

/* ---- wide-batch AlphaZero search ------------------------------------------
 * Legal moves of `side` (pseudo-legal moves of every piece, less those that
 * leave the mover's general attacked or facing the other general on an open
 * file), as from/to square pairs in moves[2i], moves[2i+1]; *count gets the
 * number (CNNUE_ERR_WORKSPACE when it exceeds capacity).  Board as above. */
int cnnue_az_legal_moves(const int8_t* board, int side, uint8_t* moves, int capacity, int* count);

/* AzSearchLimits (src/az/alphazero.rs:22-66) less the seed and root
 * Dirichlet noise: the PUCT constants, max_depth (0 = simulations), first
 * play urgency, policy softmax temperature, draw score and value scale. */
typedef struct cnnue_mcts_limits {
  int64_t simulations;
  float cpuct, cpuct_at_root, cpuct_base, cpuct_factor, cpuct_base_at_root, cpuct_factor_at_root;
  int64_t max_depth;
  float fpu_value, fpu_value_at_root, policy_softmax_temp, draw_score, value_scale;
} cnnue_mcts_limits;
/* AzSearchLimits::default (simulations 10000, cpuct 1.5, base 19652, factor
 * 2, fpu 0.30 / 0.20 at the root, temperature 1, draw score 0, scale 1). */
void cnnue_mcts_default_limits(cnnue_mcts_limits* limits);

/* A search over many roots in lockstep: each round every tree descends to one
 * leaf and all leaves go to the GPU evaluator as one batch (trunk refresh of
 * the side to move, policy accumulator refresh, threat logits when active,
 * value head and the policy logits of the leaf's legal moves).  Replaces the
 * batch-of-four scheduler alphazero_search_batch4_reusing
 * (src/az/alphazero.rs:388-521) with AzTree's selection, expansion and
 * backup (:959-1817).  The rules engine's repetition adjudication and rule
 * history are not restated: every leaf of a tree takes its root's rule
 * context (NULL = zeros).  Host-side leaf work runs on n_threads threads
 * (<= 0: up to 16).  The model and weights must outlive the search. */
typedef struct cnnue_mcts cnnue_mcts;
int cnnue_mcts_create(const cnnue_az_model* model, const cnnue_az_weights* weights, int n_threads,
                      cnnue_mcts** out);
int cnnue_mcts_destroy(cnnue_mcts* search);
/* boards [n_roots][90], sides [n_roots], rule_context [n_roots][7] or NULL.
 * Runs limits->simulations simulations per root; *n_evaluations (optional)
 * gets the number of network evaluations (leaves) spent. */
int cnnue_mcts_search(cnnue_mcts* search, const int8_t* boards, const uint8_t* sides,
                      const float* rule_context, int64_t n_roots, const cnnue_mcts_limits* limits,
                      void* stream, uint64_t* n_evaluations);
/* Wall-clock seconds of the last search by phase: seconds[0] selection and
 * leaf preparation (legal moves, and each new leaf's network inputs:
 * features, threats, move records), [1] assembly and launch of the batches
 * (pinned host buffers, copies, kernels), [2] waiting for a batch's GPU
 * evaluation (the roots are split in two halves whose batches alternate, so
 * the GPU mostly runs while the other half is being selected), [3]
 * finalisation and backup; *rounds (optional) the number of GPU batches. */
int cnnue_mcts_stats(const cnnue_mcts* search, double* seconds, uint64_t* rounds);
/* Root statistics of the last search: per root move (from/to pairs) its
 * visits, prior and Q (root player's view), the index of the best move
 * (visits, then Q, then prior: best_root_child, src/az/alphazero.rs:
 * 1693-1716), the root's Q and visit count.  Output arrays may be NULL. */
int cnnue_mcts_result(const cnnue_mcts* search, int64_t root, uint8_t* moves, uint32_t* visits,
                      float* priors, float* q, int capacity, int* n_moves, int* best, float* root_q,
                      uint32_t* root_visits);

#ifdef __cplusplus
}
#endif
#endif /* CNNUE_H */
