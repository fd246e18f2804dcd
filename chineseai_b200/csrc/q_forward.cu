// q_forward.cu - quantised HalfKA NNUE evaluation on sm_100a.
//
// Work per position: two perspectives x (bias + ~17 gathered int16 rows of
// 2 KB), the pairwise clipped-ReLU pack to 1024 uint8, then the bucket's int8
// stack 1024->16->32->1.  The gather dominates (69.6 KB of rows per position
// against 16 K int8 MACs); the FT table (23 MB) stays resident in L2, so the
// kernel is bound by L2->SM transfer of random 2 KB rows.  On B200 plain
// 16-byte loads of such rows top out near 10 TB/s per GPU, while 1-D bulk
// copies (cp.async.bulk, the TMA engine) reach ~16 TB/s when enough warps
// issue them, so rows travel by bulk copy into shared memory:
//
//   * one CTA = 4 consumer warps evaluating one position at a time plus 4
//     producer warps; 2 CTAs per SM;
//   * the producers copy every FT row (2 KB) into a ring of 6 stages x 8
//     rows of shared memory (full/empty mbarrier pair per stage); each list
//     of rows (one perspective's active features; for the update also the
//     parent row and the removed rows) starts a fresh stage, stages are dealt
//     round-robin to the producer warps and one lane per warp issues;
//   * consumer thread t owns the 16-byte column chunk t of every row of both
//     perspectives: per stage one wait, up to 8 shared loads, int16
//     wraparound adds as native 16x2 adds (add.s16x2, one instruction per
//     word; a list's last partial stage adds only its rows), one release;
//   * the pairwise pack pairs chunk t with chunk t^64 (exchanged through
//     shared memory; clamps by min.relu.s16x2, products by dp2a); L1 = 32
//     dp4a per thread, a 16-way warp reduce-scatter and a 4-warp sum; warp 0
//     then runs L2/L3;
//   * positions are first grouped by bucket (a two-kernel counting sort) and
//     each CTA walks a contiguous slice of that order, so the current bucket's
//     16 KB of L1 weights stay in registers (16 x 8 bytes per thread).
#include <algorithm>
#include <utility>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "pipeline.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace cnnue {
namespace q {

constexpr int kF = CNNUE_Q_FEATURES;
constexpr int kCols = CNNUE_Q_COLS;
constexpr int kRowBytes = kCols * 2;
constexpr int kNB = CNNUE_Q_BUCKETS;
constexpr int kL1 = CNNUE_Q_L1;
constexpr int kL2 = CNNUE_Q_L2;
constexpr unsigned kFull = 0xffffffffu;

struct DevWeights {
  const int16_t* ft;
  const int16_t* bias;
  const int8_t* l1w;
  const int32_t* l1b;
  const int8_t* l2w;
  const int32_t* l2b;
  const int8_t* l3w;
  const int32_t* l3b;
};

// ---------------------------------------------------------------------------
// Stage 3: fused gather + pack + bucket stack.
// ---------------------------------------------------------------------------
// int16 pair arithmetic with the sm_90+ 16x2 integer instructions: add wraps
// per halfword (the FT's int16 wraparound), min.relu clamps to [0, b].
__device__ __forceinline__ uint32_t add16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.s16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t clamp16x2_0_127(uint32_t a) {
  uint32_t d;
  asm("min.relu.s16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(0x007f007fu));
  return d;
}
__device__ __forceinline__ uint4 vadd(uint4 a, uint4 b) {
  return make_uint4(add16x2(a.x, b.x), add16x2(a.y, b.y), add16x2(a.z, b.z), add16x2(a.w, b.w));
}
// a - b per halfword, as a + (~b + 1).
__device__ __forceinline__ uint4 vsub(uint4 a, uint4 b) {
  return make_uint4(add16x2(a.x, add16x2(~b.x, 0x00010001u)), add16x2(a.y, add16x2(~b.y, 0x00010001u)),
                    add16x2(a.z, add16x2(~b.z, 0x00010001u)), add16x2(a.w, add16x2(~b.w, 0x00010001u)));
}

// Four packed outputs from two words of the low half (columns j, j+1 and
// j+2, j+3) and the matching words of the high half (columns j+512 ...):
// (clamp(a,0,127) * clamp(b,0,127)) >> 7 per column, as bytes j..j+3.  Each
// product is below 2^14, so the two products of a word sit in its two
// halfwords and one 32-bit shift by 7 leaves both results in bytes 0 and 2.
__device__ __forceinline__ uint32_t pack_quad(uint32_t lo0, uint32_t hi0, uint32_t lo1, uint32_t hi1) {
  const uint32_t a0 = clamp16x2_0_127(lo0), b0 = clamp16x2_0_127(hi0);
  const uint32_t a1 = clamp16x2_0_127(lo1), b1 = clamp16x2_0_127(hi1);
  // dp2a with the clamped partner word as bytes: b = (b_lo, 0, b_hi, 0), so
  // the low dot is a_lo * b_lo and the low dot of b >> 8 is a_hi * b_hi.
  const uint32_t p0 = __dp2a_lo(a0, b0, 0u) | (__dp2a_lo(a0, b0 >> 8, 0u) << 16);
  const uint32_t p1 = __dp2a_lo(a1, b1, 0u) | (__dp2a_lo(a1, b1 >> 8, 0u) << 16);
  return __byte_perm(p0 >> 7, p1 >> 7, 0x6420);
}

struct ForwardArgs {
  DevWeights w;
  const uint16_t* idx;        // forward: active lists; update: added lists
  uint32_t n_idx;
  const uint32_t* offsets;    // [2n+1]
  const uint16_t* rem;        // update only
  uint32_t n_rem;
  const uint32_t* rem_offsets;
  const int16_t* parent;      // update only, [n][2][1024]
  const uint8_t* flags;       // update only, [2n]
  int16_t* acc_out;           // [n][2][1024] or null
  int32_t* scores;
  uint8_t* packed;            // split path: [n][1024] packed activations in sorted order
  const uint32_t* inv;        // split path: sorted slot of every position
  int natural;                // 1: walk positions in batch order (split path), 0: in sorted order
  int64_t n;
  const uint32_t* perm;
  const uint8_t* sorted_bucket;
  uint32_t* status;
  unsigned long long wait_ns;  // limit of every bounded wait
  // Test hook of the bounded waits: CTA stall_block never issues its stage
  // stall_stage (no transaction count, no copies), so the consumers' wait on
  // it runs out.  0xffffffff = off.
  uint32_t stall_block, stall_stage;
};

// ===========================================================================
// Fused evaluation kernel.  One CTA: 4 consumer warps evaluating one
// position at a time and 4 (forward) or 2 (update) producer warps that copy every FT row
// (2 KB) by cp.async.bulk into a ring of kSlots shared-memory slots, so up to
// kSlots rows per CTA are in flight without holding registers.  Every
// consumer thread t owns the 16-byte column chunk t of every row (both
// perspectives), which balances the two perspectives' row counts across the
// four warps; the pairwise pack exchanges the partner half (chunk t^64)
// through shared memory.  Bad feature indices are redirected to an all-zero
// row kept after the table.
// ===========================================================================
constexpr int kStageRows = 8;                    // rows per pipeline stage
constexpr int kStages = 6;                       // stages in the ring
constexpr int kSlots = kStages * kStageRows;     // 48 row slots, 96 KB
// Producer warps (one issuing lane each): four in the forward, whose active
// rows fill stages fast; two in the update, where every producer walking
// every position's bookkeeping costs the consumers issue slots (measured:
// 0.488 -> 0.439 ms per 65,536 updates, forward unchanged).
constexpr int kProducersEval = 4;
constexpr int kProducersUpdate = 2;
constexpr int producers_of(bool update) { return update ? kProducersUpdate : kProducersEval; }
constexpr int kPrefetch = 4;                     // positions of index lists loaded ahead
static_assert(kProducersEval <= kStages && kProducersUpdate <= kStages,
              "parity waits on the empty barriers need producers <= kStages");
constexpr int kBulkConsumers = 128;
constexpr int bulk_threads(bool update) { return kBulkConsumers + 32 * producers_of(update); }
constexpr int kBulkMinBlocks = 2;

struct BulkSmem {
  uint8_t ring[kSlots][kRowBytes];
  uint64_t full[kStages];   // completes when a stage's rows have landed
  uint64_t empty[kStages];  // completes when all consumer warps released a stage
  uint32_t issued[kStages]; // latest stage announced on full[s] (0xffffffff: none)
  uint4 xbuf[kBulkConsumers];
  int32_t red[2][4][16];
  uint8_t y1s[16];
  int abort;
};

struct Seg {
  uint32_t beg, cnt;
};

struct PosDesc {
  uint32_t pos;
  int bucket;
  uint32_t init[2];  // 1: the perspective starts from its parent row
  Seg rem[2], add[2];
};

__device__ __forceinline__ Seg clamp_seg(const uint32_t* off, int64_t i, uint32_t n) {
  const uint32_t b = min(off[i], n);
  const uint32_t e = min(max(off[i + 1], b), n);
  return Seg{b, e - b};
}

template <bool kUpdate>
__device__ __forceinline__ PosDesc load_desc(const ForwardArgs& a, int64_t i) {
  PosDesc d;
  d.pos = a.natural ? (uint32_t)i : a.perm[i];
  d.bucket = a.sorted_bucket[i];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int64_t ps = 2 * (int64_t)d.pos + p;
    d.add[p] = clamp_seg(a.offsets, ps, a.n_idx);
    if (kUpdate) {
      const bool refresh = (a.flags[ps] & 1) != 0;
      d.init[p] = refresh ? 0u : 1u;
      d.rem[p] = refresh ? Seg{0, 0} : clamp_seg(a.rem_offsets, ps, a.n_rem);
    } else {
      d.init[p] = 0;
      d.rem[p] = Seg{0, 0};
    }
  }
  return d;
}

// The consumers' descriptor of the next position, in two halves so that its
// global loads overlap a position's work: load_raw issues every load (the
// removed-list offsets unconditionally: they exist for every list), and
// finish_desc clamps as load_desc does, once the values have arrived.
struct RawDesc {
  uint32_t pos;
  int bucket;
  uint32_t o[2][2], ro[2][2];
  uint8_t fl[2];
};

template <bool kUpdate>
__device__ __forceinline__ RawDesc load_raw(const ForwardArgs& a, uint32_t pos, int bucket) {
  RawDesc r;
  r.pos = pos;
  r.bucket = bucket;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int64_t ps = 2 * (int64_t)pos + p;
    r.o[p][0] = a.offsets[ps];
    r.o[p][1] = a.offsets[ps + 1];
    if (kUpdate) {
      r.fl[p] = a.flags[ps];
      r.ro[p][0] = a.rem_offsets[ps];
      r.ro[p][1] = a.rem_offsets[ps + 1];
    }
  }
  return r;
}

template <bool kUpdate>
__device__ __forceinline__ PosDesc finish_desc(const ForwardArgs& a, const RawDesc& r) {
  PosDesc d;
  d.pos = r.pos;
  d.bucket = r.bucket;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const uint32_t b = min(r.o[p][0], a.n_idx);
    d.add[p] = Seg{b, min(max(r.o[p][1], b), a.n_idx) - b};
    if (kUpdate) {
      const bool refresh = (r.fl[p] & 1) != 0;
      d.init[p] = refresh ? 0u : 1u;
      const uint32_t rb = min(r.ro[p][0], a.n_rem);
      d.rem[p] = refresh ? Seg{0, 0} : Seg{rb, min(max(r.ro[p][1], rb), a.n_rem) - rb};
    } else {
      d.init[p] = 0;
      d.rem[p] = Seg{0, 0};
    }
  }
  return d;
}

__device__ __forceinline__ uint32_t desc_rows(const PosDesc& d) {
  return d.init[0] + d.rem[0].cnt + d.add[0].cnt + d.init[1] + d.rem[1].cnt + d.add[1].cnt;
}

// Stage layout.  Each position contributes one row sequence per perspective,
// starting on a fresh stage of at most kStageRows rows: in the forward the
// active rows; in the update the parent row (unless the perspective is
// refreshed), then the removed rows (subtracted), then the added rows - one
// sequence, so a typical update perspective (1 + 2 + 3 rows) fills a single
// stage.  int16 wraparound sums are order-free, so grouping does not change
// results.  Both sides walk stages, not rows.  Stage st lives in ring slots
// (st % kStages) * kStageRows ...; lane 0 of its producer warp performs the
// stage's barrier operations
// and bulk copies.  Stages are dealt round-robin to the producer warps (stage
// st belongs to warp st % kProducers), so consecutive stages are issued in
// parallel; one bulk copy occupies the issuing warp for ~100 cycles.  Every
// producer warp walks all positions of the CTA's slice; the index lists are
// prefetched kPrefetch positions ahead.
template <int kSR = kStageRows>
__device__ __forceinline__ uint32_t n_stages(uint32_t rows) {
  return (rows + kSR - 1) / kSR;
}

// Ring geometry: kSR rows per stage, kNS stages; Smem has ring[kSR * kNS],
// full/empty/issued[kNS] and abort.
template <int kProducers, int kSR = kStageRows, int kNS = kStages, class Smem = BulkSmem>
struct Producer {
  static_assert(kProducers <= kNS, "parity waits on the empty barriers need producers <= stages");
  Smem* sm;
  uint32_t* status;
  int w;      // producer index
  int lane;
  bool ok;    // false once a wait gave up or the CTA aborted (stop issuing)
  unsigned long long wait_ns;
  uint32_t stall_stage;  // this CTA's stage to leave unissued (test hook), or 0xffffffff

  // Lane 0: wait until stage st's slots are free (all consumer warps released
  // stage st - kNS), then announce `rows` rows on the stage's barrier.
  // Parity waits cannot alias here: this warp's previous stage was st -
  // kProducers, whose own wait already saw stage st - kProducers - kNS
  // released, and kProducers <= kNS, so the empty barrier is at most one
  // phase behind the phase waited for.
  // After an abort nothing more is announced, so every full barrier has at
  // most its latest announced phase outstanding (recorded in sm->issued for
  // the teardown drain).
  __device__ __forceinline__ bool begin_stage(uint32_t st, uint32_t rows) {
    const uint32_t sidx = st % kNS, use = st / kNS;
    if (!ok) return false;
    if (use > 0 && !pipe::mbar_wait_sleep(&sm->empty[sidx], (use - 1) & 1u, &sm->abort, status, wait_ns)) {
      ok = false;
      return false;
    }
    if (*(volatile int*)&sm->abort) {
      ok = false;
      return false;
    }
    if (st == stall_stage) return false;  // test hook: the stage stays unannounced
    pipe::mbar_arrive_expect_tx(&sm->full[sidx], rows * kRowBytes);
    sm->issued[sidx] = st;
    return true;
  }
  __device__ __forceinline__ void copy(uint32_t st, uint32_t j, const char* src) {
    const uint32_t sidx = st % kNS;
    pipe::bulk_copy_g2s(sm->ring[sidx * kSR + j], src, kRowBytes, &sm->full[sidx]);
  }

  // Issues this warp's stages among st0, st0+1, ... (the stages of list[seg]).
  // `head` holds lst[seg.beg + lane] for the first 32 entries (prefetched).
  __device__ __forceinline__ void list(const char* ft, const uint16_t* lst, Seg seg, uint32_t head,
                                       uint32_t st0) {
    const uint32_t ns = n_stages<kSR>(seg.cnt);
    uint32_t k = (uint32_t)((w - (int)(st0 % kProducers) + kProducers) % kProducers);
    for (; k < ns; k += kProducers) {
      const uint32_t st = st0 + k;
      const uint32_t first = k * kSR;
      const uint32_t rows = min((uint32_t)kSR, seg.cnt - first);
      uint32_t f = head;
      if (first >= 32) f = (uint32_t)lane < rows ? lst[seg.beg + first + lane] : 0u;
      const int src_lane0 = first >= 32 ? 0 : (int)first;
      if (f >= (uint32_t)kF) {  // bad index -> the zero row (only lanes that hold an entry)
        atomicOr(status, CNNUE_STATUS_BAD_INDEX);
        f = kF;
      }
      bool go = false;
      if (lane == 0) go = begin_stage(st, rows);
      for (uint32_t j = 0; j < rows; ++j) {
        const uint32_t fj = __shfl_sync(kFull, f, src_lane0 + (int)j);
        if (lane == 0 && go) copy(st, j, ft + (size_t)fj * kRowBytes);
      }
    }
  }

  // Update mode: the stages of one perspective's sequence [parent row if
  // init][removed rows][added rows].  `head_rem` / `head_add` hold the first
  // 32 entries of the two lists (prefetched); row r of the sequence resolves
  // lane-parallel (lane j -> row first + j).
  __device__ __forceinline__ void update_seq(const char* ft, const char* parent_row, uint32_t init,
                                             const uint16_t* rem_list, Seg rem, uint32_t head_rem,
                                             const uint16_t* add_list, Seg add, uint32_t head_add, uint32_t st0) {
    const uint32_t total = init + rem.cnt + add.cnt;
    const uint32_t ns = n_stages<kSR>(total);
    uint32_t k = (uint32_t)((w - (int)(st0 % kProducers) + kProducers) % kProducers);
    for (; k < ns; k += kProducers) {
      const uint32_t st = st0 + k;
      const uint32_t first = k * kSR;
      const uint32_t rows = min((uint32_t)kSR, total - first);
      const uint32_t r = first + (uint32_t)lane;
      const uint32_t ir = r - init;            // index into the removed list (when in range)
      const uint32_t ia = r - init - rem.cnt;  // index into the added list (when in range)
      const uint32_t hr = __shfl_sync(kFull, head_rem, (int)(ir & 31u));
      const uint32_t ha = __shfl_sync(kFull, head_add, (int)(ia & 31u));
      uint32_t f = 0, par = 0;
      if ((uint32_t)lane < rows) {
        if (r < init) {
          par = 1;
        } else if (ir < rem.cnt) {
          f = ir < 32 ? hr : rem_list[rem.beg + ir];
        } else {
          f = ia < 32 ? ha : add_list[add.beg + ia];
        }
        if (!par && f >= (uint32_t)kF) {  // bad index -> the zero row
          atomicOr(status, CNNUE_STATUS_BAD_INDEX);
          f = kF;
        }
      }
      bool go = false;
      if (lane == 0) go = begin_stage(st, rows);
      for (uint32_t j = 0; j < rows; ++j) {
        const uint32_t fj = __shfl_sync(kFull, f, (int)j);
        const uint32_t pj = __shfl_sync(kFull, par, (int)j);
        if (lane == 0 && go) copy(st, j, pj ? parent_row : ft + (size_t)fj * kRowBytes);
      }
    }
  }
};

// Consumer of an update perspective's sequence: rows [0, init) set from the
// parent (acc starts at zero then), [init, init + n_rem) subtracted, the rest
// added.  The thread's 16 bytes of every row start at col_byte.  Returns the
// next stage number.
template <int kSR = kStageRows, int kNS = kStages, class Smem = BulkSmem>
__device__ __forceinline__ uint32_t consume_update(Smem& sm, uint32_t st, uint32_t init, uint32_t n_rem,
                                                   uint32_t n_add, int col_byte, int lane, uint32_t* status,
                                                   unsigned long long wait_ns, uint4& acc) {
  const uint32_t total = init + n_rem + n_add;
  uint4 rem = make_uint4(0, 0, 0, 0);  // sum of the removed rows, subtracted once at the end
  uint32_t sidx = st % kNS, phase = (st / kNS) & 1u;
  for (uint32_t first = 0; first < total; first += kSR, ++st) {
    const uint32_t rows = min((uint32_t)kSR, total - first);
    pipe::mbar_wait_sleep(&sm.full[sidx], phase, &sm.abort, status, wait_ns);
    const uint8_t* slot = &sm.ring[sidx * kSR][col_byte];
    uint4 v[kSR];
#pragma unroll
    for (int j = 0; j < kSR; ++j)
      v[j] = (uint32_t)j < rows ? *reinterpret_cast<const uint4*>(slot + j * kRowBytes) : make_uint4(0, 0, 0, 0);
    __syncwarp();
    if (lane == 0) pipe::mbar_arrive(&sm.empty[sidx]);
#pragma unroll
    for (int j = 0; j < kSR; ++j) {
      const uint32_t r = first + (uint32_t)j;
      if (r >= init && r < init + n_rem)
        rem = vadd(rem, v[j]);
      else
        acc = vadd(acc, v[j]);
    }
    if (++sidx == (uint32_t)kNS) {
      sidx = 0;
      phase ^= 1u;
    }
  }
  acc = vsub(acc, rem);
  return st;
}

// Consumer: adds the rows of one list into acc (the thread's 16 bytes of
// every row start at col_byte).  Full stages take an unrolled tree of adds;
// the list's last, partial stage adds only its rows.  Returns the next stage
// number.
template <int kSR = kStageRows, int kNS = kStages, class Smem = BulkSmem>
__device__ __forceinline__ uint32_t consume_list(Smem& sm, uint32_t st, uint32_t cnt, int col_byte, int lane,
                                                 uint32_t* status, unsigned long long wait_ns, uint4& acc) {
  uint32_t sidx = st % kNS, phase = (st / kNS) & 1u;
  for (uint32_t first = 0; first < cnt; first += kSR, ++st) {
    const uint32_t rows = min((uint32_t)kSR, cnt - first);
    pipe::mbar_wait_sleep(&sm.full[sidx], phase, &sm.abort, status, wait_ns);
    const uint8_t* slot = &sm.ring[sidx * kSR][col_byte];
    if (rows == (uint32_t)kSR) {
      uint4 v[kSR];
#pragma unroll
      for (int j = 0; j < kSR; ++j) v[j] = *reinterpret_cast<const uint4*>(slot + j * kRowBytes);
      __syncwarp();
      if (lane == 0) pipe::mbar_arrive(&sm.empty[sidx]);
#pragma unroll
      for (int h = kSR / 2; h >= 1; h /= 2)
#pragma unroll
        for (int j = 0; j < h; ++j) v[j] = vadd(v[j], v[j + h]);
      acc = vadd(acc, v[0]);
    } else {
      // rows in [1, kSR): pairs, then a single row
      uint4 s = make_uint4(0, 0, 0, 0);
      uint32_t j = 0;
      for (; j + 2 <= rows; j += 2)
        s = vadd(s, vadd(*reinterpret_cast<const uint4*>(slot + j * kRowBytes),
                         *reinterpret_cast<const uint4*>(slot + (j + 1) * kRowBytes)));
      if (j < rows) s = vadd(s, *reinterpret_cast<const uint4*>(slot + j * kRowBytes));
      __syncwarp();
      if (lane == 0) pipe::mbar_arrive(&sm.empty[sidx]);
      acc = vadd(acc, s);
    }
    if (++sidx == (uint32_t)kNS) {
      sidx = 0;
      phase ^= 1u;
    }
  }
  return st;
}

template <int kSR = kStageRows>
__device__ __forceinline__ uint32_t desc_stages(const PosDesc& d) {
  return n_stages<kSR>(d.init[0] + d.rem[0].cnt + d.add[0].cnt) +
         n_stages<kSR>(d.init[1] + d.rem[1].cnt + d.add[1].cnt);
}

// Lane-parallel descriptor of position i (valid lanes only).
template <bool kUpdate>
__device__ __forceinline__ void lane_desc(const ForwardArgs& a, int64_t i, bool valid, PosDesc& d) {
  if (!valid) {
    d.pos = 0;
    d.bucket = 0;
    d.init[0] = d.init[1] = 0;
    d.rem[0] = d.rem[1] = d.add[0] = d.add[1] = Seg{0, 0};
    return;
  }
  d = load_desc<kUpdate>(a, i);
}

__device__ __forceinline__ Seg shfl_seg(Seg s, int src) {
  return Seg{__shfl_sync(kFull, s.beg, src), __shfl_sync(kFull, s.cnt, src)};
}

__device__ __forceinline__ PosDesc shfl_desc(const PosDesc& m, int src) {
  PosDesc d;
  d.pos = __shfl_sync(kFull, m.pos, src);
  d.bucket = 0;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    d.init[p] = __shfl_sync(kFull, m.init[p], src);
    d.rem[p] = shfl_seg(m.rem[p], src);
    d.add[p] = shfl_seg(m.add[p], src);
  }
  return d;
}

// Prefetched first 32 entries of each index list of one position.
struct ListHead {
  uint32_t rem[2], add[2];
};

template <bool kUpdate>
__device__ __forceinline__ ListHead load_heads(const ForwardArgs& a, const PosDesc& d, int lane) {
  ListHead h;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    h.add[p] = (uint32_t)lane < d.add[p].cnt ? a.idx[d.add[p].beg + lane] : 0u;
    h.rem[p] = kUpdate && (uint32_t)lane < d.rem[p].cnt ? a.rem[d.rem[p].beg + lane] : 0u;
  }
  return h;
}

// Producer warps of a CTA's slice [begin, end) of the sorted positions:
// warp w of kP walks every position, issues the stages dealt to it (stage st
// belongs to warp st % kP) and finally drains the ring.
template <bool kUpdate, int kP, int kSR, int kNS, class Smem>
__device__ __forceinline__ void produce(Smem& sm, const ForwardArgs& a, int64_t begin, int64_t end, int w,
                                        int lane) {
  Producer<kP, kSR, kNS, Smem> pr{&sm, a.status, w, lane, true, a.wait_ns,
                                 blockIdx.x == a.stall_block ? a.stall_stage : 0xffffffffu};
  const char* ft = (const char*)a.w.ft;
  const char* par_lo = (const char*)a.parent;
  uint32_t st_base = 0;  // stage number of the batch's first position
  for (int64_t b0 = begin; b0 < end; b0 += 32) {
    const int nb = (int)min((int64_t)32, end - b0);
    PosDesc mine;
    lane_desc<kUpdate>(a, b0 + lane, lane < nb, mine);
    const uint32_t my_ns = lane < nb ? desc_stages<kSR>(mine) : 0u;
    uint32_t incl = my_ns;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t x = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += x;
    }
    const uint32_t excl = incl - my_ns;
    const uint32_t batch_stages = __shfl_sync(kFull, incl, 31);
    // index-list heads of positions q .. q+3 (a rotating window)
    ListHead h0{}, h1{}, h2{}, h3{};
    if (0 < nb) h0 = load_heads<kUpdate>(a, shfl_desc(mine, 0), lane);
    if (1 < nb) h1 = load_heads<kUpdate>(a, shfl_desc(mine, 1), lane);
    if (2 < nb) h2 = load_heads<kUpdate>(a, shfl_desc(mine, 2), lane);
    if (3 < nb) h3 = load_heads<kUpdate>(a, shfl_desc(mine, 3), lane);
    for (int q = 0; q < nb; ++q) {
      const PosDesc cur = shfl_desc(mine, q);
      const ListHead head = h0;
      h0 = h1;
      h1 = h2;
      h2 = h3;
      if (q + kPrefetch < nb) h3 = load_heads<kUpdate>(a, shfl_desc(mine, q + kPrefetch), lane);
      uint32_t st = st_base + __shfl_sync(kFull, excl, q);
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        if (kUpdate) {
          pr.update_seq(ft, par_lo + (2 * (int64_t)cur.pos + p) * kRowBytes, cur.init[p], a.rem, cur.rem[p],
                        head.rem[p], a.idx, cur.add[p], head.add[p], st);
          st += n_stages<kSR>(cur.init[p] + cur.rem[p].cnt + cur.add[p].cnt);
        } else {
          pr.list(ft, a.idx, cur.add[p], head.add[p], st);
          st += n_stages<kSR>(cur.add[p].cnt);
        }
      }
    }
    st_base += batch_stages;
  }
  // Teardown: once every producer has stopped announcing stages, stay
  // resident until the latest announced stage of every ring slot has
  // landed (after an abort too; bounded), so no copy is in flight into
  // this CTA's shared memory when it ends.  Only the latest announced phase
  // of a slot can be outstanding (a slot is re-announced only after its
  // previous stage was consumed), so the parity waits are exact.
  named_bar_sync(2, 32 * kP);
  if (lane == 0) {
    for (int s = pr.w; s < kNS; s += kP) {
      const uint32_t last = sm.issued[s];
      if (last != 0xffffffffu) pipe::mbar_wait_drain(&sm.full[s], (last / kNS) & 1u, a.status);
    }
  }
  __syncwarp();
}

// Lean forward producers for the split path, which walks positions in batch
// order: per chunk of 32 positions each lane loads one position's offsets (a
// lane per position), the stage counts
// are scanned across the warp, and per position only the two lists' begin
// and length are shuffled out; a stage's row indices are read from global
// memory (lane j: row j of the stage) when the warp reaches it.  Stage st
// belongs to warp st % kP; the ring protocol and teardown are Producer's.
template <int kP, int kSR, int kNS, class Smem>
__device__ __forceinline__ void produce_forward(Smem& sm, const ForwardArgs& a, int64_t begin, int64_t end, int w,
                                                int lane) {
  Producer<kP, kSR, kNS, Smem> pr{&sm, a.status, w, lane, true, a.wait_ns,
                                 blockIdx.x == a.stall_block ? a.stall_stage : 0xffffffffu};
  const char* ft = (const char*)a.w.ft;
  uint32_t st_base = 0;  // stage number of the chunk's first position
  for (int64_t b0 = begin; b0 < end; b0 += 32) {
    const int nb = (int)min((int64_t)32, end - b0);
    Seg s0{0, 0}, s1{0, 0};
    if (lane < nb) {
      const int64_t ps = 2 * (b0 + lane);
      s0 = clamp_seg(a.offsets, ps, a.n_idx);
      s1 = clamp_seg(a.offsets, ps + 1, a.n_idx);
    }
    const uint32_t my_ns = n_stages<kSR>(s0.cnt) + n_stages<kSR>(s1.cnt);
    uint32_t incl = my_ns;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t x = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += x;
    }
    const uint32_t excl = incl - my_ns;
    const uint32_t chunk_stages = __shfl_sync(kFull, incl, 31);
    for (int q = 0; q < nb; ++q) {
      uint32_t st = st_base + __shfl_sync(kFull, excl, q);
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const uint32_t beg = __shfl_sync(kFull, p ? s1.beg : s0.beg, q);
        const uint32_t cnt = __shfl_sync(kFull, p ? s1.cnt : s0.cnt, q);
        const uint32_t ns = n_stages<kSR>(cnt);
        for (uint32_t k = (uint32_t)((w - (int)(st % kP) + kP) % kP); k < ns; k += kP) {
          const uint32_t sn = st + k, first = k * kSR;
          const uint32_t rows = min((uint32_t)kSR, cnt - first);
          uint32_t f = (uint32_t)lane < rows ? (uint32_t)a.idx[beg + first + lane] : 0u;
          if ((uint32_t)lane < rows && f >= (uint32_t)kF) {  // bad index -> the zero row
            atomicOr(a.status, CNNUE_STATUS_BAD_INDEX);
            f = kF;
          }
          bool go = false;
          if (lane == 0) go = pr.begin_stage(sn, rows);
          for (uint32_t j = 0; j < rows; ++j) {
            const uint32_t fj = __shfl_sync(kFull, f, (int)j);
            if (lane == 0 && go) pr.copy(sn, j, ft + (size_t)fj * kRowBytes);
          }
        }
        st += ns;
      }
    }
    st_base += chunk_stages;
  }
  // Teardown as in produce().
  named_bar_sync(2, 32 * kP);
  if (lane == 0) {
    for (int s = w; s < kNS; s += kP) {
      const uint32_t last = sm.issued[s];
      if (last != 0xffffffffu) pipe::mbar_wait_drain(&sm.full[s], (last / kNS) & 1u, a.status);
    }
  }
  __syncwarp();
}

// Forward producers and consumers of the gather kernel with their ring
// positions held in registers: a producer warp w issues exactly the stages
// w, w + kP, w + 2 kP, ... (stage st belongs to warp st % kP), so its slot
// and use count advance by kP per stage without a division; consumers walk
// every stage and bump their barrier and slot addresses.
template <int kP, int kSR, int kNS, class Smem>
__device__ __forceinline__ void produce_forward_fast(Smem& sm, const ForwardArgs& a, int64_t begin, int64_t end,
                                                     int w, int lane) {
  static_assert(kP <= kNS, "a producer's slot advances by kP < kNS per stage");
  const uint32_t full0 = pipe::smem_addr(&sm.full[0]), empty0 = pipe::smem_addr(&sm.empty[0]);
  const uint32_t ring0 = pipe::smem_addr(&sm.ring[0][0]);
  const char* ft = (const char*)a.w.ft;
  const uint32_t stall = blockIdx.x == a.stall_block ? a.stall_stage : 0xffffffffu;
  uint32_t s_next = (uint32_t)w;  // this warp's next stage
  uint32_t sidx = (uint32_t)w, use = 0;
  bool ok = true;
  uint32_t st_base = 0;  // stage number of the chunk's first position
  for (int64_t b0 = begin; b0 < end && ok; b0 += 32) {
    const int nb = (int)min((int64_t)32, end - b0);
    Seg s0{0, 0}, s1{0, 0};
    if (lane < nb) {
      const int64_t ps = 2 * (b0 + lane);
      s0 = clamp_seg(a.offsets, ps, a.n_idx);
      s1 = clamp_seg(a.offsets, ps + 1, a.n_idx);
    }
    const uint32_t my_ns = n_stages<kSR>(s0.cnt) + n_stages<kSR>(s1.cnt);
    uint32_t incl = my_ns;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t x = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += x;
    }
    const uint32_t excl = incl - my_ns;
    const uint32_t chunk_stages = __shfl_sync(kFull, incl, 31);
    for (int q = 0; q < nb && ok; ++q) {
      uint32_t st = st_base + __shfl_sync(kFull, excl, q);
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const uint32_t beg = __shfl_sync(kFull, p ? s1.beg : s0.beg, q);
        const uint32_t cnt = __shfl_sync(kFull, p ? s1.cnt : s0.cnt, q);
        const uint32_t st_end = st + n_stages<kSR>(cnt);
        while (ok && s_next < st_end) {
          const uint32_t first = (s_next - st) * kSR;
          const uint32_t rows = min((uint32_t)kSR, cnt - first);
          uint32_t f = (uint32_t)lane < rows ? (uint32_t)a.idx[beg + first + lane] : 0u;
          if ((uint32_t)lane < rows && f >= (uint32_t)kF) {  // bad index -> the zero row
            atomicOr(a.status, CNNUE_STATUS_BAD_INDEX);
            f = kF;
          }
          uint32_t fj[kSR];
#pragma unroll
          for (int j = 0; j < kSR; ++j) fj[j] = __shfl_sync(kFull, f, j);
          if (lane == 0) {
            bool go = use == 0 || pipe::mbar_wait_addr(empty0 + 8 * sidx, (use - 1) & 1u, &sm.abort, a.status,
                                                       a.wait_ns);
            if (go && *(volatile int*)&sm.abort) go = false;
            if (!go) {
              ok = false;
            } else if (s_next != stall) {  // the stall test hook leaves its stage unannounced
              const uint32_t bar = full0 + 8 * sidx;
              pipe::mbar_expect_tx_addr(bar, rows * kRowBytes);
              sm.issued[sidx] = s_next;
              const uint32_t dst = ring0 + sidx * (kSR * kRowBytes);
#pragma unroll
              for (int j = 0; j < kSR; ++j)
                if ((uint32_t)j < rows)
                  pipe::bulk_copy_g2s_addr(dst + j * kRowBytes, ft + ((size_t)fj[j] << 11), kRowBytes, bar);
            }
          }
          ok = __shfl_sync(kFull, ok, 0);
          s_next += kP;
          sidx += kP;
          if (sidx >= (uint32_t)kNS) {
            sidx -= kNS;
            ++use;
          }
        }
        st = st_end;
      }
    }
    st_base += chunk_stages;
  }
  // Teardown as in produce().
  named_bar_sync(2, 32 * kP);
  if (lane == 0) {
    for (int s = w; s < kNS; s += kP) {
      const uint32_t last = sm.issued[s];
      if (last != 0xffffffffu) pipe::mbar_wait_drain(&sm.full[s], (last / kNS) & 1u, a.status);
    }
  }
  __syncwarp();
}

// A consumer thread's position in the ring (addresses of the current stage).
struct ConsumerRing {
  uint32_t full, empty, slot;  // slot: this thread's 16 bytes of the stage's first row
  uint32_t sidx, phase;
};

template <int kSR, int kNS>
__device__ __forceinline__ void ring_advance(ConsumerRing& r) {
  r.full += 8;
  r.empty += 8;
  r.slot += kSR * kRowBytes;
  if (++r.sidx == (uint32_t)kNS) {
    r.sidx = 0;
    r.full -= 8 * kNS;
    r.empty -= 8 * kNS;
    r.slot -= kNS * kSR * kRowBytes;
    r.phase ^= 1u;
  }
}

// Adds the rows of one forward list into acc.
template <int kSR, int kNS>
__device__ __forceinline__ void consume_list_fast(ConsumerRing& r, volatile int* abort, uint32_t cnt, int lane,
                                                  uint32_t* status, unsigned long long wait_ns, uint4& acc) {
  static_assert((kSR & (kSR - 1)) == 0, "the tree of adds of a full stage needs a power-of-two stage");
  for (uint32_t first = 0; first < cnt; first += kSR) {
    const uint32_t rows = min((uint32_t)kSR, cnt - first);
    pipe::mbar_wait_addr(r.full, r.phase, abort, status, wait_ns);
    if (rows == (uint32_t)kSR) {
      uint4 v[kSR];
#pragma unroll
      for (int j = 0; j < kSR; ++j) v[j] = pipe::lds128(r.slot + j * kRowBytes);
      __syncwarp();
      if (lane == 0) pipe::mbar_arrive_addr(r.empty);
#pragma unroll
      for (int h = kSR / 2; h >= 1; h /= 2)
#pragma unroll
        for (int j = 0; j < h; ++j) v[j] = vadd(v[j], v[j + h]);
      acc = vadd(acc, v[0]);
    } else {
      uint4 s = pipe::lds128(r.slot);
      for (uint32_t j = 1; j < rows; ++j) s = vadd(s, pipe::lds128(r.slot + j * kRowBytes));
      __syncwarp();
      if (lane == 0) pipe::mbar_arrive_addr(r.empty);
      acc = vadd(acc, s);
    }
    ring_advance<kSR, kNS>(r);
  }
}

// Adds the rows of one forward list into two accumulators: the thread's
// 16 bytes of every row at the ring slot (column chunk c) and 1 KB further
// (chunk c + 64, its pack partner).
template <int kSR, int kNS>
__device__ __forceinline__ void consume_list_fast2(ConsumerRing& r, volatile int* abort, uint32_t cnt, int lane,
                                                   uint32_t* status, unsigned long long wait_ns, uint4& acc_lo,
                                                   uint4& acc_hi) {
  static_assert((kSR & (kSR - 1)) == 0, "the tree of adds of a full stage needs a power-of-two stage");
  for (uint32_t first = 0; first < cnt; first += kSR) {
    const uint32_t rows = min((uint32_t)kSR, cnt - first);
    pipe::mbar_wait_addr(r.full, r.phase, abort, status, wait_ns);
    if (rows == (uint32_t)kSR) {
      uint4 v[kSR];
#pragma unroll
      for (int j = 0; j < kSR; ++j) v[j] = pipe::lds128(r.slot + j * kRowBytes);
#pragma unroll
      for (int h = kSR / 2; h >= 1; h /= 2)
#pragma unroll
        for (int j = 0; j < h; ++j) v[j] = vadd(v[j], v[j + h]);
      acc_lo = vadd(acc_lo, v[0]);
#pragma unroll
      for (int j = 0; j < kSR; ++j) v[j] = pipe::lds128(r.slot + 1024 + j * kRowBytes);
      __syncwarp();
      if (lane == 0) pipe::mbar_arrive_addr(r.empty);
#pragma unroll
      for (int h = kSR / 2; h >= 1; h /= 2)
#pragma unroll
        for (int j = 0; j < h; ++j) v[j] = vadd(v[j], v[j + h]);
      acc_hi = vadd(acc_hi, v[0]);
    } else {
      uint4 s = pipe::lds128(r.slot), t = pipe::lds128(r.slot + 1024);
      for (uint32_t j = 1; j < rows; ++j) {
        s = vadd(s, pipe::lds128(r.slot + j * kRowBytes));
        t = vadd(t, pipe::lds128(r.slot + 1024 + j * kRowBytes));
      }
      __syncwarp();
      if (lane == 0) pipe::mbar_arrive_addr(r.empty);
      acc_lo = vadd(acc_lo, s);
      acc_hi = vadd(acc_hi, t);
    }
    ring_advance<kSR, kNS>(r);
  }
}

template <bool kUpdate, bool kWriteAcc>
__global__ void __launch_bounds__(bulk_threads(kUpdate), kBulkMinBlocks) q_bulk_kernel(const ForwardArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  BulkSmem& sm = *reinterpret_cast<BulkSmem*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      pipe::mbar_init(&sm.full[s], 1);
      pipe::mbar_init(&sm.empty[s], kBulkConsumers / 32);
      sm.issued[s] = 0xffffffffu;
    }
    sm.abort = 0;
    pipe::mbar_init_fence();
  }
  __syncthreads();

  const int64_t begin = a.n * blockIdx.x / gridDim.x;
  const int64_t end = a.n * (blockIdx.x + 1) / gridDim.x;

  if (warp >= kBulkConsumers / 32) {
    produce<kUpdate, producers_of(kUpdate), kStageRows, kStages>(sm, a, begin, end, warp - kBulkConsumers / 32,
                                                                 lane);
    return;
  }

  // -------------------------------- consumers ------------------------------
  const int t = threadIdx.x;  // chunk t: columns [8t, 8t+8) of every row
  const uint4 bias = __ldg((const uint4*)((const char*)a.w.bias + t * 16));
  int cur_bucket = -1;
  uint2 w1[kL1];
  uint4 w2row = make_uint4(0, 0, 0, 0);
  int32_t b1v = 0, b2v = 0, w3v = 0, b3v = 0;
  int parity = 0;
  uint32_t st = 0;  // next stage number
  PosDesc nxt;
  if (begin < end) nxt = load_desc<kUpdate>(a, begin);
  // position and bucket of the position after the next (loaded an iteration
  // before its descriptor loads need them)
  uint32_t pos_n = begin + 1 < end ? a.perm[begin + 1] : 0u;
  int bucket_n = begin + 1 < end ? (int)a.sorted_bucket[begin + 1] : 0;

  for (int64_t i = begin; i < end; ++i) {
    const PosDesc d = nxt;
    const bool has_next = i + 1 < end;
    RawDesc raw;
    if (has_next) raw = load_raw<kUpdate>(a, pos_n, bucket_n);
    if (i + 2 < end) {
      pos_n = a.perm[i + 2];
      bucket_n = (int)a.sorted_bucket[i + 2];
    }
    if (d.bucket != cur_bucket) {
      cur_bucket = d.bucket;
      const int8_t* w1p = a.w.l1w + (size_t)d.bucket * kL1 * kCols + 8 * t;
#pragma unroll
      for (int k = 0; k < kL1; ++k) w1[k] = __ldg((const uint2*)(w1p + (size_t)k * kCols));
      w2row = __ldg((const uint4*)(a.w.l2w + ((size_t)d.bucket * kL2 + lane) * kL1));
      b2v = __ldg(a.w.l2b + d.bucket * kL2 + lane);
      w3v = __ldg(a.w.l3w + d.bucket * kL2 + lane);
      b1v = lane < kL1 ? __ldg(a.w.l1b + d.bucket * kL1 + lane) : 0;
      b3v = __ldg(a.w.l3b + d.bucket);
    }

    uint4 acc[2];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      uint4 v = bias;
      if (kUpdate) {
        if (d.init[p]) v = make_uint4(0, 0, 0, 0);  // the parent row replaces the bias
        st = consume_update(sm, st, d.init[p], d.rem[p].cnt, d.add[p].cnt, t * 16, lane, a.status, a.wait_ns, v);
      } else {
        st = consume_list(sm, st, d.add[p].cnt, t * 16, lane, a.status, a.wait_ns, v);
      }
      acc[p] = v;
    }
    if (kWriteAcc) {
      *(uint4*)((char*)(a.acc_out + (2 * (int64_t)d.pos) * kCols) + t * 16) = acc[0];
      *(uint4*)((char*)(a.acc_out + (2 * (int64_t)d.pos + 1) * kCols) + t * 16) = acc[1];
    }

    // ---- pairwise pack: chunk t pairs with chunk t ^ 64 ----------------------
    const bool lo = t < 64;
    sm.xbuf[t] = lo ? acc[1] : acc[0];
    named_bar_sync(1, kBulkConsumers);
    const uint4 other = sm.xbuf[t ^ 64];
    const uint4 plo = lo ? acc[0] : other;  // columns j   of the packed perspective
    const uint4 phi = lo ? other : acc[1];  // columns j+512
    const uint32_t x0 = pack_quad(plo.x, phi.x, plo.y, phi.y);
    const uint32_t x1 = pack_quad(plo.z, phi.z, plo.w, phi.w);

    int32_t v[kL1];
#pragma unroll
    for (int k = 0; k < kL1; ++k) v[k] = __dp4a((int)x1, (int)w1[k].y, __dp4a((int)x0, (int)w1[k].x, 0));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const bool up = lane & 16;
      const int32_t send = up ? v[j] : v[j + 8];
      const int32_t keep = up ? v[j + 8] : v[j];
      v[j] = keep + __shfl_xor_sync(kFull, send, 16);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool up = lane & 8;
      const int32_t send = up ? v[j] : v[j + 4];
      const int32_t keep = up ? v[j + 4] : v[j];
      v[j] = keep + __shfl_xor_sync(kFull, send, 8);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const bool up = lane & 4;
      const int32_t send = up ? v[j] : v[j + 2];
      const int32_t keep = up ? v[j + 2] : v[j];
      v[j] = keep + __shfl_xor_sync(kFull, send, 4);
    }
    {
      const bool up = lane & 2;
      const int32_t send = up ? v[0] : v[1];
      const int32_t keep = up ? v[1] : v[0];
      v[0] = keep + __shfl_xor_sync(kFull, send, 2);
    }
    v[0] += __shfl_xor_sync(kFull, v[0], 1);
    if ((lane & 1) == 0) sm.red[parity][warp][lane >> 1] = v[0];
    named_bar_sync(1, kBulkConsumers);

    if (warp == 0) {
      if (lane < kL1) {
        const int32_t s = b1v + sm.red[parity][0][lane] + sm.red[parity][1][lane] +
                          sm.red[parity][2][lane] + sm.red[parity][3][lane];
        sm.y1s[lane] = (uint8_t)min(max(s >> 6, 0), 127);
      }
      __syncwarp();
      const uint4 y = *(const uint4*)sm.y1s;
      int32_t s2 = b2v;
      s2 = __dp4a((int)y.x, (int)w2row.x, s2);
      s2 = __dp4a((int)y.y, (int)w2row.y, s2);
      s2 = __dp4a((int)y.z, (int)w2row.z, s2);
      s2 = __dp4a((int)y.w, (int)w2row.w, s2);
      const int32_t y2 = min(max(s2 >> 6, 0), 127);
      int32_t s3 = (int32_t)(int8_t)w3v * y2;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s3 += __shfl_xor_sync(kFull, s3, o);
      if (lane == 0) a.scores[d.pos] = b3v + s3;
      __syncwarp();
    }
    parity ^= 1;
    if (has_next) nxt = finish_desc<kUpdate>(a, raw);
  }
}


// ===========================================================================
// Split evaluation, kernel 1 of 2: gather + pack.  Same ring protocol as the
// fused kernel, on 3 stages x 8 rows per CTA, 4 CTAs per SM and 3 producer
// warps.  Every consumer warp waits on and releases every stage, so the ring's
// handshakes cost instruction issue per stage: 8-row stages halve them per
// row, and the forward runs two consumer warps whose lanes own two 16-byte
// chunks of every row (gather_forward_consumer; 331 -> 312 us per 65,536
// positions), the update four.  Measured per 65,536 positions with the L2 flushed (forward incl. the
// bucket sort and stacks / update): 4 x 6 rows, 4 CTAs, 4 producers 358.5 /
// 295.6 us; 8 x 3, 4, 3: 329.6 / 295.1 us; 8 x 3, 3, 3: 327.7 / 316.0 us;
// 8 x 4, 3, 4: 334.1 / 302.9 us; 8 x 3, 4, 2: 389.9 / 294.0 us; 16-row
// stages 453-455 / 518-592 us.  (Among 4-row rings, 12 x 4 with 2 CTAs per
// SM, 8 x 4 with 3 and 4 x 4 with 5 were slower than 6 x 4 with 4.)  In the
// update, the four consumer warps own the 16-byte column chunks so that a
// chunk's pack partner (columns j and j + 512) sits in the same warp: lane
// l < 16 of warp w owns chunk 16w + l, lane l + 16 owns chunk 64 + 16w + l.
// After a position's two perspectives are summed, partner lanes swap one
// perspective's chunk with a single 16-byte shuffle exchange, lane l < 16
// packs perspective 0 and lane l + 16 perspective 1, and each lane stores its
// 8 packed bytes (in the forward a lane holds both chunks of a pair and packs
// both perspectives itself): 1024 uint8 per position, written at the
// position's sorted slot.  The CTAs walk positions in batch order (a CTA's index lists are
// contiguous, which the producers' per-stage index loads find in L1; the
// sorted order scatters them and measured ~110 us slower per 65,536).  No
// barrier joins the consumer warps; the bucket stacks run in kernel 2 over
// the packed rows.
// ===========================================================================
constexpr int kGRows = 8;
constexpr int kGStages = 3;
constexpr int kGMinBlocks = 4;  // CTAs per SM (ring 48 KB each)
constexpr int kGProducersEval = 3;
constexpr int kGProducersUpdate = 2;
constexpr int gproducers_of(bool update) { return update ? kGProducersUpdate : kGProducersEval; }
// consumer warps: two in the forward (lane l of warp w owns column chunks
// 32w + l and its pack partner 32w + l + 64), four in the update
constexpr int gconsumers_of(bool update) { return update ? 4 : 2; }
constexpr int gather_threads(bool update) { return 32 * gconsumers_of(update) + 32 * gproducers_of(update); }

struct GatherSmem {
  uint8_t ring[kGRows * kGStages][kRowBytes];
  uint64_t full[kGStages];
  uint64_t empty[kGStages];
  uint32_t issued[kGStages];
  int abort;
};

// Forward consumers of the gather (two warps): lane l of warp w owns column
// chunk c = 32w + l (columns [8c, 8c + 8)) and its pack partner c + 64
// (columns j + 512) of every row, so each stage costs a warp one wait and one
// release for 2 x 8 rows of 16 bytes, and the pack needs no exchange: lane l
// packs both perspectives of chunk c and stores 8 bytes of each.
template <bool kWriteAcc>
__device__ __forceinline__ void gather_forward_consumer(GatherSmem& sm, const ForwardArgs& a, int64_t begin,
                                                        int64_t end, int warp, int lane) {
  const int c = 32 * warp + lane;
  const uint4 bias_lo = __ldg((const uint4*)((const char*)a.w.bias + c * 16));
  const uint4 bias_hi = __ldg((const uint4*)((const char*)a.w.bias + (c + 64) * 16));
  ConsumerRing ring{pipe::smem_addr(&sm.full[0]), pipe::smem_addr(&sm.empty[0]),
                    pipe::smem_addr(&sm.ring[0][0]) + (uint32_t)(c * 16), 0u, 0u};
  PosDesc nxt;
  if (begin < end) nxt = finish_desc<false>(a, load_raw<false>(a, (uint32_t)begin, 0));
  // launched as a programmatic dependent of the bucket sort's scatter: the
  // inverse order (written by it) is complete and visible only after this
  // wait; the producers read only the batch's lists and never wait
  asm volatile("griddepcontrol.wait;" ::: "memory");
  uint32_t slot_n = begin < end ? a.inv[begin] : 0u;  // sorted slot of the next position
  for (int64_t i = begin; i < end; ++i) {
    const PosDesc d = nxt;
    const uint32_t slot = slot_n;
    const bool has_next = i + 1 < end;
    RawDesc raw;
    if (has_next) {
      raw = load_raw<false>(a, (uint32_t)(i + 1), 0);
      slot_n = a.inv[i + 1];
    }
    uint4 lo[2], hi[2];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      lo[p] = bias_lo;
      hi[p] = bias_hi;
      consume_list_fast2<kGRows, kGStages>(ring, &sm.abort, d.add[p].cnt, lane, a.status, a.wait_ns, lo[p], hi[p]);
    }
    if (kWriteAcc) {
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        char* row = (char*)(a.acc_out + (2 * (int64_t)d.pos + p) * kCols);
        *(uint4*)(row + c * 16) = lo[p];
        *(uint4*)(row + (c + 64) * 16) = hi[p];
      }
    }
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      uint2 out;
      out.x = pack_quad(lo[p].x, hi[p].x, lo[p].y, hi[p].y);
      out.y = pack_quad(lo[p].z, hi[p].z, lo[p].w, hi[p].w);
      *(uint2*)(a.packed + (size_t)slot * CNNUE_Q_PACKED + (p ? CNNUE_Q_HALF : 0) + 8 * c) = out;
    }
    if (has_next) nxt = finish_desc<false>(a, raw);
  }
}

template <bool kUpdate, bool kWriteAcc>
__global__ void __launch_bounds__(gather_threads(kUpdate), kGMinBlocks) q_gather_kernel(const ForwardArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  GatherSmem& sm = *reinterpret_cast<GatherSmem*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the stack kernel may be scheduled once every CTA of this grid is running:
  // it sets up, then waits for this grid's packed rows
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGStages; ++s) {
      pipe::mbar_init(&sm.full[s], 1);
      pipe::mbar_init(&sm.empty[s], gconsumers_of(kUpdate));
      sm.issued[s] = 0xffffffffu;
    }
    sm.abort = 0;
    pipe::mbar_init_fence();
  }
  __syncthreads();

  const int64_t begin = a.n * blockIdx.x / gridDim.x;
  const int64_t end = a.n * (blockIdx.x + 1) / gridDim.x;

  if (warp >= gconsumers_of(kUpdate)) {
    if (kUpdate)
      produce<true, gproducers_of(kUpdate), kGRows, kGStages>(sm, a, begin, end, warp - gconsumers_of(kUpdate), lane);
    else
      produce_forward_fast<gproducers_of(kUpdate), kGRows, kGStages>(sm, a, begin, end, warp - gconsumers_of(kUpdate),
                                                                     lane);
    return;
  }
  if (!kUpdate) {
    gather_forward_consumer<kWriteAcc>(sm, a, begin, end, warp, lane);
    return;
  }

  // -------------------------------- consumers ------------------------------
  const bool lo = lane < 16;
  const int sub = lane & 15;
  const int chunk = lo ? 16 * warp + sub : 64 + 16 * warp + sub;  // columns [8 chunk, 8 chunk + 8)
  const int col_byte = chunk * 16;
  const uint4 bias = __ldg((const uint4*)((const char*)a.w.bias + col_byte));
  uint32_t st = 0;  // next stage number (update path)
  ConsumerRing ring{pipe::smem_addr(&sm.full[0]), pipe::smem_addr(&sm.empty[0]),
                    pipe::smem_addr(&sm.ring[0][0]) + (uint32_t)col_byte, 0u, 0u};
  PosDesc nxt;
  if (begin < end) nxt = finish_desc<kUpdate>(a, load_raw<kUpdate>(a, (uint32_t)begin, 0));
  // launched as a programmatic dependent of the bucket sort's scatter: the
  // inverse order (written by it) is complete and visible only after this
  // wait; the producers read only the batch's lists and never wait
  asm volatile("griddepcontrol.wait;" ::: "memory");
  uint32_t slot_n = begin < end ? a.inv[begin] : 0u;  // sorted slot of the next position

  for (int64_t i = begin; i < end; ++i) {
    const PosDesc d = nxt;
    const uint32_t slot = slot_n;
    const bool has_next = i + 1 < end;
    RawDesc raw;
    if (has_next) {
      raw = load_raw<kUpdate>(a, (uint32_t)(i + 1), 0);
      slot_n = a.inv[i + 1];
    }

    uint4 acc[2];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      uint4 v = bias;
      if (kUpdate) {
        if (d.init[p]) v = make_uint4(0, 0, 0, 0);  // the parent row replaces the bias
        st = consume_update<kGRows, kGStages>(sm, st, d.init[p], d.rem[p].cnt, d.add[p].cnt, col_byte, lane,
                                              a.status, a.wait_ns, v);
      } else {
        consume_list_fast<kGRows, kGStages>(ring, &sm.abort, d.add[p].cnt, lane, a.status, a.wait_ns, v);
      }
      acc[p] = v;
    }
    if (kWriteAcc) {
      *(uint4*)((char*)(a.acc_out + (2 * (int64_t)d.pos) * kCols) + col_byte) = acc[0];
      *(uint4*)((char*)(a.acc_out + (2 * (int64_t)d.pos + 1) * kCols) + col_byte) = acc[1];
    }
    // lane l < 16 keeps perspective 0's low chunk and takes its high partner;
    // lane l + 16 keeps perspective 1's high chunk and takes its low partner
    const uint4 give = lo ? acc[1] : acc[0];
    uint4 take;
    take.x = __shfl_xor_sync(kFull, give.x, 16);
    take.y = __shfl_xor_sync(kFull, give.y, 16);
    take.z = __shfl_xor_sync(kFull, give.z, 16);
    take.w = __shfl_xor_sync(kFull, give.w, 16);
    const uint4 plo = lo ? acc[0] : take;  // columns j of the packed perspective
    const uint4 phi = lo ? take : acc[1];  // columns j + 512
    uint2 out;
    out.x = pack_quad(plo.x, phi.x, plo.y, phi.y);
    out.y = pack_quad(plo.z, phi.z, plo.w, phi.w);
    *(uint2*)(a.packed + (size_t)slot * CNNUE_Q_PACKED + (lo ? 0 : CNNUE_Q_HALF) + 8 * (16 * warp + sub)) = out;
    if (has_next) nxt = finish_desc<kUpdate>(a, raw);
  }
}

constexpr int kStackTile = 128;  // rows of one bucket per stack tile

// ===========================================================================
// Split evaluation, kernel 2 of 2 (tensor cores): the bucket stacks over the
// packed rows.  L1 of a tile of 128 rows of one bucket is the bucket GEMM
// D[128 x 16] = X[128 x 1024] (uint8) . W1[16 x 1024]^T (int8) on tcgen05
// (kind::i8, int32 accumulator in TMEM): X arrives by 2-D TMA in 128-byte K
// chunks (128B swizzle) through a 2-stage ring, W1 by one bulk copy of the
// bucket's pre-tiled weights.  Warps 0-3 then read their rows' 16 sums from
// TMEM (lane = row) and run the L1 activation, L2 and L3 in registers.
// Warp 4 loads (and owns TMEM), warp 5 issues the MMAs.  Two stages (about
// 50 KB of shared memory) let 4 CTAs share an SM, so the ~530 tiles of a
// 65,536-position batch run in one wave: 4 us less per forward and per update
// than with 4 stages (2 CTAs per SM), 3 stages in between.
// ===========================================================================
constexpr int kTcStages = 2;
constexpr int kTcChunk = 128;                          // K bytes per stage
constexpr int kTcChunks = CNNUE_Q_PACKED / kTcChunk;   // 8
constexpr int kTcThreads = 192;
constexpr int kTcTileBytes = kStackTile * kTcChunk;    // 16 KB
constexpr int kTcWTileBytes = kL1 * kTcChunk;          // 2 KB

struct StackTcSmem {
  alignas(1024) uint8_t a[kTcStages][kTcTileBytes];
  alignas(1024) uint8_t b[kTcChunks][kTcWTileBytes];
  uint64_t loaded[kTcStages];
  uint64_t empty[kTcStages];
  uint64_t wload;
  uint64_t accum;
  uint64_t drain;
  alignas(16) int8_t w2[kL2][kL1];  // read and written as 16-byte rows
  int32_t b2[kL2];
  int32_t b1[kL1];
  int8_t w3[kL2];
  uint32_t tmem_base;
  int bucket, start, count;
  int abort;
};

// Byte offset of (row, k) of a K-chunk tile (rows of 128 bytes, 128B swizzle:
// the 16-byte chunk c of row r sits at chunk position c ^ (r % 8)).
__host__ __device__ constexpr uint32_t sw128_offset(int row, int k) {
  return (uint32_t)(row * 128 + ((((k >> 4) ^ row) & 7) << 4) + (k & 15));
}

__global__ void __launch_bounds__(kTcThreads) q_stack_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                                const ForwardArgs a, const uint8_t* w1tiles,
                                                                const WorkspaceHeader* hdr) {
  extern __shared__ uint8_t smem_raw[];
  StackTcSmem& sm =
      *reinterpret_cast<StackTcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    // tile blockIdx.x among the buckets' tiles, in bucket order
    uint32_t g = blockIdx.x;
    sm.bucket = -1;
    for (int b = 0; b < kNB; ++b) {
      const uint32_t c = hdr->counts[b];
      const uint32_t tiles = (c + kStackTile - 1) / kStackTile;
      if (g < tiles) {
        sm.bucket = b;
        sm.start = (int)(hdr->cursors[b] + g * kStackTile);
        sm.count = (int)min((uint32_t)kStackTile, c - g * kStackTile);
        break;
      }
      g -= tiles;
    }
    for (int s = 0; s < kTcStages; ++s) {
      pipe::mbar_init(&sm.loaded[s], 1);
      pipe::mbar_init(&sm.empty[s], 1);
    }
    pipe::mbar_init(&sm.wload, 1);
    pipe::mbar_init(&sm.accum, 1);
    pipe::mbar_init(&sm.drain, 1);
    sm.abort = 0;
    pipe::mbar_init_fence();
  }
  __syncthreads();
  const int b = sm.bucket;
  if (b < 0) return;  // past the last tile (uniform across the CTA; no TMEM held yet)
  if (warp == 4) {
    tc::tmem_alloc(pipe::smem_addr(&sm.tmem_base), 32);
    tc::tmem_relinquish();
  }
  if (tid < kL2 * kL1 / 16) ((uint4*)&sm.w2[0][0])[tid] = __ldg((const uint4*)(a.w.l2w + (size_t)b * kL2 * kL1) + tid);
  if (tid < kL2) {
    sm.b2[tid] = __ldg(a.w.l2b + b * kL2 + tid);
    sm.w3[tid] = __ldg(a.w.l3w + b * kL2 + tid);
  }
  if (tid < kL1) sm.b1[tid] = __ldg(a.w.l1b + b * kL1 + tid);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  // launched as a programmatic dependent of the gather: its packed rows are
  // complete and visible only after this wait (the set-up above reads only
  // weights and the sort's bucket counts, done before the gather began)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const uint32_t tmem = sm.tmem_base;
  const int start = sm.start, count = sm.count;

  if (warp < 4) {
    // ---- epilogue: TMEM lane = row of the tile.
    const bool ok = pipe::mbar_wait(&sm.accum, 0, &sm.abort, a.status, a.wait_ns);
    tc::fence_after_sync();
    uint32_t v[16];
    __syncwarp();
    tc::tmem_ld16(tmem + ((uint32_t)(32 * warp) << 16), v);
    tc::wait_ld();
    const int t = tid;
    if (ok && t < count) {
      uint32_t y1[4] = {0, 0, 0, 0};
#pragma unroll
      for (int o = 0; o < kL1; ++o) {
        const uint32_t y = (uint32_t)min(max(((int32_t)v[o] + sm.b1[o]) >> 6, 0), 127);
        y1[o >> 2] |= y << (8 * (o & 3));
      }
      int32_t s3 = 0;
#pragma unroll 8
      for (int j = 0; j < kL2; ++j) {
        const uint4 wv = *(const uint4*)&sm.w2[j][0];
        int32_t s2 = sm.b2[j];
        s2 = __dp4a((int)y1[0], (int)wv.x, s2);
        s2 = __dp4a((int)y1[1], (int)wv.y, s2);
        s2 = __dp4a((int)y1[2], (int)wv.z, s2);
        s2 = __dp4a((int)y1[3], (int)wv.w, s2);
        s3 += (int32_t)sm.w3[j] * min(max(s2 >> 6, 0), 127);
      }
      a.scores[a.perm[start + t]] = __ldg(a.w.l3b + b) + s3;
    }
  } else if (warp == 4) {
    // ---- loads: the bucket's W1 tiles once, then X chunk by chunk.
    if (lane == 0) {
      pipe::mbar_arrive_expect_tx(&sm.wload, kTcChunks * kTcWTileBytes);
      pipe::bulk_copy_g2s(&sm.b[0][0], w1tiles + (size_t)b * kTcChunks * kTcWTileBytes, kTcChunks * kTcWTileBytes,
                          &sm.wload);
      int issued = 0;
      for (int kc = 0; kc < kTcChunks; ++kc) {
        const int s = kc % kTcStages, u = kc / kTcStages;
        if (u > 0 && !pipe::mbar_wait(&sm.empty[s], (u - 1) & 1, &sm.abort, a.status, a.wait_ns)) break;
        pipe::mbar_arrive_expect_tx(&sm.loaded[s], kTcTileBytes);
        tc::tma_load_2d(pipe::smem_addr(sm.a[s]), &tmap_x, kc * kTcChunk, start, pipe::smem_addr(&sm.loaded[s]));
        ++issued;
      }
      // after an abort: let the copies in flight land before the CTA ends
      if (sm.abort) {
        pipe::mbar_wait_drain(&sm.wload, 0, a.status);
        for (int kc = max(0, issued - kTcStages); kc < issued; ++kc)
          pipe::mbar_wait_drain(&sm.loaded[kc % kTcStages], (kc / kTcStages) & 1, a.status);
      }
    }
    __syncwarp();
  } else {
    // ---- MMA issuer.
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_u8s8_s32(kStackTile, kL1);
      bool ok = pipe::mbar_wait(&sm.wload, 0, &sm.abort, a.status, a.wait_ns);
      for (int kc = 0; ok && kc < kTcChunks; ++kc) {
        const int s = kc % kTcStages, u = kc / kTcStages;
        if (!pipe::mbar_wait(&sm.loaded[s], u & 1, &sm.abort, a.status, a.wait_ns)) break;
        tc::fence_after_sync();
        const uint32_t a0 = pipe::smem_addr(sm.a[s]), b0 = pipe::smem_addr(sm.b[kc]);
#pragma unroll
        for (int kk = 0; kk < kTcChunk / 32; ++kk) {
          const uint64_t ad = tc::smem_desc(a0 + kk * 32, 0, 1024, tc::kSwizzle128B);
          const uint64_t bd = tc::smem_desc(b0 + kk * 32, 0, 1024, tc::kSwizzle128B);
          tc::mma_i8(tmem, ad, bd, idesc, (kc | kk) != 0 ? 1u : 0u);
        }
        tc::commit(pipe::smem_addr(&sm.empty[s]));
      }
      tc::commit(pipe::smem_addr(&sm.accum));
      // every MMA issued has completed before TMEM is freed
      tc::commit(pipe::smem_addr(&sm.drain));
      pipe::mbar_wait_drain(&sm.drain, 0, a.status);
    }
    __syncwarp();
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 4) tc::tmem_dealloc(tmem, 32);
}

}  // namespace q
}  // namespace cnnue

// ===========================================================================
// Host side
// ===========================================================================
using namespace cnnue;
using namespace cnnue::q;

struct cnnue_q_model {
  int device = 0;
  DevWeights w{};
  void* blob = nullptr;
  int sm_count = 0;
  uint8_t* w1tiles = nullptr;  // [16 buckets][8 K chunks][16 rows x 128 B], 128B-swizzled (tensor-core B)
  int grid_eval = 0;     // fused kernel (the no-allocation entry point)
  int grid_gather = 0;   // split path, forward
  int grid_gather_update = 0;
  // Staging for cnnue_q_forward_host.
  void* stage = nullptr;
  size_t stage_bytes = 0;
};

namespace {

int check_launch(const char* what) { return check_launch_error(what); }

// Workspace of the split path: the bucket-sort workspace, then the packed
// activations [n][1024] uint8 in sorted order, then the sorted slot of every
// position [n] uint32.
size_t packed_offset(int64_t n) { return align_up(bucket_workspace_bytes(n), 256); }
size_t inv_offset(int64_t n) { return packed_offset(n) + align_up((size_t)(n > 0 ? n : 0) * CNNUE_Q_PACKED, 256); }
size_t q_workspace_bytes(int64_t n) { return inv_offset(n) + align_up((size_t)(n > 0 ? n : 0) * 4, 256); }
uint32_t* ws_inv(void* ws, int64_t n) { return (uint32_t*)((char*)ws + inv_offset(n)); }

int validate_common(const cnnue_q_model* m, int64_t n, void* ws, size_t ws_bytes) {
  if (!m) return set_error(CNNUE_ERR_INVALID_ARG, "model is null");
  if (n < 0 || n > (int64_t)INT32_MAX)
    return set_error(CNNUE_ERR_INVALID_ARG, "n_positions %lld out of range", (long long)n);
  if (n > 0 && !ws) return set_error(CNNUE_ERR_INVALID_ARG, "workspace is null");
  if (((uintptr_t)ws & 255u) != 0) return set_error(CNNUE_ERR_INVALID_ARG, "workspace must be 256-byte aligned");
  if (n > 0 && ws_bytes < q_workspace_bytes(n))
    return set_error(CNNUE_ERR_WORKSPACE, "workspace %zu bytes < %zu required", ws_bytes,
                     q_workspace_bytes(n));
  return CNNUE_OK;
}

int launch_sort(const cnnue_q_model* m, const uint32_t* d_offsets, uint32_t n_indices,
                const uint8_t* d_count0, int64_t n, void* ws, cudaStream_t s, uint32_t* inv,
                const uint32_t* d_extra0 = nullptr, uint32_t n_extra0 = 0, const uint32_t* d_extra1 = nullptr,
                uint32_t n_extra1 = 0) {
  (void)m;
  return launch_bucket_sort(d_offsets, n_indices, d_count0, n, 1, kNB, ws, s, inv, d_extra0, n_extra0, d_extra1,
                            n_extra1);
}

// Arguments with the default wait limit and the stall hook off.
ForwardArgs base_args() {
  ForwardArgs a{};
  a.wait_ns = pipe::kWaitLimitNs;
  a.stall_block = 0xffffffffu;
  a.stall_stage = 0xffffffffu;
  return a;
}

size_t stack_tc_smem_bytes() { return sizeof(StackTcSmem) + 1024; }

// Launches `kernel` as a programmatic dependent of the stream's previous
// kernel: it may be scheduled while that one finishes, and waits for it with
// griddepcontrol.wait before reading its results.
template <typename... KArgs, typename... Args>
int launch_dependent(const char* what, void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem,
                     cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) return cuda_error(e, what);
  return check_launch(what);
}

// The bucket stacks of the split path over the packed rows (tensor cores).
int launch_stack(const cnnue_q_model* m, const ForwardArgs& a, const WorkspaceView& v, cudaStream_t s) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = tma_encode_fn();
  if (!fn) return set_error(CNNUE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)CNNUE_Q_PACKED, (cuuint64_t)a.n};
  const cuuint64_t strides[1] = {(cuuint64_t)CNNUE_Q_PACKED};
  const cuuint32_t box[2] = {(cuuint32_t)kTcChunk, (cuuint32_t)kStackTile};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a.packed, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(CNNUE_ERR_CUDA, "cuTensorMapEncodeTiled(packed rows) failed (%d)", (int)r);
  const int64_t tiles = (a.n + kStackTile - 1) / kStackTile + kNB;  // bound on the buckets' tiles
  return launch_dependent("q_stack_tc_kernel", q_stack_tc_kernel, (unsigned)tiles, kTcThreads, stack_tc_smem_bytes(),
                          s, map, a, (const uint8_t*)m->w1tiles, (const WorkspaceHeader*)v.hdr);
}

// Forward over the sorted order (split path): gather + pack, then the stacks.
int launch_eval(const cnnue_q_model* m, const uint16_t* d_idx, uint32_t n_idx,
                const uint32_t* d_offsets, int64_t n, int32_t* d_scores, int16_t* d_acc, void* ws,
                cudaStream_t s, const ForwardArgs& hooks = base_args()) {
  WorkspaceView v = carve_workspace(ws, n);
  ForwardArgs a = hooks;
  a.w = m->w;
  a.idx = d_idx;
  a.n_idx = n_idx;
  a.offsets = d_offsets;
  a.acc_out = d_acc;
  a.scores = d_scores;
  a.packed = (uint8_t*)ws + packed_offset(n);
  a.inv = ws_inv(ws, n);
  a.natural = 1;
  a.n = n;
  a.perm = v.perm;
  a.sorted_bucket = v.sorted_bucket;
  a.status = &v.hdr->status;
  const int grid = (int)std::min<int64_t>(m->grid_gather, n);
  const size_t smem = sizeof(GatherSmem);
  const int st = d_acc ? launch_dependent("q_gather_kernel", q_gather_kernel<false, true>, (unsigned)grid,
                                          gather_threads(false), smem, s, a)
                       : launch_dependent("q_gather_kernel", q_gather_kernel<false, false>, (unsigned)grid,
                                          gather_threads(false), smem, s, a);
  if (st) return st;
  return launch_stack(m, a, v, s);
}

// Fused single-kernel forward (gather, pack and stacks in one kernel; needs
// only the bucket-sort workspace): the no-allocation entry point's path.
int launch_fused(const cnnue_q_model* m, const uint16_t* d_idx, uint32_t n_idx,
                 const uint32_t* d_offsets, int64_t n, int32_t* d_scores, void* ws, cudaStream_t s) {
  WorkspaceView v = carve_workspace(ws, n);
  ForwardArgs a = base_args();
  a.w = m->w;
  a.idx = d_idx;
  a.n_idx = n_idx;
  a.offsets = d_offsets;
  a.scores = d_scores;
  a.n = n;
  a.perm = v.perm;
  a.sorted_bucket = v.sorted_bucket;
  a.status = &v.hdr->status;
  const int grid = (int)std::min<int64_t>(m->grid_eval, n);
  q_bulk_kernel<false, false><<<grid, bulk_threads(false), sizeof(BulkSmem), s>>>(a);
  return check_launch("q_bulk_kernel");
}

bool misaligned16(const void* p) { return p != nullptr && ((uintptr_t)p & 15u) != 0; }

int check_indices_args(const void* idx, uint32_t n_idx, const void* offsets, const void* out,
                       int64_t n) {
  if (n == 0) return CNNUE_OK;
  if (!offsets || !out) return set_error(CNNUE_ERR_INVALID_ARG, "null offsets or output");
  if (n_idx > 0 && !idx) return set_error(CNNUE_ERR_INVALID_ARG, "null indices");
  return CNNUE_OK;
}

}  // namespace

extern "C" {

int cnnue_q_model_create(const cnnue_q_weights* w, int device, cnnue_q_model** out) {
  if (!w || !out) return set_error(CNNUE_ERR_INVALID_ARG, "null weights or out");
  if (!w->ft_weight || !w->ft_bias || !w->l1_weight || !w->l1_bias || !w->l2_weight ||
      !w->l2_bias || !w->l3_weight || !w->l3_bias)
    return set_error(CNNUE_ERR_INVALID_ARG, "a weight pointer is null");
  *out = nullptr;
  int n_dev = 0;
  if (cudaGetDeviceCount(&n_dev) != cudaSuccess || n_dev == 0)
    return set_error(CNNUE_ERR_NO_DEVICE, "no CUDA device");
  if (device < 0 || device >= n_dev)
    return set_error(CNNUE_ERR_NO_DEVICE, "device %d out of range (%d devices)", device, n_dev);
  DeviceGuard guard(device);
  if (guard.status) return guard.status;

  const size_t sz_ft = (size_t)(kF + 1) * kCols * 2, sz_bias = kCols * 2;  // + zero row
  const size_t sz_l1w = (size_t)kNB * kL1 * kCols, sz_l1b = kNB * kL1 * 4;
  const size_t sz_l2w = (size_t)kNB * kL2 * kL1, sz_l2b = kNB * kL2 * 4;
  const size_t sz_l3w = kNB * kL2, sz_l3b = kNB * 4;
  const size_t sizes[8] = {sz_ft, sz_bias, sz_l1w, sz_l1b, sz_l2w, sz_l2b, sz_l3w, sz_l3b};
  const void* srcs[8] = {w->ft_weight, w->ft_bias, w->l1_weight, w->l1_bias,
                         w->l2_weight, w->l2_bias, w->l3_weight, w->l3_bias};
  size_t offs[8], total = 0;
  for (int i = 0; i < 8; ++i) {
    offs[i] = total;
    total += align_up(sizes[i], 256);
  }
  auto* m = new cnnue_q_model();
  m->device = device;
  cudaError_t e = cudaMalloc(&m->blob, total);
  if (e != cudaSuccess) {
    delete m;
    return cuda_error(e, "cudaMalloc(weights)");
  }
  e = cudaMemset(m->blob, 0, total);
  for (int i = 0; i < 8 && e == cudaSuccess; ++i) {
    const size_t bytes = i == 0 ? (size_t)kF * kCols * 2 : sizes[i];  // row kF stays zero
    e = cudaMemcpy((char*)m->blob + offs[i], srcs[i], bytes, cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) {
    cudaFree(m->blob);
    delete m;
    return cuda_error(e, "cudaMemcpy(weights)");
  }
  char* b = (char*)m->blob;
  m->w.ft = (const int16_t*)(b + offs[0]);
  m->w.bias = (const int16_t*)(b + offs[1]);
  m->w.l1w = (const int8_t*)(b + offs[2]);
  m->w.l1b = (const int32_t*)(b + offs[3]);
  m->w.l2w = (const int8_t*)(b + offs[4]);
  m->w.l2b = (const int32_t*)(b + offs[5]);
  m->w.l3w = (const int8_t*)(b + offs[6]);
  m->w.l3b = (const int32_t*)(b + offs[7]);

  {
    // W1 as the stack kernel's tensor-core B operand: per bucket and 128-byte
    // K chunk a 16-row tile in the 128B-swizzled K-major layout.
    const size_t tile_bytes = (size_t)kNB * kTcChunks * kTcWTileBytes;
    std::vector<uint8_t> tiles(tile_bytes);
    for (int b = 0; b < kNB; ++b)
      for (int kc = 0; kc < kTcChunks; ++kc)
        for (int o = 0; o < kL1; ++o)
          for (int k = 0; k < kTcChunk; ++k)
            tiles[((size_t)b * kTcChunks + kc) * kTcWTileBytes + sw128_offset(o, k)] =
                (uint8_t)w->l1_weight[((size_t)b * kL1 + o) * kCols + kc * kTcChunk + k];
    e = cudaMalloc(&m->w1tiles, tile_bytes);
    if (e == cudaSuccess) e = cudaMemcpy(m->w1tiles, tiles.data(), tile_bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      if (m->w1tiles) cudaFree(m->w1tiles);
      cudaFree(m->blob);
      delete m;
      return cuda_error(e, "W1 tiles");
    }
  }
  cudaDeviceGetAttribute(&m->sm_count, cudaDevAttrMultiProcessorCount, device);
  const int smem = (int)sizeof(BulkSmem);
  cudaFuncSetAttribute(q_bulk_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const int gsmem = (int)sizeof(GatherSmem);
  cudaFuncSetAttribute(q_gather_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsmem);
  cudaFuncSetAttribute(q_gather_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsmem);
  cudaFuncSetAttribute(q_gather_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsmem);
  cudaFuncSetAttribute(q_stack_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)stack_tc_smem_bytes());
  int occ_eval = 0, occ_g = 0, occ_gu = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_eval, q_bulk_kernel<false, false>, bulk_threads(false), smem);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_g, q_gather_kernel<false, false>, gather_threads(false), gsmem);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_gu, q_gather_kernel<true, true>, gather_threads(true), gsmem);
  m->grid_eval = m->sm_count * std::max(occ_eval, 1);
  m->grid_gather = m->sm_count * std::max(occ_g, 1);
  m->grid_gather_update = m->sm_count * std::max(occ_gu, 1);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFree(m->blob);
    cudaFree(m->w1tiles);
    delete m;
    return cuda_error(e, "kernel attributes");
  }
  *out = m;
  return CNNUE_OK;
}

int cnnue_q_model_destroy(cnnue_q_model* m) {
  if (!m) return CNNUE_OK;
  DeviceGuard guard(m->device);
  if (m->blob) cudaFree(m->blob);
  if (m->w1tiles) cudaFree(m->w1tiles);
  if (m->stage) cudaFree(m->stage);
  delete m;
  return CNNUE_OK;
}

size_t cnnue_q_workspace_bytes(int64_t n_positions) { return q_workspace_bytes(n_positions); }

int cnnue_q_bucket_sort(const cnnue_q_model* m, const uint32_t* d_offsets, uint32_t n_indices,
                        int64_t n, void* ws, size_t ws_bytes, void* stream) {
  int st = validate_common(m, n, ws, ws_bytes);
  if (st) return st;
  if (n == 0) return CNNUE_OK;
  if (!d_offsets) return set_error(CNNUE_ERR_INVALID_ARG, "null offsets");
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  return launch_sort(m, d_offsets, n_indices, nullptr, n, ws, (cudaStream_t)stream, ws_inv(ws, n));
}

int cnnue_q_forward_sorted(const cnnue_q_model* m, const uint16_t* d_idx, uint32_t n_idx,
                           const uint32_t* d_offsets, int64_t n, int32_t* d_scores, void* ws,
                           size_t ws_bytes, void* stream) {
  int st = validate_common(m, n, ws, ws_bytes);
  if (st) return st;
  st = check_indices_args(d_idx, n_idx, d_offsets, d_scores, n);
  if (st) return st;
  if (n == 0) return CNNUE_OK;
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  return launch_eval(m, d_idx, n_idx, d_offsets, n, d_scores, nullptr, ws, (cudaStream_t)stream);
}

int cnnue_q_forward_acc(const cnnue_q_model* m, const uint16_t* d_idx, uint32_t n_idx,
                        const uint32_t* d_offsets, int64_t n, int32_t* d_scores, int16_t* d_acc,
                        void* ws, size_t ws_bytes, void* stream) {
  int st = validate_common(m, n, ws, ws_bytes);
  if (st) return st;
  st = check_indices_args(d_idx, n_idx, d_offsets, d_scores, n);
  if (st) return st;
  if (n == 0) return CNNUE_OK;
  if (misaligned16(d_acc)) return set_error(CNNUE_ERR_INVALID_ARG, "d_acc must be 16-byte aligned");
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  st = launch_sort(m, d_offsets, n_idx, nullptr, n, ws, s, ws_inv(ws, n));
  if (st) return st;
  return launch_eval(m, d_idx, n_idx, d_offsets, n, d_scores, d_acc, ws, s);
}

int cnnue_q_forward(const cnnue_q_model* m, const uint16_t* d_idx, uint32_t n_idx,
                    const uint32_t* d_offsets, int64_t n, int32_t* d_scores, void* ws,
                    size_t ws_bytes, void* stream) {
  return cnnue_q_forward_acc(m, d_idx, n_idx, d_offsets, n, d_scores, nullptr, ws, ws_bytes,
                             stream);
}

int cnnue_q_forward_host(cnnue_q_model* m, const uint16_t* h_idx, uint32_t n_idx,
                         const uint32_t* h_offsets, int64_t n, int32_t* h_scores, void* stream) {
  if (!m) return set_error(CNNUE_ERR_INVALID_ARG, "model is null");
  if (n < 0 || n > (int64_t)INT32_MAX) return set_error(CNNUE_ERR_INVALID_ARG, "bad n_positions");
  if (n == 0) return CNNUE_OK;
  if (!h_offsets || !h_scores || (n_idx > 0 && !h_idx))
    return set_error(CNNUE_ERR_INVALID_ARG, "null host buffer");
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t b_idx = align_up((size_t)n_idx * 2, 256);
  const size_t b_off = align_up((size_t)(2 * n + 1) * 4, 256);
  const size_t b_sc = align_up((size_t)n * 4, 256);
  const size_t b_ws = align_up(q_workspace_bytes(n), 256);
  const size_t need = b_idx + b_off + b_sc + b_ws;
  if (need > m->stage_bytes) {
    if (m->stage) {
      CNNUE_CUDA_TRY(cudaStreamSynchronize(s));
      cudaFree(m->stage);
      m->stage = nullptr;
      m->stage_bytes = 0;
    }
    CNNUE_CUDA_TRY(cudaMalloc(&m->stage, need));
    m->stage_bytes = need;
  }
  char* p = (char*)m->stage;
  uint16_t* d_idx = (uint16_t*)p;
  uint32_t* d_off = (uint32_t*)(p + b_idx);
  int32_t* d_sc = (int32_t*)(p + b_idx + b_off);
  void* ws = p + b_idx + b_off + b_sc;
  if (n_idx) CNNUE_CUDA_TRY(cudaMemcpyAsync(d_idx, h_idx, (size_t)n_idx * 2, cudaMemcpyHostToDevice, s));
  CNNUE_CUDA_TRY(cudaMemcpyAsync(d_off, h_offsets, (size_t)(2 * n + 1) * 4, cudaMemcpyHostToDevice, s));
  int st = launch_sort(m, d_off, n_idx, nullptr, n, ws, s, ws_inv(ws, n));
  if (st) return st;
  st = launch_eval(m, d_idx, n_idx, d_off, n, d_sc, nullptr, ws, s);
  if (st) return st;
  CNNUE_CUDA_TRY(cudaMemcpyAsync(h_scores, d_sc, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
  int status = CNNUE_OK;
  st = cnnue_read_status(ws, stream, &status);
  if (st) return st;
  return status;
}

int cnnue_q_forward_stall_test(const cnnue_q_model* m, const uint16_t* d_idx, uint32_t n_idx,
                               const uint32_t* d_offsets, int64_t n, int32_t* d_scores, void* ws,
                               size_t ws_bytes, uint32_t stall_block, uint32_t stall_stage,
                               uint64_t wait_limit_ns, void* stream) {
  int st = validate_common(m, n, ws, ws_bytes);
  if (st) return st;
  st = check_indices_args(d_idx, n_idx, d_offsets, d_scores, n);
  if (st) return st;
  if (n == 0) return CNNUE_OK;
  if (wait_limit_ns == 0 || wait_limit_ns > pipe::kWaitLimitNs)
    return set_error(CNNUE_ERR_INVALID_ARG, "wait limit must be in (0, %llu] ns", pipe::kWaitLimitNs);
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  st = launch_sort(m, d_offsets, n_idx, nullptr, n, ws, s, ws_inv(ws, n));
  if (st) return st;
  ForwardArgs hooks = base_args();
  hooks.wait_ns = wait_limit_ns;
  hooks.stall_block = stall_block;
  hooks.stall_stage = stall_stage;
  return launch_eval(m, d_idx, n_idx, d_offsets, n, d_scores, nullptr, ws, s, hooks);
}

int cnnue_q_update(const cnnue_q_model* m, const int16_t* d_parent, const uint8_t* d_flags,
                   const uint16_t* d_rem, uint32_t n_rem, const uint32_t* d_rem_offsets,
                   const uint16_t* d_add, uint32_t n_add, const uint32_t* d_add_offsets,
                   const uint8_t* d_count0, int64_t n, int16_t* d_child, int32_t* d_scores,
                   void* ws, size_t ws_bytes, void* stream) {
  int st = validate_common(m, n, ws, ws_bytes);
  if (st) return st;
  if (n == 0) return CNNUE_OK;
  if (!d_parent || !d_flags || !d_rem_offsets || !d_add_offsets || !d_count0 || !d_child ||
      !d_scores || (n_rem && !d_rem) || (n_add && !d_add))
    return set_error(CNNUE_ERR_INVALID_ARG, "null update buffer");
  if (misaligned16(d_parent) || misaligned16(d_child))
    return set_error(CNNUE_ERR_INVALID_ARG, "d_parent and d_child must be 16-byte aligned");
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  cudaStream_t s = (cudaStream_t)stream;
  // the sort also checks the removed and added lists' offsets
  st = launch_sort(m, nullptr, 0, d_count0, n, ws, s, ws_inv(ws, n), d_rem_offsets, n_rem, d_add_offsets, n_add);
  if (st) return st;
  WorkspaceView v = carve_workspace(ws, n);
  ForwardArgs a = base_args();
  a.packed = (uint8_t*)ws + packed_offset(n);
  a.inv = ws_inv(ws, n);
  a.natural = 1;
  a.w = m->w;
  a.idx = d_add;
  a.n_idx = n_add;
  a.offsets = d_add_offsets;
  a.rem = d_rem;
  a.n_rem = n_rem;
  a.rem_offsets = d_rem_offsets;
  a.parent = d_parent;
  a.flags = d_flags;
  a.acc_out = d_child;
  a.scores = d_scores;
  a.n = n;
  a.perm = v.perm;
  a.sorted_bucket = v.sorted_bucket;
  a.status = &v.hdr->status;
  const int grid = (int)std::min<int64_t>(m->grid_gather_update, n);
  st = launch_dependent("q_gather_kernel<update>", q_gather_kernel<true, true>, (unsigned)grid, gather_threads(true),
                        sizeof(GatherSmem), s, a);
  if (st) return st;
  return launch_stack(m, a, v, s);
}

}  // extern "C"


// ---------------------------------------------------------------------------
// Pipelined host-buffer evaluation: a caller-owned context with two slots,
// each with its own stream, device staging (indices, offsets, scores,
// workspace) and pinned status word, so one batch's host-to-device copies run
// while the previous batch's kernels do.  Created once (it allocates); the
// calls allocate nothing.
// ---------------------------------------------------------------------------
struct cnnue_q_stream_ctx {
  static constexpr int kSlots = 2;
  const cnnue_q_model* model = nullptr;
  int64_t max_n = 0;
  uint32_t max_idx = 0;
  struct Slot {
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr;
    char* dev = nullptr;
    uint32_t* h_status = nullptr;  // pinned
    bool busy = false;
    uint64_t ticket = 0;
    int launch_status = CNNUE_OK;
  } slot[kSlots];
  uint64_t next_ticket = 0;
};

namespace {

struct SlotLayout {
  size_t idx, off, sc, ws, total;
};

SlotLayout slot_layout(int64_t n, uint32_t n_idx) {
  SlotLayout l;
  l.idx = 0;
  l.off = align_up((size_t)n_idx * 2 + 2, 256);
  l.sc = l.off + align_up((size_t)(2 * n + 1) * 4, 256);
  l.ws = l.sc + align_up((size_t)n * 4, 256);
  l.total = l.ws + align_up(q_workspace_bytes(n), 256);
  return l;
}

void ctx_free(cnnue_q_stream_ctx* c) {
  for (auto& sl : c->slot) {
    if (sl.stream) cudaStreamSynchronize(sl.stream);
    if (sl.dev) cudaFree(sl.dev);
    if (sl.h_status) cudaFreeHost(sl.h_status);
    if (sl.done) cudaEventDestroy(sl.done);
    if (sl.stream) cudaStreamDestroy(sl.stream);
  }
  delete c;
}

}  // namespace

extern "C" {

int cnnue_q_ctx_create(const cnnue_q_model* m, int64_t max_positions, uint32_t max_indices,
                       cnnue_q_stream_ctx** out) {
  if (!m || !out) return set_error(CNNUE_ERR_INVALID_ARG, "null model or out");
  if (max_positions <= 0 || max_positions > (int64_t)INT32_MAX)
    return set_error(CNNUE_ERR_INVALID_ARG, "max_positions %lld out of range", (long long)max_positions);
  *out = nullptr;
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  auto* c = new cnnue_q_stream_ctx();
  c->model = m;
  c->max_n = max_positions;
  c->max_idx = max_indices;
  const SlotLayout l = slot_layout(max_positions, max_indices);
  for (auto& sl : c->slot) {
    cudaError_t e = cudaStreamCreateWithFlags(&sl.stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaMalloc(&sl.dev, l.total);
    if (e == cudaSuccess) e = cudaMallocHost(&sl.h_status, 64);
    if (e != cudaSuccess) {
      ctx_free(c);
      return cuda_error(e, "cnnue_q_ctx_create");
    }
  }
  *out = c;
  return CNNUE_OK;
}

int cnnue_q_ctx_destroy(cnnue_q_stream_ctx* c) {
  if (!c) return CNNUE_OK;
  DeviceGuard guard(c->model->device);
  ctx_free(c);
  return CNNUE_OK;
}

int cnnue_q_ctx_next_stream(const cnnue_q_stream_ctx* c, void** stream) {
  if (!c || !stream) return set_error(CNNUE_ERR_INVALID_ARG, "null context or stream");
  *stream = (void*)c->slot[c->next_ticket % cnnue_q_stream_ctx::kSlots].stream;
  return CNNUE_OK;
}

int cnnue_q_forward_host_async(cnnue_q_stream_ctx* c, const uint16_t* h_idx, uint32_t n_idx,
                               const uint32_t* h_offsets, int64_t n, int32_t* h_scores, uint64_t* ticket) {
  if (!c || !ticket) return set_error(CNNUE_ERR_INVALID_ARG, "null context or ticket");
  if (n < 0 || n > c->max_n)
    return set_error(CNNUE_ERR_INVALID_ARG, "n_positions %lld outside [0, %lld] of the context", (long long)n,
                     (long long)c->max_n);
  if (n_idx > c->max_idx)
    return set_error(CNNUE_ERR_INVALID_ARG, "n_indices %u above the context's %u", n_idx, c->max_idx);
  if (n > 0 && (!h_offsets || !h_scores || (n_idx > 0 && !h_idx)))
    return set_error(CNNUE_ERR_INVALID_ARG, "null host buffer");
  auto& sl = c->slot[c->next_ticket % cnnue_q_stream_ctx::kSlots];
  if (sl.busy)
    return set_error(CNNUE_ERR_INVALID_ARG, "two calls of this context are in flight: wait for ticket %llu first",
                     (unsigned long long)sl.ticket);
  const cnnue_q_model* m = c->model;
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  const SlotLayout l = slot_layout(c->max_n, c->max_idx);
  uint16_t* d_idx = (uint16_t*)(sl.dev + l.idx);
  uint32_t* d_off = (uint32_t*)(sl.dev + l.off);
  int32_t* d_sc = (int32_t*)(sl.dev + l.sc);
  void* ws = sl.dev + l.ws;
  cudaStream_t s = sl.stream;
  int st = CNNUE_OK;
  *sl.h_status = 0;
  if (n > 0) {
    if (n_idx) CNNUE_CUDA_TRY(cudaMemcpyAsync(d_idx, h_idx, (size_t)n_idx * 2, cudaMemcpyHostToDevice, s));
    CNNUE_CUDA_TRY(cudaMemcpyAsync(d_off, h_offsets, (size_t)(2 * n + 1) * 4, cudaMemcpyHostToDevice, s));
    st = launch_sort(m, d_off, n_idx, nullptr, n, ws, s, ws_inv(ws, n));
    if (!st) st = launch_eval(m, d_idx, n_idx, d_off, n, d_sc, nullptr, ws, s);
    if (!st) {
      CNNUE_CUDA_TRY(cudaMemcpyAsync(h_scores, d_sc, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
      CNNUE_CUDA_TRY(cudaMemcpyAsync(sl.h_status, ws, 4, cudaMemcpyDeviceToHost, s));
    }
  }
  CNNUE_CUDA_TRY(cudaEventRecord(sl.done, s));
  sl.busy = true;
  sl.ticket = c->next_ticket++;
  sl.launch_status = st;
  *ticket = sl.ticket;
  return CNNUE_OK;
}

int cnnue_q_ctx_wait(cnnue_q_stream_ctx* c, uint64_t ticket, int* status) {
  if (!c || !status) return set_error(CNNUE_ERR_INVALID_ARG, "null context or status");
  auto& sl = c->slot[ticket % cnnue_q_stream_ctx::kSlots];
  if (!sl.busy || sl.ticket != ticket)
    return set_error(CNNUE_ERR_INVALID_ARG, "ticket %llu is not in flight", (unsigned long long)ticket);
  DeviceGuard guard(c->model->device);
  if (guard.status) return guard.status;
  CNNUE_CUDA_TRY(cudaEventSynchronize(sl.done));
  sl.busy = false;
  *status = sl.launch_status ? sl.launch_status : status_from_word(*sl.h_status);
  return CNNUE_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// No-allocation entry point: the bucket-sort scratch of cnnue_q_forward lives
// in this file-scope device array instead of a caller workspace.  Host code
// must not hand `g_noalloc_scratch` itself to a kernel (on the host it is only
// a stand-in for the device symbol); its device address is looked up once per
// device with cudaGetSymbolAddress and cached.
// ---------------------------------------------------------------------------
static __device__ __align__(256) uint8_t g_noalloc_scratch[CNNUE_Q_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_device_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on `device` (must be current).
int noalloc_scratch(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (device < 0 || device >= kNoAllocMaxDevices)
    return set_error(CNNUE_ERR_NO_DEVICE, "device %d beyond the no-allocation table", device);
  if (g_noalloc_device_ptr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(no-allocation scratch)");
    g_noalloc_device_ptr[device] = p;
  }
  *out = g_noalloc_device_ptr[device];
  return CNNUE_OK;
}

}  // namespace

extern "C" int cnnue_q_forward_noalloc(const cnnue_q_model* m, const uint16_t* d_idx,
                                       uint32_t n_idx, const uint32_t* d_offsets, int64_t n,
                                       int32_t* d_scores, void* stream) {
  if (!m) return set_error(CNNUE_ERR_INVALID_ARG, "model is null");
  if (n < 0) return set_error(CNNUE_ERR_INVALID_ARG, "n_positions %lld is negative", (long long)n);
  if (n > CNNUE_Q_NOALLOC_MAX_POSITIONS)
    return set_error(CNNUE_ERR_INVALID_ARG,
                     "n_positions %lld exceeds the %d positions the no-allocation entry point's "
                     "fixed scratch holds; split the batch or call cnnue_q_forward with a workspace",
                     (long long)n, CNNUE_Q_NOALLOC_MAX_POSITIONS);
  int st = check_indices_args(d_idx, n_idx, d_offsets, d_scores, n);
  if (st) return st;
  if (n == 0) return CNNUE_OK;
  if (bucket_workspace_bytes(n) > sizeof(g_noalloc_scratch))
    return set_error(CNNUE_ERR_INTERNAL, "no-allocation scratch smaller than the workspace layout");
  DeviceGuard guard(m->device);
  if (guard.status) return guard.status;
  void* ws = nullptr;
  st = noalloc_scratch(m->device, &ws);
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
  // launch_sort zeroes the scratch header (status word, bucket counts and
  // cursors); the rest of the scratch is fully rewritten by every call.
  st = launch_sort(m, d_offsets, n_idx, nullptr, n, ws, s, nullptr);
  if (st) return st;
  st = launch_fused(m, d_idx, n_idx, d_offsets, n, d_scores, ws, s);
  if (st) return st;
  int status = CNNUE_OK;
  st = cnnue_read_status(ws, stream, &status);
  if (st) return st;
  return status;
}
