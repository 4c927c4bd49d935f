// Long-context verify attention on tcgen05 tensor cores (sm_100a).
//
// The second tcgen05 implementation of swiftLLM's paged attention for Target
// verify rows (swiftLLM/swiftllm/worker/kernels/paged_attn.py:9-222, rows built
// in nebulasd/src/nebulasd/workers/target/backend.py:102-111), for batches
// whose prefixes are long (thousands of tokens per unit), where the steady
// state dominates and the issue rate of the tensor-core instructions is the
// limit.  verify_attn.cu serves short prefixes, where fixed per-launch and
// per-piece costs dominate.
//
// Orientation: the KV tokens are the MMAs' M dimension.  A stage is 128
// tokens (eight 16-token blocks).  S^T = K Q^T is one M=128 x N=16..64 TMEM
// accumulator (eight K=16 MMAs over the head dimension, whatever the number
// of query columns: the GQA heads x adjacent rows of one request, up to 64),
// and O^T += V^T P^T (M = the 128 head-dim values, N = 64 query columns, one
// K=16 MMA per block).  A stage of 32 KB of K and 32 KB of V therefore costs
// each of the two issuing threads eight MMAs, half the issue work per byte of
// an M = query-rows tile with 64-token N.
//
// One persistent CTA per SM (the driver places a single CTA that allocates
// tensor memory on an SM); plan.cuh gives each an equal, cost-weighted share
// of KV tiles.  Warp roles (8 warps):
//   warp 0      K producer: 16 lanes issue a stage's sixteen 64-column TMA
//               boxes (128-byte swizzle) into a 2-slot ring and publish the
//               stage's block flags; block-table rows come batches ahead.
//   warp 1      S issuer (one thread): Q of the next piece by TMA into the
//               other half of a double buffer; S^T per stage into one of four
//               TMEM tiles, so that it runs ahead of the softmax.
//   warp 2      V producer: the V boxes into a 2-slot ring.
//   warp 3      P V issuer (one thread): O^T += V^T P^T into one of two TMEM
//               accumulators (one per piece, so that a piece's epilogue
//               overlaps the next piece's first products).
//   warps 4..7  softmax / epilogue: thread t owns token t of a stage (TMEM
//               lane t) across all query columns: scale, mask, exponentiate
//               against the columns' running maxima, store P^T as fp16.  The
//               maxima are uniform over the 128 threads and move only when a
//               score exceeds them by more than 2^8 (lazy rescale); the four
//               warps vote on that through the S-release barrier they arrive
//               on anyway, and reduce only when the vote says so.
// A unit split across CTAs is merged by the CTA whose piece of it ends last.
//
// Every wait is bounded (about 2 s); on expiry the kernel records an error
// bit, stops issuing work, waits (bounded) for its own copies and MMAs, frees
// its TMEM and returns.  The softmax warps synchronise only through mbarriers
// with bounded waits, never named barriers, so an abort strands no warp.  No
// TMA multicast is used.  The kernel is launched with programmatic stream
// serialisation: the set-up that reads no input (barriers, TMEM, tensor-map
// prefetch) runs before griddepcontrol.wait, beside the previous launch's tail.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "attn_common.cuh"
#include "sm100.cuh"

namespace neb {
namespace vlong {
using namespace sm100;

constexpr int kVThreads = 256;
constexpr int kKWarp = 0;
constexpr int kSWarp = 1;
constexpr int kVWarp = 2;
constexpr int kPVWarp = 3;
constexpr int kSoftmaxWarp0 = 4;                          // warps 4..7: TMEM lane quadrants 0..3
constexpr int kSoftmaxThreads = 128;
constexpr int kStageBlocks = 8;                           // 16-token KV blocks per stage
constexpr int kStageTokens = kStageBlocks * kBlockTokens;  // 128: the MMAs' M
constexpr int kKRing = 2;                                 // K ring slots (one stage each)
constexpr int kVRing = 2;                                 // V ring slots
constexpr int kSBufs = 4;                                 // S^T tiles in TMEM
constexpr int kPBufs = 2;                                 // P^T buffers in shared memory
constexpr int kOBufs = 2;                                 // O^T accumulators in TMEM
constexpr int kFlagSlots = 8;                             // block-flag ring (see the K producer)
constexpr int kMaxQ = 64;                                 // query columns per unit (gqa x rows)
constexpr int kMaxGqa = 64;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSCols = 64;                           // S^T tile b at columns 64 b
constexpr uint32_t kOCol = kSBufs * kSCols;               // O^T tile b at columns 256 + 64 b
constexpr long long kWaitLimit = 4000000000LL;
constexpr int kPieceCost = 56;                             // a piece's fixed cost, in tiles (plan.cuh CostSplit)
static_assert(kFlagSlots >= kKRing + kSBufs, "a flag slot is reused only after the softmax read it");
static_assert(kOCol + kOBufs * kMaxQ <= kTmemCols, "the S and O tiles fit the TMEM allocation");
static_assert(kStageBlocks * 2 <= 32, "one lane per TMA box of a stage");

// Shared memory map (offsets from a 1024-byte aligned base).
constexpr uint32_t kQHalf = kMaxQ * 128;            // 64 query rows x one 64-column half
constexpr uint32_t kQBuf = 2 * kQHalf;              // Q of one piece
constexpr uint32_t kKVHalf = kStageTokens * 128;    // 128 tokens x one 64-column half of K or V
constexpr uint32_t kStageBytes = 2 * kKVHalf;       // one stage of K (or V)
constexpr uint32_t kPBuf = kStageTokens * 128;      // P^T of a stage: 64 fp16 columns per token
constexpr uint32_t kQOff = 0;                       // two Q buffers
constexpr uint32_t kKOff = kQOff + 2 * kQBuf;
constexpr uint32_t kVOff = kKOff + kKRing * kStageBytes;
constexpr uint32_t kPOff = kVOff + kVRing * kStageBytes;
constexpr uint32_t kBarOff = kPOff + kPBufs * kPBuf;
constexpr uint32_t kRedOff = kBarOff + 1024;        // float [2][64][4]: the softmax warps' reductions
constexpr uint32_t kLensOff = kRedOff + 2048;       // int [2][64]: query-column lengths of a piece
constexpr uint32_t kMaxOff = kLensOff + 512;        // float [64]: the column maxima at a piece's end
constexpr uint32_t kPlanOff = kMaxOff + 256;
static_assert(kKVHalf % 1024 == 0 && kPBuf % 1024 == 0 && kQHalf % 1024 == 0, "swizzle atoms stay aligned");

// Largest row count whose plan arrays still fit next to the fixed buffers
// (227 KiB per CTA, less the alignment pad and 256 bytes of static shared memory).
constexpr int kVerifyMaxRows = ((232448 - 1024 - 256 - (int)kPlanOff) / 4 - 8) / 3 - 1;
static_assert(kVerifyMaxRows >= 1024, "room for the plan of a large verify batch");

struct VerifyShared;

// What every role needs to know about the launch and its own CTA.
struct Ctx {
  const AttnParams* p;
  VerifyShared* sh;
  uint8_t* smem;
  PlanSmem ps;
  int ng, hk, gqa, oob_row, group_rows;
  long long total, workers, w, t_begin, t_end;
  CostSplit split;  // which worker owns which tiles
  uint32_t tmem;
};

struct VerifyShared {
  Ctx ctx;                       // the launch context, written once by thread 0
  uint64_t k_full[kKRing];       // K of the slot's stage landed
  uint64_t k_empty[kKRing];      // S of the slot's stage completed
  uint64_t v_full[kVRing];       // V of the slot's stage landed
  uint64_t v_empty[kVRing];      // P V of the slot's stage completed
  uint64_t flags_full[kFlagSlots];
  uint64_t s_full[kSBufs];       // S^T of the tile's stage completed
  uint64_t s_empty[kSBufs];      // the four softmax warps read the tile (and voted)
  uint64_t p_full[kPBufs];       // the four softmax warps stored P^T
  uint64_t pv_done[kPBufs];      // P V of the buffer's stage completed
  uint64_t q_full[2];
  uint64_t q_empty[2];
  uint64_t o_full[kOBufs];       // every P V of the accumulator's piece completed
  uint64_t o_empty[kOBufs];      // the softmax warps read the accumulator out
  uint64_t grp[2];               // the softmax warps' own synchronisations
  uint64_t s_final;
  uint64_t pv_final;
  uint32_t tmem_base;
  int32_t abort_flag;
  int32_t merge_flag;
  int32_t blk[kFlagSlots][kStageBlocks];
  uint32_t vote[kSBufs][4];
  int32_t min4[2][4];
};
static_assert(sizeof(VerifyShared) <= 1024, "barrier block fits its slot");

__host__ __device__ inline size_t verify_smem_bytes(int num_rows) {
  return 1024 + kPlanOff + plan_smem_bytes(num_rows, true);
}

struct VerifyArgs {
  AttnParams p;
  int oob_row;  // first row past the end of the K/V tensor maps (loads there return zeros)
};

// The pieces of one worker: a cursor over its tile range (plan.cuh).
struct PieceCursor {
  const PlanSmem* ps;
  int ng, hk, g;
  long long t, t_end;
  __device__ __noinline__ void init(const PlanSmem* planp, int ngroups, int kvh, long long begin, long long end) {
    ps = planp;
    ng = ngroups;
    hk = kvh;
    t = begin;
    t_end = end;
    g = begin < end ? find_group(ps->gprefix, ng, begin, hk) : 0;
  }
  // Fills (group, kv_head, tile_lo, tile_hi, nb, unit_start); false when done.
  __device__ __forceinline__ bool next(int& grp, int& kv_head, int& lo, int& hi, int& nb, long long& unit_start) {
    if (t >= t_end) return false;
    while ((long long)hk * ps->gprefix[g + 1] <= t) ++g;
    nb = ps->gprefix[g + 1] - ps->gprefix[g];
    const long long gbase = (long long)hk * ps->gprefix[g];
    const int rel = (int)(t - gbase);  // < hk * nb
    kv_head = rel / nb;
    lo = rel - kv_head * nb;
    const int cnt = (int)min((long long)(nb - lo), t_end - t);
    hi = lo + cnt;
    unit_start = gbase + (long long)kv_head * nb;
    grp = g;
    t += cnt;
    return true;
  }
};

__device__ __forceinline__ int stages_of(int lo, int hi) { return (hi - lo + kStageBlocks - 1) / kStageBlocks; }

// Query columns of a unit rounded up to the S^T tile's N (a multiple of 16).
__device__ __forceinline__ int s_cols(int nq) { return (nq + 15) & ~15; }

__device__ __forceinline__ void raise_abort(VerifyShared* sh, const AttnParams& p) {
  if (atomicExch(&sh->abort_flag, 1) == 0) record_error(p, kErrTimeout);
}
__device__ __forceinline__ bool aborted(VerifyShared* sh) {
  return *reinterpret_cast<volatile int32_t*>(&sh->abort_flag) != 0;
}
// Slow path of wait_or_abort, out of line: one copy serves every call site.
// The thread sleeps in hardware while the phase is incomplete.
__device__ __noinline__ bool wait_or_abort_slow(VerifyShared* sh, const AttnParams& p, uint64_t* bar,
                                                uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait_sleep(bar, parity, 20000)) {
    if (aborted(sh) || clock64() - t0 > kWaitLimit) {
      raise_abort(sh, p);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ bool wait_or_abort(VerifyShared* sh, const AttnParams& p, uint64_t* bar,
                                              uint32_t parity) {
  return mbar_try_wait(bar, parity) || wait_or_abort_slow(sh, p, bar, parity);
}

// One arrival per softmax warp (count 4): the warp's lanes are first gathered
// with __syncwarp, which orders their earlier shared/tensor/global memory work.
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// A synchronisation of the four softmax warps on their own pair of mbarriers
// (use u takes barrier u % 2, phase u / 2); every warp makes the same uses.
__device__ __forceinline__ bool group_sync(VerifyShared* sh, const AttnParams& p, uint32_t& uses) {
  const uint32_t u = uses++;
  warp_arrive(&sh->grp[u & 1]);
  return wait_or_abort(sh, p, &sh->grp[u & 1], (u >> 1) & 1);
}

// Block-table rows of a producer warp's tiles, in the order the warp consumes
// them (the worker's flattened tile range).  Lane l holds tile base + 32k + l
// of batch k = 0, 1, 2; batch 2 is in flight while batches 0 and 1 are used.
struct TileFeed {
  const AttnParams* p;
  const PlanSmem* ps;
  int ng, oob_row;
  long long t_end, base;
  int r0, v0, r1, v1, r2, v2;

  // The fetch of one lane's tile in two steps, so that several batches' loads
  // can be in flight together: locate() finds the unit and reads the seq id,
  // table_pos()/finish() read and check the block-table entry.
  struct Pending {
    int sid, tile, kv_head;
    bool in_range;  // false: tile past the worker's range
  };
  __device__ __forceinline__ Pending locate(long long bt) const {
    Pending q{0, 0, 0, false};
    const long long t = bt + (threadIdx.x & 31);
    if (t >= t_end) return q;
    const int hk = p->num_kv_heads;
    const int g = find_group(ps->gprefix, ng, t, hk);
    const int nb = ps->gprefix[g + 1] - ps->gprefix[g];
    const int rel = (int)(t - (long long)hk * ps->gprefix[g]);  // < hk * nb
    q.kv_head = rel / nb;
    q.tile = rel - q.kv_head * nb;
    q.sid = ps->gsid[g];
    q.in_range = true;
    return q;
  }
  __device__ __forceinline__ long long table_pos(const Pending& q, uint32_t& err) const {
    if (!q.in_range) return -1;
    if (q.sid < 0 || q.sid >= p->bt_rows) {
      err |= kErrSeqId;
      return -1;
    }
    if (q.tile >= p->mbs) {
      err |= kErrTooManyBlocks;
      return -1;
    }
    return (long long)q.sid * p->mbs + q.tile;
  }
  __device__ __forceinline__ void finish(const Pending& q, long long pos, long long blk, uint32_t& err, int& r,
                                         int& v) const {
    r = oob_row;
    v = 0;
    if (pos < 0) return;  // no table entry read
    if (blk < 0 || blk >= p->num_blocks) {
      err |= kErrBlockIndex;
      return;
    }
    v = 1;
    r = (int)(((blk * p->num_layers + p->cur_layer) * p->num_kv_heads + q.kv_head) * kBlockTokens);
  }
  __device__ __forceinline__ void fetch(long long bt, int& r, int& v) const {
    uint32_t err = 0;
    const Pending q = locate(bt);
    const long long i = table_pos(q, err);
    finish(q, i, i >= 0 ? (long long)__ldg(p->block_table + i) : 0, err, r, v);
    if (err) record_error(*p, err);
  }
  __device__ void init(const AttnParams* pp, const PlanSmem* pps, int ngroups, int oob, long long begin,
                       long long end) {
    p = pp;
    ps = pps;
    ng = ngroups;
    oob_row = oob;
    t_end = end;
    base = begin;
    const Pending q0 = locate(base), q1 = locate(base + 32), q2 = locate(base + 64);
    uint32_t err = 0;
    const long long i0 = table_pos(q0, err), i1 = table_pos(q1, err), i2 = table_pos(q2, err);
    const long long b0 = i0 >= 0 ? (long long)__ldg(p->block_table + i0) : 0;
    const long long b1 = i1 >= 0 ? (long long)__ldg(p->block_table + i1) : 0;
    const long long b2 = i2 >= 0 ? (long long)__ldg(p->block_table + i2) : 0;
    finish(q0, i0, b0, err, r0, v0);
    finish(q1, i1, b1, err, r1, v1);
    finish(q2, i2, b2, err, r2, v2);
    if (err) record_error(*p, err);
  }
  // Row and flag of tile pos + b (b per lane), for base <= pos + b < base + 64.
  __device__ __forceinline__ void get_lane(long long pos, int b, int& r, int& v) const {
    const int d = (int)(pos + b - base);
    const int ra = __shfl_sync(0xffffffffu, r0, d & 31), rb = __shfl_sync(0xffffffffu, r1, d & 31);
    const int va = __shfl_sync(0xffffffffu, v0, d & 31), vb = __shfl_sync(0xffffffffu, v1, d & 31);
    r = d < 32 ? ra : rb;
    v = d < 32 ? va : vb;
  }
  // Drops the batches before `pos` and starts fetching the ones after.
  __device__ __forceinline__ void advance(long long pos) {
    while (pos >= base + 32) {
      r0 = r1; v0 = v1;
      r1 = r2; v1 = v2;
      base += 32;
      fetch(base + 64, r2, v2);
    }
  }
};

// ------------------------------------------------------------------ producers
// One function serves the K warp (flags: it also publishes the block flags)
// and the V warp, over a ring of `ring` one-stage slots.  Stage G sits in slot
// G % ring; the slot frees when the MMAs that read it (S for K, P V for V) are
// done.  The block flags of stage G go to flag slot G % kFlagSlots: before
// they are written, slot G % ring was freed by S of stage G - ring, which was
// issued once the softmax released S tile (G - ring) % kSBufs after stage
// G - ring - kSBufs, and the softmax reads a stage's flags before it releases
// its S tile, so flag slots with kFlagSlots >= ring + kSBufs are free.
__device__ __noinline__ void producer(const Ctx& c, const CUtensorMap* tmap, uint64_t* full, uint64_t* empty,
                                      uint32_t ring_off, int ring, bool flags) {
  const AttnParams& p = *c.p;
  VerifyShared* sh = c.sh;
  const int lane = threadIdx.x & 31;
  // K and V tiles are read once: let them leave L2 first, so that the kernel's
  // code, the plan inputs, q and the merge partials stay cached.
  const uint64_t kv_policy = l2_evict_first_policy();
  TileFeed feed;
  feed.init(&p, &c.ps, c.ng, c.oob_row, c.t_begin, c.t_end);
  PieceCursor cur;
  cur.init(&c.ps, c.ng, c.hk, c.t_begin, c.t_end);
  int s_lo = 0, s_hi = 0;
  // Lane l < 16 carries box l of a stage: block l & 7, half l >> 3.
  const int b = lane & (kStageBlocks - 1), hf = (lane >> 3) & 1;
  int G = 0, slot = 0, used = 0;
  uint32_t phase = 0;  // parity of the slot's current use
  long long pos = c.t_begin;
  for (;;) {
    if (s_lo >= s_hi) {
      int g, h, nb;
      long long ustart;
      if (!cur.next(g, h, s_lo, s_hi, nb, ustart)) break;
    }
    const int nblk = min(kStageBlocks, s_hi - s_lo);
    s_lo += nblk;
    int row, valid;
    feed.get_lane(pos, b, row, valid);
    int waited = 1;
    if (lane == 0) {
      waited = wait_or_abort(sh, p, &empty[slot], phase ^ 1u);
      if (waited) mbar_arrive_expect_tx(&full[slot], (uint32_t)nblk * 2u * 2048u);
    }
    waited = __shfl_sync(0xffffffffu, waited, 0);
    if (!waited) break;
    // One lane per 64-column box, so that the stage's loads leave together.
    if (lane < 2 * kStageBlocks && b < nblk)
      tma_load_2d_hint(c.smem + ring_off + slot * kStageBytes + hf * kKVHalf + b * 2048, tmap, &full[slot],
                       64 * hf, row, kv_policy);
    if (flags) {
      if (lane < kStageBlocks) sh->blk[G % kFlagSlots][lane] = lane < nblk ? valid : 0;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->flags_full[G % kFlagSlots]);
    }
    ++used;
    ++G;
    pos += nblk;
    feed.advance(pos);
    if (++slot == ring) {
      slot = 0;
      phase ^= 1u;
    }
  }
  // Wait (bounded) for every copy this warp issued before the CTA can exit.
  if (lane == 0)
#pragma unroll 1
    for (int u = (used > ring ? used - ring : 0); u < used; ++u)
      mbar_wait(&full[u % ring], (uint32_t)((u / ring) & 1), kWaitLimit);
}

// ------------------------------------------------------------------- S issuer
// Q of piece i goes to buffer i % 2 as soon as piece i - 2 is done with it,
// i.e. a whole piece ahead of its first S.  A Q box is gqa heads x group_rows
// rows of one 64-column half; the unit's query column j = r * gqa + head sits
// in row j of the buffer (rows past the unit belong to other units or past
// the tensor, and their S^T columns are never used).
struct QFeeder {
  PieceCursor cur;
  int qi, qg, qh, qlo, qhi, qnb;
  long long qus;
  bool qhave;
  __device__ __noinline__ bool feed(const Ctx& c, const CUtensorMap* tmap_q, int cur_piece, int need) {
    VerifyShared* sh = c.sh;
    while (qhave && qi <= cur_piece + 1) {
      const int b = qi & 1;
      if (qi >= 2) {
        const uint32_t par = (uint32_t)(((qi - 2) >> 1) & 1);
        if (qi > need) {
          if (!mbar_test_wait(&sh->q_empty[b], par)) return true;
        } else if (!wait_or_abort(sh, *c.p, &sh->q_empty[b], par)) {
          return false;
        }
      }
      const uint32_t box_bytes = (uint32_t)(c.gqa * c.group_rows) * 128u;
      mbar_arrive_expect_tx(&sh->q_full[b], 2u * box_bytes);
      const int first_row = c.ps.gfirst[qg];
#pragma unroll 1
      for (int dh = 0; dh < 2; ++dh)
        tma_load_3d(c.smem + kQOff + b * kQBuf + dh * kQHalf, tmap_q, &sh->q_full[b], dh * 64, qh * c.gqa,
                    first_row);
      ++qi;
      qhave = cur.next(qg, qh, qlo, qhi, qnb, qus);
    }
    return true;
  }
};

__device__ __noinline__ void s_issuer(const Ctx& c, const CUtensorMap* tmap_q) {
  const AttnParams& p = *c.p;
  VerifyShared* sh = c.sh;
  const uint32_t q_base = smem_u32(c.smem + kQOff);
  const uint32_t k_base = smem_u32(c.smem + kKOff);
  const uint32_t tmem = c.tmem;
  QFeeder qf;
  qf.cur.init(&c.ps, c.ng, c.hk, c.t_begin, c.t_end);
  qf.qi = 0;
  qf.qhave = qf.cur.next(qf.qg, qf.qh, qf.qlo, qf.qhi, qf.qnb, qf.qus);
  PieceCursor cur;
  cur.init(&c.ps, c.ng, c.hk, c.t_begin, c.t_end);
  int g, h, lo, hi, nb;
  long long ustart;
  int G = 0;
  bool ok = true;
  for (int piece = 0; ok && cur.next(g, h, lo, hi, nb, ustart); ++piece) {
    const int nst = stages_of(lo, hi);
    const int b = piece & 1;
    if (!qf.feed(c, tmap_q, piece, piece) || !wait_or_abort(sh, p, &sh->q_full[b], (uint32_t)((piece >> 1) & 1)))
      break;
    const int nq = (c.ps.gfirst[g + 1] - c.ps.gfirst[g]) * c.gqa;
    const uint32_t idesc_s = idesc_f16_f32(kStageTokens, s_cols(nq), false, false);
    // Descriptors of the eight K=16 steps over the head dimension: the base's
    // address field plus a constant (shared-memory addresses / 16 stay below 2^14).
    const uint64_t b0 = smem_desc_sw128(q_base + b * kQBuf, 16, 1024);
    for (int s = 0; s < nst; ++s, ++G) {
      const int slot = G % kKRing, sb = G % kSBufs;
      if (!wait_or_abort(sh, p, &sh->k_full[slot], (uint32_t)((G / kKRing) & 1)) ||
          !wait_or_abort(sh, p, &sh->s_empty[sb], (uint32_t)(((G / kSBufs) & 1) ^ 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t a0 = smem_desc_sw128(k_base + slot * kStageBytes, 16, 1024);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16(tmem + sb * kSCols, a0 + (((kk >> 2) * kKVHalf + (kk & 3) * 32) >> 4),
                b0 + (((kk >> 2) * kQHalf + (kk & 3) * 32) >> 4), idesc_s, kk > 0 ? 1u : 0u);
      mma_commit(&sh->s_full[sb]);
      mma_commit(&sh->k_empty[slot]);
      if (s == nst - 1) mma_commit(&sh->q_empty[b]);
      if (qf.qhave && qf.qi <= piece + 1 && !qf.feed(c, tmap_q, piece, piece)) {
        ok = false;
        break;
      }
    }
  }
  mma_commit(&sh->s_final);
  mbar_wait(&sh->s_final, 0, kWaitLimit);
  // Q loads issued for pieces that never ran (after an abort) must land before exit.
#pragma unroll 1
  for (int i = (qf.qi > 2 ? qf.qi - 2 : 0); i < qf.qi; ++i)
    mbar_wait(&sh->q_full[i & 1], (uint32_t)((i >> 1) & 1), kWaitLimit);
}

// ----------------------------------------------------------------- P V issuer
// O^T (head dim x 64 query columns) += V^T (head dim x 16 tokens, V read as an
// MN-major operand) x P^T (16 tokens x 64 columns, MN-major), one MMA per block.
__device__ __noinline__ void pv_issuer(const Ctx& c) {
  const AttnParams& p = *c.p;
  VerifyShared* sh = c.sh;
  const uint32_t v_base = smem_u32(c.smem + kVOff);
  const uint32_t p_base = smem_u32(c.smem + kPOff);
  const uint32_t idesc_pv = idesc_f16_f32(kStageTokens, kMaxQ, true, true);
  const uint32_t tmem = c.tmem;
  PieceCursor cur;
  cur.init(&c.ps, c.ng, c.hk, c.t_begin, c.t_end);
  int g, h, lo, hi, nb;
  long long ustart;
  int G = 0;
  bool ok = true;
  for (int piece = 0; ok && cur.next(g, h, lo, hi, nb, ustart); ++piece) {
    const int nst = stages_of(lo, hi);
    const int ob = piece % kOBufs;
    for (int s = 0; s < nst; ++s, ++G) {
      const int slot = G % kVRing, pb = G % kPBufs;
      if (!wait_or_abort(sh, p, &sh->p_full[pb], (uint32_t)((G / kPBufs) & 1)) ||
          !wait_or_abort(sh, p, &sh->v_full[slot], (uint32_t)((G / kVRing) & 1)) ||
          (s == 0 && piece >= kOBufs &&
           !wait_or_abort(sh, p, &sh->o_empty[ob], (uint32_t)(((piece - kOBufs) / kOBufs) & 1)))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int nblk = min(kStageBlocks, hi - (lo + s * kStageBlocks));
      const uint64_t va0 = smem_desc_sw128(v_base + slot * kStageBytes, kKVHalf, 1024);
      const uint64_t pb0 = smem_desc_sw128(p_base + pb * kPBuf, kPBuf, 1024);
#pragma unroll
      for (int kb = 0; kb < kStageBlocks; ++kb) {
        if (kb < nblk)
          mma_f16(tmem + kOCol + ob * kMaxQ, va0 + ((kb * 2048) >> 4), pb0 + ((kb * 2048) >> 4), idesc_pv,
                  (s == 0 && kb == 0) ? 0u : 1u);
      }
      mma_commit(&sh->v_empty[slot]);
      mma_commit(&sh->pv_done[pb]);
      if (s == nst - 1) mma_commit(&sh->o_full[ob]);
    }
  }
  mma_commit(&sh->pv_final);
  mbar_wait(&sh->pv_final, 0, kWaitLimit);
}

// -------------------------------------------------------------------- softmax
// The unit rows of a piece.
struct PieceRows {
  int g, h, lo, hi, nb;
  long long ustart;
  int first_row, nrows, nq;
};

// Element offset of query column j of a unit in q / o ([rows][heads][128]).
__device__ __forceinline__ long long column_offset(const AttnParams& p, int first_row, int kv_head, int gqa, int j) {
  const int r = j / gqa;
  return ((long long)(first_row + r) * p.num_q_heads + kv_head * gqa + (j - r * gqa)) * kHeadDim;
}

// Sum of the four warps' parts of column j (reduction buffer rb, [64][4]).
__device__ __forceinline__ float sum4(const float* rb, int j) {
  const float4 v = *reinterpret_cast<const float4*>(rb + 4 * j);
  return (v.x + v.y) + (v.z + v.w);
}

// Merge of a unit split across CTAs by the 128 softmax threads: each (query
// column, 8-value chunk) folds the pieces' partials in worker order, four
// slots per round with their loads issued together, and writes fp16.  The
// arithmetic does not depend on which CTA merges, so results are reproducible.
// A piece with no unmasked token (lse -inf) carries no weight; all empty gives
// 0/0 = NaN, as in the reference's phase 2 (paged_attn.py:131-149).
static __device__ __noinline__ void merge_unit(const AttnParams& p, int first_row, int nq, int kv_head, int gqa,
                                               long long w0, long long w1, int tid) {
#pragma unroll 1
  for (int c = tid; c < nq * 16; c += kSoftmaxThreads) {
    const int j = c >> 4, q8 = (c & 15) * 8;
    float mx = neg_inf(), den = 0.f;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll 1
    for (long long wb = w0; wb <= w1; wb += 4) {
      float le[4];
      float4 va[4], vb[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        le[k] = neg_inf();
        va[k] = vb[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (wb + k <= w1) {
          const long long slot = piece_slot(wb + k, w0);
          le[k] = __ldcg(p.part_lse + slot * p.nq + j);
          const float4* src = reinterpret_cast<const float4*>(p.part_o + (slot * p.nq + j) * kHeadDim + q8);
          va[k] = __ldcg(src);
          vb[k] = __ldcg(src + 1);
        }
      }
      const float cm = fmaxf(fmaxf(le[0], le[1]), fmaxf(le[2], le[3]));
      if (cm == neg_inf()) continue;
      if (cm > mx) {
        const float sc = fast_exp2(mx - cm);  // 0 while nothing was folded in yet
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] *= sc;
        den *= sc;
        mx = cm;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (le[k] == neg_inf()) continue;
        const float wt = fast_exp2(le[k] - mx);
        acc[0] += wt * va[k].x; acc[1] += wt * va[k].y; acc[2] += wt * va[k].z; acc[3] += wt * va[k].w;
        acc[4] += wt * vb[k].x; acc[5] += wt * vb[k].y; acc[6] += wt * vb[k].z; acc[7] += wt * vb[k].w;
        den += wt;
      }
    }
    const float inv = 1.f / den;
    uint4 out;
    out.x = f2_to_h2(acc[0] * inv, acc[1] * inv);
    out.y = f2_to_h2(acc[2] * inv, acc[3] * inv);
    out.z = f2_to_h2(acc[4] * inv, acc[5] * inv);
    out.w = f2_to_h2(acc[6] * inv, acc[7] * inv);
    *reinterpret_cast<uint4*>(p.o + column_offset(p, first_row, kv_head, gqa, j) + q8) = out;
  }
}

// Rare: a score exceeded its column's maximum by more than 2^8 after the
// first stage of a piece.  The columns whose maximum moves get
// alpha = 2^(m_old - m_new) on l and on O^T (once every P V so far is done).
template <int N>
__device__ __forceinline__ bool rescale_piece(const Ctx& c, const float* rb, float (&m)[N], float (&l)[N], int G,
                                              int pi) {
  const AttnParams& p = *c.p;
  VerifyShared* sh = c.sh;
  float alpha[N];
  bool rescale = false;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const float4 w = *reinterpret_cast<const float4*>(rb + 4 * j);
    const float cm = fmaxf(fmaxf(w.x, w.y), fmaxf(w.z, w.w));
    alpha[j] = 1.f;
    if (cm > m[j] + 8.f) {
      if (m[j] != neg_inf()) {
        alpha[j] = fast_exp2(m[j] - cm);
        rescale = true;
      }
      m[j] = cm;
    }
    l[j] *= alpha[j];
  }
  if (!rescale) return true;
  if (!wait_or_abort(sh, p, &sh->pv_done[(G - 1) % kPBufs], (uint32_t)(((G - 1) / kPBufs) & 1))) return false;
  tc_fence_after();
  const uint32_t oaddr = c.tmem + kOCol + (pi % kOBufs) * kMaxQ + ((uint32_t)(32 * ((threadIdx.x >> 5) & 3)) << 16);
#pragma unroll
  for (int c0 = 0; c0 < N; c0 += 16) {
    uint32_t o[16];
    tmem_ld_32x32b_x16(oaddr + c0, o);
    tmem_wait_ld();
#pragma unroll
    for (int k = 0; k < 16; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha[c0 + k]);
    tmem_st_32x32b_x16(oaddr + c0, o);
  }
  tmem_wait_st();
  tc_fence_before();
  return true;
}

// End of a piece: column sums over the 128 tokens, O^T read out of TMEM and
// staged as fp32 [column][head dim] in the P buffers (idle: every P V of the
// piece is done), then written with rolled loops of 16-byte stores: fp16
// output rows, or for a unit split across CTAs its partial (O / l and
// m + log2 l), counted in; the piece that completes the unit merges.
template <int N>
__device__ __forceinline__ bool piece_epilogue(const Ctx& c, const PieceRows& r, int pi, const float (&m)[N],
                                               float (&l)[N], uint32_t& grp_uses) {
  const AttnParams& p = *c.p;
  VerifyShared* sh = c.sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qd = warp & 3;
  const int tid = threadIdx.x - kSoftmaxWarp0 * 32;
  const uint32_t lane_addr = (uint32_t)(32 * qd) << 16;
#pragma unroll 1
  for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
    for (int j = 0; j < N; ++j) l[j] += __shfl_xor_sync(0xffffffffu, l[j], o);
  float* rb = reinterpret_cast<float*>(c.smem + kRedOff) + (grp_uses & 1) * 4 * kMaxQ;
  float* msm = reinterpret_cast<float*>(c.smem + kMaxOff);
  if (lane == 0)
#pragma unroll
    for (int j = 0; j < N; ++j) rb[4 * j + qd] = l[j];
  if (tid == 0)
#pragma unroll
    for (int j = 0; j < N; ++j) msm[j] = m[j];
  const int ob = pi % kOBufs;
  if (!wait_or_abort(sh, p, &sh->o_full[ob], (uint32_t)((pi / kOBufs) & 1))) return false;
  tc_fence_after();
  uint32_t oraw[N];
  tmem_ld_32x32b_cols<N>(c.tmem + kOCol + ob * kMaxQ + lane_addr, oraw);
  tmem_wait_ld();
  tc_fence_before();
  warp_arrive(&sh->o_empty[ob]);
  float* stg = reinterpret_cast<float*>(c.smem + kPOff);
#pragma unroll
  for (int j = 0; j < N; ++j) stg[j * kHeadDim + tid] = __uint_as_float(oraw[j]);
  if (!group_sync(sh, p, grp_uses)) return false;
  const int gqa = c.gqa;
  if (r.lo == 0 && r.hi == r.nb) {
#pragma unroll 1
    for (int ci = tid; ci < r.nq * 16; ci += kSoftmaxThreads) {
      const int j = ci >> 4, q8 = (ci & 15) * 8;
      const float inv = 1.f / sum4(rb, j);
      const float4 a = *reinterpret_cast<const float4*>(stg + j * kHeadDim + q8);
      const float4 b = *reinterpret_cast<const float4*>(stg + j * kHeadDim + q8 + 4);
      uint4 out;
      out.x = f2_to_h2(a.x * inv, a.y * inv);
      out.y = f2_to_h2(a.z * inv, a.w * inv);
      out.z = f2_to_h2(b.x * inv, b.y * inv);
      out.w = f2_to_h2(b.z * inv, b.w * inv);
      *reinterpret_cast<uint4*>(p.o + column_offset(p, r.first_row, r.h, gqa, j) + q8) = out;
    }
    return true;
  }
  const long long w0 = c.split.worker_of_tile(r.ustart);
  const long long w1 = c.split.worker_of_tile(r.ustart + r.nb - 1);
  const long long slot = piece_slot(c.w, w0);
  const long long unit = (long long)r.g * c.hk + r.h;
#pragma unroll 1
  for (int ci = tid; ci < r.nq * 32; ci += kSoftmaxThreads) {
    const int j = ci >> 5, q4 = (ci & 31) * 4;
    const float inv = 1.f / sum4(rb, j);
    float4 a = *reinterpret_cast<const float4*>(stg + j * kHeadDim + q4);
    a.x *= inv; a.y *= inv; a.z *= inv; a.w *= inv;
    __stcg(reinterpret_cast<float4*>(p.part_o + (slot * p.nq + j) * kHeadDim + q4), a);
  }
#pragma unroll 1
  for (int j = tid; j < r.nq; j += kSoftmaxThreads) {
    const float lt = sum4(rb, j);
    __stcg(p.part_lse + slot * p.nq + j, lt > 0.f ? msm[j] + __log2f(lt) : neg_inf());
  }
  // Every partial store precedes thread 0's fence (mbarrier release/acquire).
  if (!group_sync(sh, p, grp_uses)) return false;
  if (tid == 0) {
    __threadfence();
    const int last = atomicAdd(p.counters + unit, 1) == (int)(w1 - w0);
    if (last) p.counters[unit] = 0;  // every piece has arrived: ready for the next call
    sh->merge_flag = last;
  }
  if (!group_sync(sh, p, grp_uses)) return false;
  if (sh->merge_flag) {
    __threadfence();
    merge_unit(p, r.first_row, r.nq, r.h, gqa, w0, w1, tid);
  }
  return true;
}

// One piece of the softmax role, for units of at most N query columns.  Thread
// tid (0..127) owns token tid of each stage (TMEM lane tid of the S^T tiles)
// and, in the epilogue, head-dim index tid (TMEM lane tid of O^T).  m[j] is
// column j's running maximum (the same in every thread), l[j] this thread's
// part of the column's sum of the fp16 P values the MMA reads.  Code that
// runs once per piece is kept compact (rolled loops over shared memory): it
// runs from a cold instruction cache.
template <int N>
__device__ __noinline__ bool softmax_piece(const Ctx& c, const PieceRows& r, int G0, int pi, uint32_t& grp_uses) {
  const AttnParams& p = *c.p;
  VerifyShared* sh = c.sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qd = warp & 3;
  const int tid = threadIdx.x - kSoftmaxWarp0 * 32;
  const uint32_t lane_addr = (uint32_t)(32 * qd) << 16;
  const float sc = p.scale_log2;
  const int gqa = c.gqa;
  float* red = reinterpret_cast<float*>(c.smem + kRedOff);
  int* lens = reinterpret_cast<int*>(c.smem + kLensOff) + (pi & 1) * kMaxQ;
  const uint32_t p_base = smem_u32(c.smem + kPOff);

  // Column lengths of the piece (0 past the unit's columns) and their minimum.
  {
    int mn = INT_MAX;
    if (tid < kMaxQ) {
      const int len = tid < r.nq ? __ldg(p.seq_lens + r.first_row + tid / gqa) : 0;
      lens[tid] = len;
      if (tid < r.nq) mn = len;
    }
    mn = __reduce_min_sync(0xffffffffu, mn);
    if (lane == 0) sh->min4[pi & 1][qd] = mn;
    if (!group_sync(sh, p, grp_uses)) return false;
  }
  const int min_len = min(min(sh->min4[pi & 1][0], sh->min4[pi & 1][1]), min(sh->min4[pi & 1][2], sh->min4[pi & 1][3]));

  float m[N], l[N];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    m[j] = neg_inf();
    l[j] = 0.f;
  }
  const int nst = stages_of(r.lo, r.hi);
  for (int s = 0; s < nst; ++s) {
    const int G = G0 + s;
    const int fs = G % kFlagSlots, sb = G % kSBufs, pb = G % kPBufs;
    if (!wait_or_abort(sh, p, &sh->flags_full[fs], (uint32_t)((G / kFlagSlots) & 1)) ||
        !wait_or_abort(sh, p, &sh->s_full[sb], (uint32_t)((G / kSBufs) & 1)))
      return false;
    tc_fence_after();
    uint32_t raw[N];
    tmem_ld_32x32b_cols<N>(c.tmem + sb * kSCols + lane_addr, raw);
    const int t0 = r.lo + s * kStageBlocks;
    const int nblk = min(kStageBlocks, r.hi - t0);
    const int bk = tid >> 4;
    const bool tok_ok = bk < nblk && sh->blk[fs][bk] != 0;  // flags read before S is released
    const int tok = t0 * kBlockTokens + tid;
    tmem_wait_ld();
    // Scores into the exp2 domain; masked (-inf) past a column's length, past
    // the stage's blocks (stale rows of the S^T tile) and on bad blocks.
    float v[N];
    if (tok_ok && tok < min_len) {
#pragma unroll
      for (int j = 0; j < N; ++j) v[j] = j < r.nq ? __uint_as_float(raw[j]) * sc : neg_inf();
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j) v[j] = (tok_ok && tok < lens[j]) ? __uint_as_float(raw[j]) * sc : neg_inf();
    }
    bool need = s == 0;  // the first stage sets the maxima
#pragma unroll
    for (int j = 0; j < N; ++j) need |= v[j] > m[j] + 8.f;
    const uint32_t any = __any_sync(0xffffffffu, need) ? 1u : 0u;
    if (lane == 0) sh->vote[sb][qd] = any;
    tc_fence_before();
    warp_arrive(&sh->s_empty[sb]);
    // The four arrivals complete the release of the tile and publish the votes.
    if (!wait_or_abort(sh, p, &sh->s_empty[sb], (uint32_t)((G / kSBufs) & 1))) return false;
    if ((sh->vote[sb][0] | sh->vote[sb][1] | sh->vote[sb][2] | sh->vote[sb][3]) != 0) {
      // Column maxima of the stage: one reduction per warp, then the four warps.
      float* rb = red + (grp_uses & 1) * 4 * kMaxQ;
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const float mx = warp_max_f32(v[j]);
        if (lane == 0) rb[4 * j + qd] = mx;
      }
      if (!group_sync(sh, p, grp_uses)) return false;
      if (s == 0) {
#pragma unroll
        for (int j = 0; j < N; ++j) {
          const float4 w = *reinterpret_cast<const float4*>(rb + 4 * j);
          m[j] = fmaxf(fmaxf(w.x, w.y), fmaxf(w.z, w.w));
        }
      } else if (!rescale_piece<N>(c, rb, m, l, G, pi)) {
        return false;
      }
    }
    // P^T row of this token: 2^(s - m) as fp16 pairs (0 where masked or no max yet).
    uint32_t pk[N / 2];
#pragma unroll
    for (int jj = 0; jj < N / 2; ++jj) {
      const int j0 = 2 * jj, j1 = 2 * jj + 1;
      const float a = m[j0] != neg_inf() ? fast_exp2(v[j0] - m[j0]) : 0.f;
      const float b = m[j1] != neg_inf() ? fast_exp2(v[j1] - m[j1]) : 0.f;
      pk[jj] = f2_to_h2(a, b);
      const float2 f = h2_to_f2(pk[jj]);
      l[j0] += f.x;
      l[j1] += f.y;
    }
    // P buffer pb is free once P V of stage G - 2 completed.
    if (G >= kPBufs && !wait_or_abort(sh, p, &sh->pv_done[pb], (uint32_t)(((G - kPBufs) / kPBufs) & 1)))
      return false;
    const uint32_t prow = p_base + pb * kPBuf + tid * 128;
    const int sw = tid & 7;
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      if (ch < N / 8)
        st_shared_v4(prow + ((ch ^ sw) << 4), pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
      else
        st_shared_v4(prow + ((ch ^ sw) << 4), 0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
    warp_arrive(&sh->p_full[pb]);
  }
  return piece_epilogue<N>(c, r, pi, m, l, grp_uses);
}
__device__ __noinline__ void softmax_role(const Ctx& c) {
  PieceCursor cur;
  cur.init(&c.ps, c.ng, c.hk, c.t_begin, c.t_end);
  auto fill = [&](PieceRows& r) -> bool {
    if (!cur.next(r.g, r.h, r.lo, r.hi, r.nb, r.ustart)) return false;
    r.first_row = c.ps.gfirst[r.g];
    r.nrows = c.ps.gfirst[r.g + 1] - r.first_row;
    r.nq = r.nrows * c.gqa;
    return true;
  };
  uint32_t grp_uses = 0;
  int G = 0;
  PieceRows r;
  for (int pi = 0; fill(r); ++pi) {
    bool ok;
    switch (s_cols(r.nq)) {
      case 16: ok = softmax_piece<16>(c, r, G, pi, grp_uses); break;
      case 32: ok = softmax_piece<32>(c, r, G, pi, grp_uses); break;
      case 48: ok = softmax_piece<48>(c, r, G, pi, grp_uses); break;
      default: ok = softmax_piece<64>(c, r, G, pi, grp_uses); break;
    }
    if (!ok) break;
    G += stages_of(r.lo, r.hi);
  }
}

__global__ void __launch_bounds__(kVThreads, 1)
    verify_attn_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                       const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ VerifyArgs args) {
  const AttnParams& p = args.p;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  VerifyShared* sh = reinterpret_cast<VerifyShared*>(smem + kBarOff);
  int* plan_mem = reinterpret_cast<int*>(smem + kPlanOff);
  __shared__ int scratch[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Set-up that reads no input, so that it runs beside the previous launch's tail.
  if (threadIdx.x == 0) {
    for (int i = 0; i < kKRing; ++i) {
      mbar_init(&sh->k_full[i], 1);
      mbar_init(&sh->k_empty[i], 1);
    }
    for (int i = 0; i < kVRing; ++i) {
      mbar_init(&sh->v_full[i], 1);
      mbar_init(&sh->v_empty[i], 1);
    }
    for (int i = 0; i < kFlagSlots; ++i) mbar_init(&sh->flags_full[i], 1);
    for (int i = 0; i < kSBufs; ++i) {
      mbar_init(&sh->s_full[i], 1);
      mbar_init(&sh->s_empty[i], 4);
    }
    for (int i = 0; i < kPBufs; ++i) {
      mbar_init(&sh->p_full[i], 4);
      mbar_init(&sh->pv_done[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh->q_full[i], 1);
      mbar_init(&sh->q_empty[i], 1);
      mbar_init(&sh->grp[i], 4);
    }
    for (int i = 0; i < kOBufs; ++i) {
      mbar_init(&sh->o_full[i], 1);
      mbar_init(&sh->o_empty[i], 4);
    }
    mbar_init(&sh->s_final, 1);
    mbar_init(&sh->pv_final, 1);
    sh->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kSWarp) {
    tmem_alloc(&sh->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (lane == 0) {
    if (warp == kKWarp) tma_prefetch_desc(&tmap_k);
    if (warp == kVWarp) tma_prefetch_desc(&tmap_v);
    if (warp == kSWarp) tma_prefetch_desc(&tmap_q);
  }
  tc_fence_before();
  grid_launch_dependents();
  grid_dependency_wait();  // inputs may come from the previous launch in the stream

  const PlanSmem ps{plan_mem, plan_mem + (p.num_rows + 1), plan_mem + 2 * (p.num_rows + 1),
                    plan_mem + 2 * (p.num_rows + 1) + 8};
  build_plan(ps, scratch, p.seq_ids, p.seq_lens, p.num_rows, p.max_group_rows);  // ends with __syncthreads
  tc_fence_after();
  // The launch context, built once in shared memory: the roles read it from
  // there rather than from a stack copy per thread (local memory).
  if (threadIdx.x == 0) {
    Ctx& c = sh->ctx;
    c.p = &p;
    c.sh = sh;
    c.smem = smem;
    c.ps = ps;
    c.ng = ps.misc[0];
    c.hk = p.num_kv_heads;
    c.gqa = p.num_q_heads / p.num_kv_heads;
    c.group_rows = p.max_group_rows;
    c.oob_row = args.oob_row;
    c.total = (long long)c.hk * ps.gprefix[c.ng];
    c.w = blockIdx.x;
    c.split.gprefix = ps.gprefix;
    c.split.ng = c.ng;
    c.split.hk = c.hk;
    c.split.pc = kPieceCost;
    c.split.vtotal = c.total + (long long)kPieceCost * c.hk * c.ng;
    c.workers = (long long)gridDim.x < c.split.vtotal ? (long long)gridDim.x : c.split.vtotal;
    c.split.workers = c.workers;
    const bool act = c.total > 0 && c.w < c.workers;
    c.t_begin = act ? c.split.begin(c.w) : 0;
    c.t_end = act ? c.split.begin(c.w + 1) : 0;
    c.tmem = sh->tmem_base;
  }
  __syncthreads();
  const Ctx& cs = sh->ctx;
  if (warp >= kSoftmaxWarp0)
    write_nan_rows(p, cs.ps, cs.ng, cs.w * 4 + (warp - kSoftmaxWarp0), (long long)gridDim.x * 4);
  const bool active = cs.total > 0 && cs.w < cs.workers;

  if (active) {
    if (warp == kKWarp) {
      producer(cs, &tmap_k, sh->k_full, sh->k_empty, kKOff, kKRing, true);
    } else if (warp == kVWarp) {
      producer(cs, &tmap_v, sh->v_full, sh->v_empty, kVOff, kVRing, false);
    } else if (warp == kSWarp) {
      if (lane == 0) s_issuer(cs, &tmap_q);
    } else if (warp == kPVWarp) {
      if (lane == 0) pv_issuer(cs);
    } else {
      softmax_role(cs);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kSWarp) tmem_dealloc(cs.tmem, kTmemCols);
}

// ------------------------------------------------------------------ host side
long long verify_workers(int device) { return num_sms(device); }

int verify_max_rows() { return kVerifyMaxRows; }

// Rows of one request per unit: a unit's gqa x rows query columns are the N of
// its S^T tile and of the P V product, at most 64.
int verify_group_rows(int gqa) {
  if (gqa < 1 || gqa > kMaxGqa) return 0;
  return kMaxQ / gqa;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// fp16 tensor map with 128-byte swizzle, cached by its full description.
static int tensor_map(CUtensorMap* map, const void* base, int rank, const unsigned long long* dims,
                      const unsigned long long* strides, const unsigned* box) {
  struct Entry {
    const void* base;
    int rank;
    unsigned long long dims[3], strides[2];
    unsigned box[3];
    CUtensorMap map;
  };
  static std::mutex mu;
  static Entry cache[32];
  static int next = 0;
  auto same = [&](const Entry& e) {
    if (e.base != base || e.rank != rank) return false;
    for (int i = 0; i < rank; ++i)
      if (e.dims[i] != dims[i] || e.box[i] != box[i] || (i + 1 < rank && e.strides[i] != strides[i])) return false;
    return true;
  };
  {
    std::lock_guard<std::mutex> lock(mu);
    for (auto& e : cache)
      if (same(e)) {
        *map = e.map;
        return NEB_OK;
      }
  }
  auto fn = encode_fn();
  NEB_REQUIRE(fn != nullptr, NEB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t d[3] = {0, 0, 0}, st[2] = {0, 0};
  cuuint32_t bx[3] = {0, 0, 0}, estr[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    if (i + 1 < rank) st[i] = strides[i];
  }
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<void*>(base), d, st, bx, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  NEB_REQUIRE(r == CUDA_SUCCESS, NEB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  std::lock_guard<std::mutex> lock(mu);
  Entry& e = cache[next];
  e.base = base;
  e.rank = rank;
  for (int i = 0; i < 3; ++i) {
    e.dims[i] = i < rank ? dims[i] : 0;
    e.box[i] = i < rank ? box[i] : 0;
    if (i < 2) e.strides[i] = i + 1 < rank ? strides[i] : 0;
  }
  e.map = *map;
  next = (next + 1) % 32;
  return NEB_OK;
}

int launch_verify(const AttnParams& p, long long workers, cudaStream_t stream) {
  const int gqa = p.num_q_heads / p.num_kv_heads;
  const unsigned long long rows =
      (unsigned long long)p.num_blocks * p.num_layers * p.num_kv_heads * kBlockTokens;
  NEB_REQUIRE(rows + kBlockTokens < (1ull << 31), NEB_ERR_UNSUPPORTED,
              "KV cache of %llu rows exceeds the verify kernel's 2^31-row tensor map", rows);
  NEB_REQUIRE(p.num_rows <= kVerifyMaxRows, NEB_ERR_UNSUPPORTED,
              "verify attention takes at most %d rows per call (got %d)", kVerifyMaxRows, p.num_rows);
  NEB_REQUIRE(gqa >= 1 && gqa <= kMaxGqa && p.max_group_rows >= 1 && p.max_group_rows <= verify_group_rows(gqa),
              NEB_ERR_INVALID, "a unit's query columns exceed the MMA tile");
  NEB_REQUIRE(p.nq >= gqa * p.max_group_rows, NEB_ERR_INVALID, "partial rows per slot below the unit size");
  NEB_REQUIRE((reinterpret_cast<uintptr_t>(p.q) & 15u) == 0, NEB_ERR_INVALID, "q must be 16-byte aligned");
  CUtensorMap tk, tv, tq;
  {
    const unsigned long long dims[2] = {128, rows}, strides[1] = {256};
    const unsigned box[2] = {64, 16};
    int rc = tensor_map(&tk, p.k_cache, 2, dims, strides, box);
    if (rc != NEB_OK) return rc;
    rc = tensor_map(&tv, p.v_cache, 2, dims, strides, box);
    if (rc != NEB_OK) return rc;
  }
  {
    // Q as [rows][q heads][128]: a box is one unit's query columns, gqa heads x group_rows rows.
    const unsigned long long dims[3] = {128, (unsigned long long)p.num_q_heads, (unsigned long long)p.num_rows};
    const unsigned long long strides[2] = {256, 256ull * p.num_q_heads};
    const unsigned box[3] = {64, (unsigned)gqa, (unsigned)p.max_group_rows};
    int rc = tensor_map(&tq, p.q, 3, dims, strides, box);
    if (rc != NEB_OK) return rc;
  }
  VerifyArgs a;
  a.p = p;
  a.oob_row = (int)rows;
  const size_t smem = verify_smem_bytes(p.num_rows);
  int device = 0;
  NEB_CUDA(cudaGetDevice(&device));
  NEB_REQUIRE(device >= 0 && device < 64, NEB_ERR_UNSUPPORTED, "device index %d out of range", device);
  static bool attr_set[64] = {};
  static std::mutex attr_mu;
  {
    std::lock_guard<std::mutex> lock(attr_mu);
    if (!attr_set[device]) {
      NEB_CUDA(cudaFuncSetAttribute(verify_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)verify_smem_bytes(kVerifyMaxRows)));
      attr_set[device] = true;
    }
  }
  // Programmatic stream serialisation: the launch may start while the previous
  // kernel in the stream finishes; the kernel waits for it (griddepcontrol.wait)
  // before it reads any input.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)workers);
  cfg.blockDim = dim3(kVThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  NEB_CUDA(cudaLaunchKernelEx(&cfg, verify_attn_kernel, tk, tv, tq, a));
  return NEB_OK;
}

}  // namespace vlong
}  // namespace neb
