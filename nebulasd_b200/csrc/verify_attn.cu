// Target verify attention on tcgen05 tensor cores (sm_100a).
//
// Replaces swiftLLM's paged decode attention as it is driven by Target verify
// (swiftLLM/swiftllm/worker/kernels/paged_attn.py:9-222 called with the k+1
// rows per request built in nebulasd/src/nebulasd/workers/target/backend.py:102-111).
// The reference runs one single-warp program per (row, q head, split), so a KV
// tile is read GQA*(k+1) times (20x for Qwen3-8B at k=4) and the dot products
// run on CUDA cores.  Here the GQA q heads of a kv head and the adjacent rows
// of one request (up to 64 query rows) are the M dimension of one MMA tile:
// every KV tile is staged once into shared memory by TMA and consumed by the
// tensor cores for all of them.
//
// One persistent CTA per SM (the driver places a single CTA that allocates
// tensor memory on an SM); plan.cuh gives each an equal share of KV tiles.
// Work moves in 64-token stages (four 16-token blocks); K and V move by TMA in
// ring slots of two stages (one transaction count and one wait per 32 KB).
// The roles wait only on their own inputs:
//   warp 0      K producer: per 16-token block two 64-column TMA boxes
//               (128-byte swizzle), one lane per box, into the K ring, once S
//               of the stages that last used the slot is done; publishes each
//               stage's block flags.  Block-table rows are fetched two 32-tile
//               batches ahead.
//   warp 1      S issuer (one thread): Q of the next piece by TMA into the
//               other half of a double buffer; S = Q K^T per stage into one of
//               four TMEM tiles (M=64, N=64), so that it runs ahead of the
//               softmax.
//   warps 2..5  softmax / epilogue: read a stage's S with tcgen05.ld, masked
//               online softmax in the exp2 domain (O is rescaled only when a
//               row's max grows by more than 2^8), P as fp16 in shared memory,
//               row sums of that P in fp32 registers; at the end of a piece
//               normalise O and store it, or store or merge a partial.
//   warp 6      V producer: the V boxes into the V ring, once P V of the
//               stages that last used the slot is done.
//   warp 7      P V issuer (one thread): O += P V (V an MN-major operand) into
//               a TMEM accumulator (M=64, N=128).
// A unit split across CTAs is merged by the CTA that finishes it last (see
// piece_epilogue and finish_units).
//
// Each role is an out-of-line function and the two producers share one, so
// that the instruction cache holds every warp's hot loop at once: with more
// code than that, the warps of an SM stall on instruction fetch.
//
// Query rows: a unit of nrows rows and gqa heads per row is cut into four
// chunks of c = gqa*ceil(nrows/4) rows; chunk q goes to MMA rows 16q.. (TMEM
// lane quadrant q, where an M=64 accumulator keeps rows 16q..16q+15), so one
// 3D TMA box per chunk loads Q and each softmax warp owns one chunk.
//
// Every wait is bounded (about 2 s); on expiry the kernel records an error
// bit, stops issuing work, waits (bounded) for its own copies and MMAs, frees
// its TMEM and returns.  No TMA multicast is used.  The kernel is launched
// with programmatic stream serialisation: it lets the next launch in the
// stream be scheduled as soon as it starts, and waits (griddepcontrol.wait)
// for the previous one before it reads any input, so that the launch gap and
// the previous launch's tail overlap.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "attn_common.cuh"
#include "sm100.cuh"

namespace neb {
using namespace sm100;

constexpr int kVThreads = 384;  // 12 warps: 0 K, 1 S, 2-5 softmax, 6 V, 7 P V, 8-11 epilogue
constexpr int kKWarp = 0;
constexpr int kSWarp = 1;
constexpr int kSoftmaxWarp0 = 2;
constexpr int kSoftmaxThreads = 128;
constexpr int kEpiWarp0 = 8;                              // epilogue warps: TMEM lane quadrants 0..3
constexpr int kEpiThreads = 128;
constexpr int kVWarp = 6;
constexpr int kPVWarp = 7;
constexpr int kStageBlocks = 8;                           // 16-token KV blocks per stage
constexpr int kStageCols = kStageBlocks * kBlockTokens;   // tokens per stage: the S tile's N
constexpr int kStageR = kStageCols / 8;                   // 8-column groups of an S tile
constexpr int kSlotStages = 1;                            // stages per K (V) ring slot: one TMA phase
constexpr int kKRing = 2;                                 // slots of the K ring
constexpr int kVRing = 2;                                 // slots of the V ring
constexpr int kSBufs = 2;                                 // S tiles in TMEM (the S issuer runs ahead)
constexpr int kFlagSlots = kSlotStages * kKRing + kSBufs;  // block-flag ring (see the K producer)
constexpr int kMaxQRows = 64;                             // query rows per unit: the MMA's M
constexpr int kMaxGqa = 16;                               // a row's heads fit one 16-row chunk
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSBuf = 128;                           // S tile b at columns 128*b
constexpr uint32_t kOCol = 256;                           // O of piece i: 128 columns at kOCol + 128 * (i % 2)
constexpr long long kWaitLimit = 4000000000LL;
constexpr int kMaxDirectOthers = 3;                      // direct merge: at most 3 other pieces
constexpr int kPieceCost = 8;                             // a piece's fixed cost, in tiles (plan.cuh CostSplit)
static_assert(kStageCols <= (int)kSBuf && kStageR % 2 == 0 && kSBufs * kSBuf <= kOCol && kOCol + 256 <= kTmemCols,
              "S tiles and both O buffers fit TMEM");
static_assert(kSlotStages == 1 && kStageBlocks == 8 && 2 * kSlotStages * kStageBlocks <= 32,
              "the producers fill a slot with one stage, one 64-column box per lane");

// Shared memory map (offsets from a 1024-byte aligned base).
constexpr uint32_t kQHalf = kMaxQRows * 128;       // one 64-column half of Q
constexpr uint32_t kQBuf = 2 * kQHalf;             // Q of one piece
constexpr uint32_t kQOff = 0;                      // two Q buffers
constexpr uint32_t kHalf = kStageBlocks * 2048;    // one 64-column half of K or V of a stage
constexpr uint32_t kStageBytes = 2 * kHalf;        // one stage of K (or V): both halves
constexpr uint32_t kSlotBytes = kSlotStages * kStageBytes;  // a ring slot
constexpr uint32_t kKOff = kQOff + 2 * kQBuf;
constexpr uint32_t kVOff = kKOff + kKRing * kSlotBytes;
constexpr uint32_t kPAtom = kMaxQRows * 128;       // 64 rows x 64 fp16 of P (one swizzle column)
constexpr uint32_t kPBuf = ((kStageCols + 63) / 64) * kPAtom;
constexpr uint32_t kPOff = kVOff + kVRing * kSlotBytes;
constexpr uint32_t kStatOff = kPOff + 2 * kPBuf;   // row max and sum of a piece: [2][64] float2
constexpr uint32_t kFeedOff = kStatOff + 2 * kMaxQRows * 8;  // the first 96 tiles' table entries (plan cache)
constexpr uint32_t kBarOff = kFeedOff + 1024;
constexpr uint32_t kPlanOff = kBarOff + 1024;
static_assert(kHalf % 1024 == 0, "swizzle atoms stay 1024-byte aligned");

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
  int ng, hk, gqa, oob_row;
  long long total, workers, w, t_begin, t_end;
  CostSplit split;  // which worker owns which tiles
  uint32_t tmem;
  int g_begin;          // group of tile t_begin
  bool pc_hit;          // the plan came from the plan cache (and so did feed_cache)
  uint32_t seq;         // launch number (plan cache)
  int32_t* pc_entry;    // this worker's entry in the slot written for the next call (null: none)
};

struct VerifyShared {
  AttnParams prm;                // the call's parameters, copied in before the inputs are read
  Ctx ctx;                       // the launch context, written once by warp 0
  uint64_t k_full[kKRing];       // K of the slot's stages landed
  uint64_t k_empty[kKRing];      // S of the slot's stages completed (one arrival per stage)
  uint64_t v_full[kVRing];       // V of the slot's stages landed
  uint64_t v_empty[kVRing];      // P V of the slot's stages completed (one arrival per stage)
  uint64_t flags_full[kFlagSlots];
  uint64_t s_full[kSBufs];
  uint64_t s_empty[kSBufs];
  uint64_t p_full[2];
  uint64_t pv_done[2];
  uint64_t q_full[2];
  uint64_t q_empty[2];
  uint64_t o_full[2];            // P V of piece i's last stage done: O buffer i % 2 complete
  uint64_t o_empty[2];           // the epilogue read O buffer i % 2 (one arrival per epilogue warp)
  uint64_t st_full[2];           // the softmax wrote piece i's row statistics (one arrival per warp)
  uint64_t st_empty[2];          // the epilogue read them
  uint64_t plan_ready;           // warp 0 wrote the plan and the context
  uint64_t s_final;
  uint64_t pv_final;
  uint32_t tmem_base;
  int32_t abort_flag;
  int32_t merge_mode;            // epilogue of the last piece: merge directly with the other partial
  long long cached_begin, cached_end;  // this worker's tile range from the plan cache
  int32_t cached_group;          // and the group of its first tile
  int32_t first_last;            // the first piece's count completed its unit: merge it at the end
  int32_t last_merge;            // the last piece's count completed its unit: merge it at the end
  int32_t lm_g, lm_h;            // that unit's group and kv head
  long long lm_w0, lm_w1;        // and its first and last workers
  int32_t blk[kFlagSlots][kStageBlocks];
};
static_assert(sizeof(VerifyShared) <= 1024, "barrier block fits its slot");

__host__ __device__ inline size_t verify_smem_bytes(int num_rows) {
  return 1024 + kPlanOff + plan_smem_bytes(num_rows, true);
}

struct VerifyArgs {
  AttnParams p;
  int oob_row;   // first row past the end of the K/V tensor maps (loads there return zeros)
  uint32_t seq;  // launch number on this workspace (plan cache slots)
};


// The pieces of one worker: a cursor over its tile range (plan.cuh).
struct PieceCursor {
  const PlanSmem* ps;
  int ng, hk, g;
  long long t, t_end;
  // g0: the group of tile `begin` when known, else -1.
  __device__ __noinline__ void init(const PlanSmem* planp, int ngroups, int kvh, long long begin, long long end,
                                    int g0 = -1) {
    ps = planp;
    ng = ngroups;
    hk = kvh;
    t = begin;
    t_end = end;
    g = begin >= end ? 0 : g0 >= 0 ? g0 : find_group(ps->gprefix, ng, begin, hk);
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

// Query rows per TMEM lane quadrant for a group of `nrows` rows.
__device__ __forceinline__ int rows_per_quad(int nrows) { return (nrows + 3) >> 2; }

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

__device__ __forceinline__ uint32_t pack_half2(float a, float b) { return f2_to_h2(a, b); }

__device__ __forceinline__ void scale_rows(uint32_t* r, int n4, float alpha_a, float alpha_b) {
#pragma unroll
  for (int i = 0; i < n4; ++i) {
    r[4 * i + 0] = __float_as_uint(__uint_as_float(r[4 * i + 0]) * alpha_a);
    r[4 * i + 1] = __float_as_uint(__uint_as_float(r[4 * i + 1]) * alpha_a);
    r[4 * i + 2] = __float_as_uint(__uint_as_float(r[4 * i + 2]) * alpha_b);
    r[4 * i + 3] = __float_as_uint(__uint_as_float(r[4 * i + 3]) * alpha_b);
  }
}

// Exchanges the two query rows a thread holds in a 16x256b TMEM load
// (row a in registers 4r, 4r+1; row b in 4r+2, 4r+3).
template <int N>
__device__ __forceinline__ void swap_rows_n(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const uint32_t t0 = r[4 * i], t1 = r[4 * i + 1];
    r[4 * i] = r[4 * i + 2];
    r[4 * i + 1] = r[4 * i + 3];
    r[4 * i + 2] = t0;
    r[4 * i + 3] = t1;
  }
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
  // resolve() reads the block-table entry.
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
  __device__ __forceinline__ void resolve(const Pending& q, int& r, int& v) const {
    r = oob_row;
    v = 0;
    if (!q.in_range) return;
    const long long blk = lookup_block(*p, q.sid, q.tile);
    if (blk >= 0) {
      v = 1;
      r = (int)(((blk * p->num_layers + p->cur_layer) * p->num_kv_heads + q.kv_head) * kBlockTokens);
    }
  }
  __device__ __forceinline__ void fetch(long long bt, int& r, int& v) const { resolve(locate(bt), r, v); }
  // A lane's tile as one word: its block-table position times 256 plus its
  // kv head, -1 for no table entry, -2 for a tile past max_blocks_per_seq.
  // The first three batches' words are what the plan cache keeps per worker.
  __device__ __forceinline__ long long entry(const Pending& q) const {
    if (!q.in_range || q.sid < 0 || q.sid >= p->bt_rows) return -1;
    if (q.tile >= p->mbs) return -2;
    return (((long long)q.sid * p->mbs + q.tile) << 8) | q.kv_head;
  }
  __device__ __forceinline__ void finish_entry(long long e, long long blk, uint32_t& err, int& r, int& v) const {
    r = oob_row;
    v = 0;
    if (e == -2) err |= kErrTooManyBlocks;
    if (e < 0) return;
    if (blk < 0 || blk >= p->num_blocks) {
      err |= kErrBlockIndex;
      return;
    }
    v = 1;
    r = (int)(((blk * p->num_layers + p->cur_layer) * p->num_kv_heads + (int)(e & 255)) * kBlockTokens);
  }
  // The first three batches, from the words in `cached` ([3][32], as left by
  // an earlier call) or located here; `e` returns this lane's words.
  __device__ void init(const AttnParams* pp, const PlanSmem* pps, int ngroups, int oob, long long begin,
                       long long end, const long long* cached, long long* e) {
    p = pp;
    ps = pps;
    ng = ngroups;
    oob_row = oob;
    t_end = end;
    base = begin;
    const int lane = threadIdx.x & 31;
    if (cached) {
#pragma unroll
      for (int k = 0; k < 3; ++k) e[k] = cached[32 * k + lane];
    } else {
#pragma unroll
      for (int k = 0; k < 3; ++k) e[k] = entry(locate(base + 32 * k));
    }
    uint32_t err = 0;
    const long long b0 = e[0] >= 0 ? (long long)__ldg(p->block_table + (e[0] >> 8)) : 0;
    const long long b1 = e[1] >= 0 ? (long long)__ldg(p->block_table + (e[1] >> 8)) : 0;
    const long long b2 = e[2] >= 0 ? (long long)__ldg(p->block_table + (e[2] >> 8)) : 0;
    finish_entry(e[0], b0, err, r0, v0);
    finish_entry(e[1], b1, err, r1, v1);
    finish_entry(e[2], b2, err, r2, v2);
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

// The first piece of a worker's range (a unit split across CTAs): its group,
// kv head and the unit's first and last workers, for the merge at the end
// when counting this piece in completed the unit.
struct FirstSplit {
  long long w0, w1;
  int g, h;
  __device__ __noinline__ void init(const Ctx& c) {
    PieceCursor cur;
    cur.init(&c.ps, c.ng, c.hk, c.t_begin, c.t_end, c.g_begin);
    int lo, hi, nb;
    long long ustart;
    cur.next(g, h, lo, hi, nb, ustart);
    w0 = c.split.worker_of_tile(ustart);
    w1 = c.split.worker_of_tile(ustart + nb - 1);
  }
};

// ------------------------------------------------------------------ producers
// One function serves the K warp (flags != 0: it also publishes the block
// flags) and the V warp, over a ring of `ring` slots (kKRing, kVRing) of one
// 128-token stage each: one TMA phase per slot, so that each wait and
// transaction count covers 32 KB.  Stage G sits in slot G % ring; the slot
// frees when the MMAs that read it (S for K, P V for V) are done.  The block
// flags of stage G go to flag slot G % kFlagSlots.  Before the flags of stage
// G are written, the slot that held stage G - kKRing has been freed, so S of
// that stage was issued, which needed S buffer (G - kKRing) % kSBufs released
// by the softmax of stage G - kKRing - kSBufs, and the softmax reads a stage's
// flags before it releases its S: flag slots with kFlagSlots >= kKRing +
// kSBufs are free.
__device__ __noinline__ void producer(const Ctx& c, const CUtensorMap* tmap, uint64_t* full, uint64_t* empty,
                                      uint32_t ring_off, int ring, int flags) {
  const AttnParams& p = *c.p;
  VerifyShared* sh = c.sh;
  const int lane = threadIdx.x & 31;
  // K and V tiles are read once: let them leave L2 first, so that the kernel's
  // code, the plan inputs, q and the merge partials stay cached.
  const uint64_t kv_policy = l2_evict_first_policy();
  TileFeed feed;
  long long e[3];
  feed.init(&p, &c.ps, c.ng, c.oob_row, c.t_begin, c.t_end, c.pc_hit ? reinterpret_cast<const long long*>(c.smem + kFeedOff) : nullptr, e);
  // The worker's stages in order, as block counts: each piece cut into
  // kStageBlocks-block stages (the last one of a piece may be shorter).
  PieceCursor cur;
  cur.init(&c.ps, c.ng, c.hk, c.t_begin, c.t_end, c.g_begin);
  int s_lo = 0, s_hi = 0;
  auto next_stage = [&](int& nblk) -> bool {
    if (s_lo >= s_hi) {
      int g, h, nb;
      long long ustart;
      if (!cur.next(g, h, s_lo, s_hi, nb, ustart)) return false;
    }
    nblk = min(kStageBlocks, s_hi - s_lo);
    s_lo += nblk;
    return true;
  };
  // Lane l < 16 carries box l of the stage: tile l & 7, half l >> 3.
  const int b = lane & (kStageBlocks - 1), hf = lane >> 3;
  int G = 0, slot = 0, used = 0;  // the stage, its slot, slots filled so far
  uint32_t phase = 0;             // parity of the slot's current use
  long long pos = c.t_begin;
  int n0 = 0;
  bool more = next_stage(n0);
  while (more) {
    int row, valid;
    feed.get_lane(pos, b, row, valid);
    int waited = 1;
    if (lane == 0) {
      waited = wait_or_abort(sh, p, &empty[slot], phase ^ 1u);
      if (waited) {
        mbar_arrive_expect_tx(&full[slot], (uint32_t)n0 * 2u * 2048u);
      }
    }
    waited = __shfl_sync(0xffffffffu, waited, 0);
    if (waited) {
      // One lane per 64-column box, so that the stage's loads leave together.
      if (hf < 2 && b < n0)
        tma_load_2d_hint(c.smem + ring_off + slot * kSlotBytes + hf * kHalf + b * 2048, tmap, &full[slot], 64 * hf,
                         row, kv_policy);
      if (flags) {
        if (hf == 0) sh->blk[G % kFlagSlots][b] = b < n0 ? valid : 0;
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh->flags_full[G % kFlagSlots]);
      }
    }
    // Once the first loads are on their way, the K warp leaves its range for
    // the next call.
    if (flags && G == 0 && c.pc_entry) {
#pragma unroll
      for (int k = 0; k < 3; ++k) reinterpret_cast<long long*>(c.pc_entry + kPcEntryFeed)[32 * k + lane] = e[k];
      if (lane == 0) {
        c.pc_entry[1] = c.g_begin;
        *reinterpret_cast<long long*>(c.pc_entry + 2) = c.t_begin;
        *reinterpret_cast<long long*>(c.pc_entry + 4) = c.t_end;
        c.pc_entry[0] = (int32_t)c.seq;
      }
    }
    if (!waited) break;
    ++used;
    pos += n0;
    feed.advance(pos);
    ++G;
    if (++slot == ring) {
      slot = 0;
      phase ^= 1u;
    }
    more = next_stage(n0);
  }
  // Wait (bounded) for every copy this warp issued before the CTA can exit.
  if (lane == 0)
#pragma unroll 1
    for (int u = (used > ring ? used - ring : 0); u < used; ++u)
      mbar_wait(&full[u % ring], (uint32_t)((u / ring) & 1), kWaitLimit);
}


// At the very end, the whole CTA merges the partials of the units its counts
// completed: the first piece's (its other parts finished first) and the last
// piece's (its count came last).
__device__ __noinline__ void finish_units(const Ctx& c) {
  const VerifyShared* sh = c.sh;
  __threadfence();
  if (sh->first_last) {
    FirstSplit fs;
    fs.init(c);
    const int first_row = c.ps.gfirst[fs.g];
    merge_unit_threads<2>(*c.p, first_row, c.ps.gfirst[fs.g + 1] - first_row, fs.h, c.gqa, fs.w0, fs.w1,
                          threadIdx.x, kVThreads);
  }
  if (sh->last_merge) {
    const int first_row = c.ps.gfirst[sh->lm_g];
    merge_unit_threads<2>(*c.p, first_row, c.ps.gfirst[sh->lm_g + 1] - first_row, sh->lm_h, c.gqa, sh->lm_w0,
                          sh->lm_w1, threadIdx.x, kVThreads);
  }
}

// ------------------------------------------------------------------- S issuer
// Q of piece i goes to buffer i % 2 as soon as piece i - 2 is done with it,
// i.e. a whole piece ahead of its first S.
struct QFeeder {
  PieceCursor cur;
  int qi, qg, qh, qlo, qhi, qnb;
  long long qus;
  bool qhave;
  // Issues the Q loads that may go now; blocks only for piece `need`.
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
      const int first_row = c.ps.gfirst[qg];
      const int nrows = c.ps.gfirst[qg + 1] - first_row;
      const int rq = rows_per_quad(nrows);
      const int nquads = (nrows + rq - 1) / rq;
      // A box is gqa heads x 16 / gqa rows of 64 columns (fewer than 16 rows
      // when gqa does not divide 16); rows past the tensor count as loaded.
      const uint32_t box_bytes = (uint32_t)(c.gqa * (16 / c.gqa)) * 128u;
      mbar_arrive_expect_tx(&sh->q_full[b], (uint32_t)nquads * 2u * box_bytes);
#pragma unroll 1
      for (int q = 0; q < nquads; ++q)
        for (int dh = 0; dh < 2; ++dh)
          tma_load_3d(c.smem + kQOff + b * kQBuf + dh * kQHalf + q * 16 * 128, tmap_q, &sh->q_full[b], dh * 64,
                      qh * c.gqa, first_row + q * rq);
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
  qf.cur.init(&c.ps, c.ng, c.hk, c.t_begin, c.t_end, c.g_begin);
  qf.qi = 0;
  qf.qhave = qf.cur.next(qf.qg, qf.qh, qf.qlo, qf.qhi, qf.qnb, qf.qus);
  PieceCursor cur;
  cur.init(&c.ps, c.ng, c.hk, c.t_begin, c.t_end, c.g_begin);
  int g, h, lo, hi, nb;
  long long ustart;
  int G = 0;
  bool ok = true;
  for (int piece = 0; ok && cur.next(g, h, lo, hi, nb, ustart); ++piece) {
    const int nst = stages_of(lo, hi);
    const int b = piece & 1;
    if (!qf.feed(c, tmap_q, piece, piece) || !wait_or_abort(sh, p, &sh->q_full[b], (uint32_t)((piece >> 1) & 1)))
      break;
    const uint32_t qb = q_base + b * kQBuf;
    for (int s = 0; s < nst; ++s, ++G) {
      const int slot = (G / kSlotStages) % kKRing, sb = G % kSBufs;
      if (!wait_or_abort(sh, p, &sh->k_full[slot], (uint32_t)((G / kSlotStages / kKRing) & 1)) ||
          !wait_or_abort(sh, p, &sh->s_empty[sb], (uint32_t)(((G / kSBufs) & 1) ^ 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int nblk = min(kStageBlocks, hi - (lo + s * kStageBlocks));
      const uint32_t idesc_s = idesc_f16_f32(kMaxQRows, 16 * nblk, false, false);
      const uint32_t kst = k_base + slot * kSlotBytes + (G % kSlotStages) * kStageBytes;
      // Descriptors of the eight K=16 steps: the base's address field plus
      // a constant (shared-memory addresses / 16 stay below 2^14).
      const uint64_t a0 = smem_desc_sw128(qb, 16, 1024), b0 = smem_desc_sw128(kst, 16, 1024);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16(tmem + sb * kSBuf, a0 + (((kk >> 2) * kQHalf + (kk & 3) * 32) >> 4),
                b0 + (((kk >> 2) * kHalf + (kk & 3) * 32) >> 4), idesc_s, kk > 0 ? 1u : 0u);
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
__device__ __noinline__ void pv_issuer(const Ctx& c) {
  const AttnParams& p = *c.p;
  VerifyShared* sh = c.sh;
  const uint32_t v_base = smem_u32(c.smem + kVOff);
  const uint32_t p_base = smem_u32(c.smem + kPOff);
  const uint32_t idesc_pv = idesc_f16_f32(kMaxQRows, 128, false, true);
  const uint32_t tmem = c.tmem;
  PieceCursor cur;
  cur.init(&c.ps, c.ng, c.hk, c.t_begin, c.t_end, c.g_begin);
  int g, h, lo, hi, nb;
  long long ustart;
  int G = 0;
  bool ok = true;
  for (int piece = 0; ok && cur.next(g, h, lo, hi, nb, ustart); ++piece) {
    const int nst = stages_of(lo, hi);
    const int ob = piece & 1;
    const uint32_t ocol = tmem + kOCol + 128u * ob;
    for (int s = 0; s < nst; ++s, ++G) {
      const int slot = (G / kSlotStages) % kVRing, sb = G & 1;
      // O buffer ob is free once the epilogue of piece - 2 has read it.
      if (!wait_or_abort(sh, p, &sh->p_full[sb], (uint32_t)((G >> 1) & 1)) ||
          !wait_or_abort(sh, p, &sh->v_full[slot], (uint32_t)((G / kSlotStages / kVRing) & 1)) ||
          (s == 0 && piece >= 2 && !wait_or_abort(sh, p, &sh->o_empty[ob], (uint32_t)(((piece - 2) >> 1) & 1)))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int nblk = min(kStageBlocks, hi - (lo + s * kStageBlocks));
      const uint32_t vst = v_base + slot * kSlotBytes + (G % kSlotStages) * kStageBytes;
      const uint64_t pa0 = smem_desc_sw128(p_base + sb * kPBuf, 16, 1024);
      const uint64_t vb0 = smem_desc_sw128(vst, kHalf, 1024);
#pragma unroll
      for (int kb = 0; kb < kStageBlocks; ++kb) {
        if (kb < nblk) {
          const uint64_t a = pa0 + (((kb >> 2) * kPAtom + (kb & 3) * 32) >> 4);
          const uint32_t acc = (s == 0 && kb == 0) ? 0u : 1u;
          mma_f16(ocol, a, vb0 + ((kb * 2048) >> 4), idesc_pv, acc);
        }
      }
      mma_commit(&sh->v_empty[slot]);
      mma_commit(&sh->pv_done[sb]);
      if (s == nst - 1) mma_commit(&sh->o_full[ob]);
    }
  }
  mma_commit(&sh->pv_final);
  mbar_wait(&sh->pv_final, 0, kWaitLimit);
}

// -------------------------------------------------------------------- softmax
// O times (alpha_a, alpha_b), in TMEM (rare: a row's max grew by more than 2^8).
__device__ __noinline__ void rescale_o(uint32_t ocol, uint32_t lane_addr, float alpha_a, float alpha_b) {
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    uint32_t orr[32];
    const uint32_t oaddr = ocol + half * 64 + lane_addr;
    tmem_ld_16x256b_x8(oaddr, orr);
    tmem_wait_ld();
    scale_rows(orr, 8, alpha_a, alpha_b);
    tmem_st_16x256b_x8(oaddr, orr);
  }
  tmem_wait_st();
}

// The rows a softmax or epilogue thread owns in a piece (the two warps of
// one TMEM lane quadrant own the same rows).
struct SoftmaxRows {
  int g, h, lo, hi, nb;
  long long ustart;
  int ja, jb, len_a, len_b;  // unit rows (-1: none) and their lengths
};

// Epilogue of piece `piece` (run by the epilogue warps while the softmax warps
// go on with the next piece): O / l as fp16 output rows, or, for a unit split
// across CTAs, a partial (O / l and m + log2 l).  m and l are the rows' final
// max and sum.  The last piece of the CTA's range first looks at the unit's
// counter: when the other pieces have been counted in already, it merges
// their partials with its own O directly.  Otherwise it writes its partial
// and counts it in; the count that completes a unit leaves the merge of its
// partials to the whole CTA at the end (finish_units).  The PV issuer may
// reuse the piece's O buffer once it has been read.
__device__ __noinline__ bool piece_epilogue(const Ctx& c, const SoftmaxRows& r, int piece, float m_a, float m_b,
                                            float l_a, float l_b, bool last_piece) {
  const AttnParams& p = *c.p;
  VerifyShared* sh = c.sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tid = threadIdx.x - kEpiWarp0 * 32;
  const int q4 = lane & 3;
  const uint32_t lane_addr = (uint32_t)(32 * (warp & 3)) << 16;
  const int gqa = c.gqa;
  const bool whole = (r.lo == 0 && r.hi == r.nb);
  const int first_row = c.ps.gfirst[r.g];
  long long w0 = 0, w1 = 0, slot = 0, unit = 0;
  bool direct = false;
  if (!whole) {
    w0 = c.split.worker_of_tile(r.ustart);
    w1 = c.split.worker_of_tile(r.ustart + r.nb - 1);
    slot = piece_slot(c.w, w0);
    unit = (long long)r.g * c.hk + r.h;
    // The counter is read while the last P V still runs.
    if (last_piece && w1 - w0 <= kMaxDirectOthers) {
      if (tid == 0) sh->merge_mode = ld_acquire_gpu(p.counters + unit) == (int)(w1 - w0);
      named_bar_sync(2, kEpiThreads);
      direct = sh->merge_mode != 0;
    }
  }
  const int ob = piece & 1;
  if (!wait_or_abort(sh, p, &sh->o_full[ob], (uint32_t)((piece >> 1) & 1))) return false;
  tc_fence_after();
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    uint32_t o[32];
    tmem_ld_16x256b_x8(c.tmem + kOCol + 128u * ob + half * 64 + lane_addr, o);
    tmem_wait_ld();
    if (half == 1) {
      tc_fence_before();
      warp_arrive(&sh->o_empty[ob]);
    }
#pragma unroll 1
    for (int x = 0; x < 2; ++x) {
      const int j = x == 0 ? r.ja : r.jb;
      if (j >= 0) {
        const float l = x == 0 ? l_a : l_b, m = x == 0 ? m_a : m_b;
        const float inv = 1.f / l;
        const int row = first_row + j / gqa;
        const int head = r.h * gqa + j % gqa;
        __half* out = p.o + ((long long)row * p.num_q_heads + head) * kHeadDim + half * 64;
        if (whole) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<uint32_t*>(out + 8 * i + 2 * q4) =
                pack_half2(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv);
        } else if (!direct) {
          float* dst = p.part_o + (slot * p.nq + j) * kHeadDim + half * 64;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            __stcg(reinterpret_cast<float2*>(dst + 8 * i + 2 * q4),
                   make_float2(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv));
          if (half == 0 && q4 == 0) __stcg(p.part_lse + slot * p.nq + j, l > 0.f ? m + __log2f(l) : neg_inf());
        } else {
          // Log-sum-exp of the unit's pieces in worker order, this one from
          // registers and the others from their partials, with the arithmetic
          // of merge_unit_threads (one round of at most four slots), so that
          // the result does not depend on which path merged the unit.  A
          // piece with no unmasked token (lse -inf) carries no weight; all
          // empty gives 0/0 = NaN, as in the reference.
          constexpr int kN = kMaxDirectOthers + 1;
          float le[kN];
          float2 v[kN][8];
          const int self = (int)(c.w - w0);
#pragma unroll
          for (int k = 0; k < kN; ++k) {
            le[k] = neg_inf();
            if (k == self) {
              le[k] = l > 0.f ? m + __log2f(l) : neg_inf();
#pragma unroll
              for (int i = 0; i < 8; ++i)
                v[k][i] = make_float2(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv);
            } else if (w0 + k <= w1) {
              const long long sk = piece_slot(w0 + k, w0);
              le[k] = __ldcg(p.part_lse + sk * p.nq + j);
              const float* src = p.part_o + (sk * p.nq + j) * kHeadDim + half * 64;
#pragma unroll
              for (int i = 0; i < 8; ++i) v[k][i] = __ldcg(reinterpret_cast<const float2*>(src + 8 * i + 2 * q4));
            }
          }
          float mx = neg_inf();
#pragma unroll
          for (int k = 0; k < kN; ++k) mx = fmaxf(mx, le[k]);
          float den = 0.f;
          float2 acc[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] = make_float2(0.f, 0.f);
          if (mx != neg_inf()) {
#pragma unroll
            for (int k = 0; k < kN; ++k) {
              if (le[k] == neg_inf()) continue;
              const float wt = fast_exp2(le[k] - mx);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                acc[i].x += wt * v[k][i].x;
                acc[i].y += wt * v[k][i].y;
              }
              den += wt;
            }
          }
          const float rden = 1.f / den;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<uint32_t*>(out + 8 * i + 2 * q4) = pack_half2(acc[i].x * rden, acc[i].y * rden);
        }
      }
      swap_rows_n<8>(o);  // row b's values into row a's registers
    }
  }
  if (!whole) {
    if (direct) {
      if (tid == 0) p.counters[unit] = 0;  // the unit is complete: ready for the next call
    } else {
      // Count the partial in (the first piece of a range, or the last); the
      // count that completes the unit leaves its merge to the whole CTA once
      // every role is done.
      named_bar_sync(2, kEpiThreads);  // every partial store precedes thread 0's fence
      if (tid == 0) {
        __threadfence();
        if (atomicAdd(p.counters + unit, 1) == (int)(w1 - w0)) {
          p.counters[unit] = 0;  // every piece has arrived: ready for the next call
          if (!last_piece) {
            sh->first_last = 1;
          } else {
            sh->lm_g = r.g;
            sh->lm_h = r.h;
            sh->lm_w0 = w0;
            sh->lm_w1 = w1;
            sh->last_merge = 1;
          }
        }
      }
    }
  }
  return true;
}

// Scores of one stage in place (sr holds the fp32 bits of a 16x256b TMEM
// load): scaled into the exp2 domain and masked to -inf, and the running max
// of each of the kRows rows this thread holds over its quad.  Element (r, e)
// of row x is sr[4r + 2x + e], at token 8r + 2*q4 + e of the stage; it is
// valid iff 8r + e < lim[x] and its block's flag is set.  Both rows go through
// one pass so that their instruction chains interleave.
template <int kRows>
__device__ __forceinline__ void mask_max_rows(uint32_t* sr, const int* lim, int blk_ok, bool blocks_ok, float sc,
                                              float* mx) {
#pragma unroll
  for (int x = 0; x < kRows; ++x)
#pragma unroll
    for (int r = 0; r < kStageR; ++r)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float v = 8 * r + e < lim[x] ? __uint_as_float(sr[4 * r + 2 * x + e]) * sc : neg_inf();
        sr[4 * r + 2 * x + e] = __float_as_uint(v);
      }
  if (!blocks_ok) {
#pragma unroll
    for (int r = 0; r < kStageR; ++r)
      if (!((blk_ok >> (r >> 1)) & 1))
#pragma unroll
        for (int x = 0; x < kRows; ++x) sr[4 * r + 2 * x] = sr[4 * r + 2 * x + 1] = __float_as_uint(neg_inf());
  }
#pragma unroll
  for (int x = 0; x < kRows; ++x) {
    float t[kStageR];
#pragma unroll
    for (int r = 0; r < kStageR; ++r)
      t[r] = fmaxf(__uint_as_float(sr[4 * r + 2 * x]), __uint_as_float(sr[4 * r + 2 * x + 1]));
#pragma unroll
    for (int w2 = kStageR / 2; w2 >= 1; w2 /= 2)
#pragma unroll
      for (int r = 0; r < w2; ++r) t[r] = fmaxf(t[r], t[r + w2]);
    mx[x] = t[0];
  }
#pragma unroll
  for (int x = 0; x < kRows; ++x) mx[x] = fmaxf(mx[x], __shfl_xor_sync(0xffffffffu, mx[x], 1));
#pragma unroll
  for (int x = 0; x < kRows; ++x) mx[x] = fmaxf(mx[x], __shfl_xor_sync(0xffffffffu, mx[x], 2));
}

// P = 2^(s - m) as fp16 pairs (the MMA operand) into the swizzled P tile for
// the kRows rows of this thread (MMA rows mrow[x]); rows with nothing
// unmasked yet (m = -inf) get zeros.  lsum[x] += the fp32 sum of the fp16
// values stored (the row sum is the sum of exactly the P the MMA reads).
template <int kRows>
__device__ __forceinline__ void store_p_rows(const uint32_t* sr, const float* m, const int* mrow, uint8_t* pbuf,
                                             int q4, float* lsum) {
  uint32_t pv[kRows][kStageR];
#pragma unroll
  for (int x = 0; x < kRows; ++x)
#pragma unroll
    for (int r = 0; r < kStageR; ++r)
      pv[x][r] = pack_half2(__uint_as_float(sr[4 * r + 2 * x]) - m[x], __uint_as_float(sr[4 * r + 2 * x + 1]) - m[x]);
#pragma unroll
  for (int x = 0; x < kRows; ++x)
#pragma unroll
    for (int r = 0; r < kStageR; ++r) pv[x][r] = m[x] != neg_inf() ? ex2_f16x2(pv[x][r]) : 0u;
#pragma unroll
  for (int x = 0; x < kRows; ++x) {
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < kStageR; ++r) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&pv[x][r]));
      acc += f.x + f.y;
    }
    lsum[x] += acc;
  }
#pragma unroll
  for (int x = 0; x < kRows; ++x) {
    uint8_t* prow = pbuf + mrow[x] * 128 + q4 * 4;
    const int sw = mrow[x] & 7;
#pragma unroll
    for (int r = 0; r < kStageR; ++r)
      *reinterpret_cast<uint32_t*>(prow + (r >> 3) * kPAtom + (((r & 7) ^ sw) << 4)) = pv[x][r];
  }
}

__device__ __noinline__ void softmax_role(const Ctx& c) {
  const AttnParams& p = *c.p;
  VerifyShared* sh = c.sh;
  uint8_t* smem = c.smem;
  const uint32_t tmem = c.tmem;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tid = threadIdx.x - kSoftmaxWarp0 * 32;  // 0..127
  const int qd = warp & 3;                             // TMEM lane quadrant of this warp
  const int q4 = lane & 3;
  const int li_a = lane >> 2, li_b = li_a + 8;          // lanes within the quadrant
  const int ma = 16 * qd + li_a, mb = ma + 8;           // MMA rows
  const uint32_t lane_addr = (uint32_t)(32 * qd) << 16;
  const float sc = p.scale_log2;
  const int gqa = c.gqa;
  // Clear P once (rows no unit writes must hold finite values); the barrier
  // orders the clearing before any thread's first P store.
#pragma unroll 1
  for (int i = tid; i < (int)(2 * kPBuf) / 16; i += kSoftmaxThreads)
    *reinterpret_cast<uint4*>(smem + kPOff + i * 16) = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  named_bar_sync(1, kSoftmaxThreads);
  PieceCursor cur;
  cur.init(&c.ps, c.ng, c.hk, c.t_begin, c.t_end, c.g_begin);
  // Unit rows of this thread in a piece's group, and their lengths (loaded a
  // piece ahead of use).
  auto fill = [&](SoftmaxRows& r) -> bool {
    if (!cur.next(r.g, r.h, r.lo, r.hi, r.nb, r.ustart)) return false;
    const int first_row = c.ps.gfirst[r.g];
    const int nrows = c.ps.gfirst[r.g + 1] - first_row;
    const int cq = gqa * rows_per_quad(nrows), nq = nrows * gqa;
    r.ja = (li_a < cq && qd * cq + li_a < nq) ? qd * cq + li_a : -1;
    r.jb = (li_b < cq && qd * cq + li_b < nq) ? qd * cq + li_b : -1;
    r.len_a = r.ja >= 0 ? __ldg(p.seq_lens + first_row + r.ja / gqa) : -1;
    r.len_b = r.jb >= 0 ? __ldg(p.seq_lens + first_row + r.jb / gqa) : -1;
    return true;
  };
  SoftmaxRows cr, nr;
  bool have = fill(cr);
  int G = 0, piece = 0;
  bool ok = true;
  float2* stats = reinterpret_cast<float2*>(smem + kStatOff);
  while (have && ok) {
    const bool have_next = fill(nr);
    const uint32_t ocol = tmem + kOCol + 128u * (piece & 1);
    const bool has_b = __any_sync(0xffffffffu, cr.jb >= 0);  // warp-uniform
    float m_a = neg_inf(), m_b = neg_inf();
    float ls[2] = {0.f, 0.f};  // this thread's part of the row sums
    const int nst = stages_of(cr.lo, cr.hi);
    for (int s = 0; s < nst; ++s, ++G) {
      const int fs = G % kFlagSlots;
      const int sbuf = G % kSBufs;  // S tile in TMEM
      const int sb = G & 1;         // P buffer
      if (!wait_or_abort(sh, p, &sh->flags_full[fs], (uint32_t)((G / kFlagSlots) & 1)) ||
          !wait_or_abort(sh, p, &sh->s_full[sbuf], (uint32_t)((G / kSBufs) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[4 * kStageR];
      {
        const uint32_t sa = tmem + sbuf * kSBuf + lane_addr;
        int r = 0;
#pragma unroll
        for (; r + 8 <= kStageR; r += 8) tmem_ld_16x256b_x8(sa + 8 * r, *reinterpret_cast<uint32_t(*)[32]>(sr + 4 * r));
        if (r + 4 <= kStageR) {
          tmem_ld_16x256b_x4(sa + 8 * r, sr + 4 * r);
          r += 4;
        }
        if (r + 2 <= kStageR) tmem_ld_16x256b_x2(sa + 8 * r, sr + 4 * r);
      }
      // The flags are read before S is released (the K producer relies on it).
      int blk_ok = 0;
#pragma unroll
      for (int b = 0; b < kStageBlocks; ++b) blk_ok |= (sh->blk[fs][b] != 0) << b;
      tmem_wait_ld();
      tc_fence_before();
      warp_arrive(&sh->s_empty[sbuf]);
      const int t0 = cr.lo + s * kStageBlocks;
      const int nblk = min(kStageBlocks, cr.hi - t0);
      const int tok0 = t0 * kBlockTokens;
      float mxs[2];
      const bool blocks_ok = __all_sync(0xffffffffu, blk_ok == (1 << nblk) - 1);
      // Columns past the row's length, or past the stage's nblk blocks (stale
      // S of an earlier stage when a piece ends inside a row), are masked.
      const int cols = nblk * kBlockTokens;
      const int lims[2] = {min(cr.len_a - tok0, cols) - 2 * q4, min(cr.len_b - tok0, cols) - 2 * q4};
      if (has_b) {
        mask_max_rows<2>(sr, lims, blk_ok, blocks_ok, sc, mxs);
      } else {
        mask_max_rows<1>(sr, lims, blk_ok, blocks_ok, sc, mxs);
        mxs[1] = neg_inf();
      }
      const float mxa = mxs[0], mxb = mxs[1];
      // Lazy rescale: the running max moves only when it grows by more than 8 (x256).
      float alpha_a = 1.f, alpha_b = 1.f;
      if (m_a == neg_inf()) {
        m_a = mxa;
      } else if (mxa > m_a + 8.f) {
        alpha_a = fast_exp2(m_a - mxa);
        m_a = mxa;
      }
      if (has_b) {
        if (m_b == neg_inf()) {
          m_b = mxb;
        } else if (mxb > m_b + 8.f) {
          alpha_b = fast_exp2(m_b - mxb);
          m_b = mxb;
        }
      }
      // P buffer sb is free once PV(G-2) completed.
      if (G >= 2 && !wait_or_abort(sh, p, &sh->pv_done[sb], (uint32_t)(((G - 2) >> 1) & 1))) {
        ok = false;
        break;
      }
      if (__any_sync(0xffffffffu, alpha_a != 1.f || alpha_b != 1.f) && s > 0) {
        if (!wait_or_abort(sh, p, &sh->pv_done[(G - 1) & 1], (uint32_t)(((G - 1) >> 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        rescale_o(ocol, lane_addr, alpha_a, alpha_b);
      }
      uint8_t* pbuf = smem + kPOff + sb * kPBuf;
      const float ms[2] = {m_a, m_b};
      const int mrows[2] = {ma, mb};
      ls[0] *= alpha_a;
      ls[1] *= alpha_b;
      if (has_b) store_p_rows<2>(sr, ms, mrows, pbuf, q4, ls);
      else store_p_rows<1>(sr, ms, mrows, pbuf, q4, ls);
      fence_proxy_async_smem();
      tc_fence_before();
      warp_arrive(&sh->p_full[sb]);
    }
    if (!ok) break;
    // Hand the rows' max and sum (each of a row's four threads holds the sum
    // of its columns) to the epilogue warps and go on with the next piece.
    ls[0] += __shfl_xor_sync(0xffffffffu, ls[0], 1);
    ls[0] += __shfl_xor_sync(0xffffffffu, ls[0], 2);
    ls[1] += __shfl_xor_sync(0xffffffffu, ls[1], 1);
    ls[1] += __shfl_xor_sync(0xffffffffu, ls[1], 2);
    const int b = piece & 1;
    if (piece >= 2 && !wait_or_abort(sh, p, &sh->st_empty[b], (uint32_t)(((piece - 2) >> 1) & 1))) break;
    if (q4 == 0) {
      stats[b * kMaxQRows + ma] = make_float2(m_a, ls[0]);
      stats[b * kMaxQRows + mb] = make_float2(m_b, ls[1]);
    }
    warp_arrive(&sh->st_full[b]);
    ++piece;
    have = have_next;
    cr = nr;
  }
}

// ------------------------------------------------------------------- epilogue
// Warps kEpiWarp0.. (lane quadrant warp % 4, the rows of the softmax warp of
// the same quadrant): per piece, the rows' statistics from the softmax, then
// piece_epilogue on the piece's O buffer.
__device__ __noinline__ void epilogue_role(const Ctx& c) {
  VerifyShared* sh = c.sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qd = warp & 3;
  const int li_a = lane >> 2, li_b = li_a + 8;
  const int ma = 16 * qd + li_a, mb = ma + 8;
  const float2* stats = reinterpret_cast<const float2*>(c.smem + kStatOff);
  PieceCursor cur;
  cur.init(&c.ps, c.ng, c.hk, c.t_begin, c.t_end, c.g_begin);
  SoftmaxRows r;
  for (int piece = 0; cur.next(r.g, r.h, r.lo, r.hi, r.nb, r.ustart); ++piece) {
    const int nrows = c.ps.gfirst[r.g + 1] - c.ps.gfirst[r.g];
    const int cq = c.gqa * rows_per_quad(nrows), nq = nrows * c.gqa;
    r.ja = (li_a < cq && qd * cq + li_a < nq) ? qd * cq + li_a : -1;
    r.jb = (li_b < cq && qd * cq + li_b < nq) ? qd * cq + li_b : -1;
    const int b = piece & 1;
    if (!wait_or_abort(sh, *c.p, &sh->st_full[b], (uint32_t)((piece >> 1) & 1))) return;
    const float2 sa = stats[b * kMaxQRows + ma], sbv = stats[b * kMaxQRows + mb];
    warp_arrive(&sh->st_empty[b]);
    if (!piece_epilogue(c, r, piece, sa.x, sbv.x, sa.y, sbv.y, cur.t >= cur.t_end)) return;
  }
}

__global__ void __launch_bounds__(kVThreads, 1)
    verify_attn_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                       const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ VerifyArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  VerifyShared* sh = reinterpret_cast<VerifyShared*>(smem + kBarOff);
  const AttnParams& p = sh->prm;
  int* plan_mem = reinterpret_cast<int*>(smem + kPlanOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  grid_launch_dependents();
  // Set-up that reads no input runs before the wait for the previous launch
  // in the stream, overlapping its tail: the parameters into shared memory
  // (the roles read them there, not through first-touch constant-cache
  // misses), barriers, tensor memory, descriptors.
  static_assert(sizeof(AttnParams) % 4 == 0 && sizeof(AttnParams) / 4 <= kVThreads, "one word per thread");
  if (threadIdx.x < sizeof(AttnParams) / 4)
    reinterpret_cast<uint32_t*>(&sh->prm)[threadIdx.x] = reinterpret_cast<const uint32_t*>(&args.p)[threadIdx.x];
  if (threadIdx.x == 0) {
    for (int i = 0; i < kKRing; ++i) {
      mbar_init(&sh->k_full[i], 1);
      mbar_init(&sh->k_empty[i], kSlotStages);
    }
    for (int i = 0; i < kVRing; ++i) {
      mbar_init(&sh->v_full[i], 1);
      mbar_init(&sh->v_empty[i], kSlotStages);
    }
    for (int i = 0; i < kFlagSlots; ++i) mbar_init(&sh->flags_full[i], 1);
    for (int i = 0; i < kSBufs; ++i) {
      mbar_init(&sh->s_full[i], 1);
      mbar_init(&sh->s_empty[i], 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh->p_full[i], 4);
      mbar_init(&sh->pv_done[i], 1);
      mbar_init(&sh->q_full[i], 1);
      mbar_init(&sh->q_empty[i], 1);
      mbar_init(&sh->o_full[i], 1);
      mbar_init(&sh->o_empty[i], 4);
      mbar_init(&sh->st_full[i], 4);
      mbar_init(&sh->st_empty[i], 4);
    }
    mbar_init(&sh->plan_ready, 1);
    sh->first_last = 0;
    sh->last_merge = 0;
    mbar_init(&sh->s_final, 1);
    mbar_init(&sh->pv_final, 1);
    sh->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kSWarp) {
    tmem_alloc(&sh->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kKWarp && lane == 0) {
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
    tma_prefetch_desc(&tmap_q);
  }
  tc_fence_before();
  __syncthreads();  // barriers and the tensor-memory address are visible to every thread
  tc_fence_after();
  if (warp == kEpiWarp0 && gridDim.x <= kPlanCacheWorkers && p.num_rows <= kMaxRows) {
    // While the previous launch finishes, an idle warp brings into L2 what the
    // call will read first, as the previous call on this workspace left it:
    // the plan cache slot and rows it checks, and the first two stages of this
    // worker's K and V.  Prefetches are hints: if the previous call's plan is
    // not this call's (or is being written), they only waste bandwidth; every
    // value used is read again after the wait.
    const int32_t* rd = p.plan_cache + (((args.seq & 1u) ^ 1u) * kPcSlotWords);
    const int32_t* wk = rd + kPcWorkers + blockIdx.x * kPcEntryWords;
    const long long e = __ldcg(reinterpret_cast<const long long*>(wk + kPcEntryFeed) + lane);
    for (int i = lane * 32; i < p.num_rows; i += 32 * 32) {
      prefetch_l2(p.seq_ids + i);
      prefetch_l2(p.seq_lens + i);
      prefetch_l2(rd + kPcIds + i);
      prefetch_l2(rd + kPcLens + i);
    }
    for (int i = lane * 32; i < 3 * (p.num_rows + 1) + 8; i += 32 * 32) prefetch_l2(rd + kPcPlan + i);
    if (lane == 0) prefetch_l2(rd);
    if (lane < 2 * kStageBlocks && e >= 0 && (e >> 8) < (long long)p.bt_rows * p.mbs &&
        (int)(e & 255) < p.num_kv_heads) {
      const long long blk = __ldcg(p.block_table + (e >> 8));
      if (blk >= 0 && blk < p.num_blocks) {
        const int row = (int)(((blk * p.num_layers + p.cur_layer) * p.num_kv_heads + (int)(e & 255)) * kBlockTokens);
        tma_prefetch_2d(&tmap_k, 0, row);
        tma_prefetch_2d(&tmap_k, 64, row);
        tma_prefetch_2d(&tmap_v, 0, row);
        tma_prefetch_2d(&tmap_v, 64, row);
      }
    }
  }
  grid_dependency_wait();  // inputs may come from the previous launch in the stream
  // The plan of the previous call on this workspace, if it is this call's:
  // every thread loads a share of it and of the rows' seq ids and lengths in
  // one round of independent loads, the plan arrays straight into place.
  const bool cacheable = gridDim.x <= kPlanCacheWorkers && p.num_rows <= kMaxRows;
  const int32_t* rd = p.plan_cache + (((args.seq & 1u) ^ 1u) * kPcSlotWords);
  bool same = cacheable;
  if (cacheable) {
    // Every load is issued before any comparison (no short-circuit between
    // loads), so that the whole check costs one memory round trip.
    for (int i = threadIdx.x; i < p.num_rows; i += kVThreads) {
      const int a = __ldcg(p.seq_ids + i), b = __ldcg(rd + kPcIds + i);
      const int c = __ldcg(p.seq_lens + i), d = __ldcg(rd + kPcLens + i);
      same &= (a == b) & (c == d);
    }
    for (int i = threadIdx.x; i < 3 * (p.num_rows + 1) + 8; i += kVThreads) plan_mem[i] = __ldcg(rd + kPcPlan + i);
    if (threadIdx.x < 32) {
      // Lanes 0..9: the key; lane 10: this worker's entry; lane 11 its range.
      const int32_t* wk = rd + kPcWorkers + blockIdx.x * kPcEntryWords;
      const long long* feed = reinterpret_cast<const long long*>(wk + kPcEntryFeed);
      const int32_t v = __ldcg(lane < 10 ? rd + lane : wk);
      const long long range = lane == 11 ? __ldcg(reinterpret_cast<const long long*>(wk + 2)) : 0;
      const long long range_end = lane == 11 ? __ldcg(reinterpret_cast<const long long*>(wk + 4)) : 0;
      const int32_t group = lane == 11 ? __ldcg(wk + 1) : 0;
      const long long f0 = __ldcg(feed + lane), f1 = __ldcg(feed + 32 + lane), f2 = __ldcg(feed + 64 + lane);
      const int32_t want = lane == 0 ? (int32_t)kPlanCacheMagic
                         : lane == 1 ? (int32_t)(args.seq - 1u)
                         : lane == 2 ? p.num_rows
                         : lane == 3 ? p.max_group_rows
                         : lane == 4 ? p.num_kv_heads
                         : lane == 5 ? p.num_q_heads
                         : lane == 6 ? (int32_t)gridDim.x
                         : lane == 7 ? kPieceCost
                         : lane == 8 ? p.mbs
                         : lane == 9 ? p.bt_rows
                         : lane == 10 ? (int32_t)(args.seq - 1u) : v;
      same &= __all_sync(0xffffffffu, v == want);
      if (lane == 11) {
        sh->cached_begin = range;
        sh->cached_end = range_end;
        sh->cached_group = group;
      }
      long long* feed_smem = reinterpret_cast<long long*>(smem + kFeedOff);
      feed_smem[lane] = f0;
      feed_smem[32 + lane] = f1;
      feed_smem[64 + lane] = f2;
    }
  }
  const bool hit = __syncthreads_and(same);
  if (warp == kKWarp) {
    // Warp 0 builds the plan and the launch context alone, releases the other
    // warps, and goes on as the K producer.  The roles read the context from
    // shared memory (one copy per CTA) rather than from a stack copy per
    // thread, which would live in local memory.
    Ctx c;
    c.p = &p;
    c.sh = sh;
    c.smem = smem;
    c.ps = PlanSmem{plan_mem, plan_mem + (p.num_rows + 1), plan_mem + 2 * (p.num_rows + 1),
                    plan_mem + 2 * (p.num_rows + 1) + 8};
    if (!hit) build_plan_warp(c.ps, p.seq_ids, p.seq_lens, p.num_rows, p.max_group_rows);
    c.ng = c.ps.misc[0];
    c.hk = p.num_kv_heads;
    c.gqa = p.num_q_heads / p.num_kv_heads;
    c.oob_row = args.oob_row;
    c.total = (long long)c.hk * c.ps.gprefix[c.ng];
    const long long launched = gridDim.x;
    c.w = blockIdx.x;
    c.split.gprefix = c.ps.gprefix;
    c.split.ng = c.ng;
    c.split.hk = c.hk;
    c.split.pc = kPieceCost;
    c.split.vtotal = c.total + (long long)kPieceCost * c.hk * c.ng;
    c.workers = c.total == 0 ? 0 : (launched < c.split.vtotal ? launched : c.split.vtotal);
    c.split.workers = c.workers;
    if (hit) {
      c.t_begin = sh->cached_begin;
      c.t_end = sh->cached_end;
      c.g_begin = sh->cached_group;
    } else {
      long long edge = 0;  // lanes 0 and 1: the first tiles of workers w and w + 1
      if (c.w < c.workers && lane < 2) edge = c.split.begin(c.w + lane);
      c.t_begin = __shfl_sync(0xffffffffu, edge, 0);
      c.t_end = __shfl_sync(0xffffffffu, edge, 1);
      c.g_begin = c.t_begin < c.t_end ? find_group(c.ps.gprefix, c.ng, c.t_begin, c.hk) : 0;
    }
    c.pc_hit = hit;
    c.seq = args.seq;
    c.pc_entry = cacheable ? p.plan_cache + (args.seq & 1u) * kPcSlotWords + kPcWorkers + blockIdx.x * kPcEntryWords
                           : nullptr;
    c.tmem = sh->tmem_base;
    if (lane == 0) sh->ctx = c;
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->plan_ready);
  }
  const bool planned = warp == kKWarp || wait_or_abort(sh, p, &sh->plan_ready, 0);
  const Ctx& cs = sh->ctx;
  // The epilogue warps, idle until the first piece ends, leave this call's
  // plan for the next call: every CTA its own range, CTA 0 the rest.
  if (planned && cacheable && warp >= kEpiWarp0) {
    const int t = threadIdx.x - kEpiWarp0 * 32;
    int32_t* wr = p.plan_cache + (args.seq & 1u) * kPcSlotWords;
    if (cs.w >= cs.workers && t == 0) {  // a CTA without tiles (the K warp writes the others' entries)
      int32_t* wk = wr + kPcWorkers + blockIdx.x * kPcEntryWords;
      *reinterpret_cast<long long*>(wk + 2) = cs.t_begin;
      *reinterpret_cast<long long*>(wk + 4) = cs.t_end;
      wk[1] = cs.g_begin;
      wk[0] = (int32_t)args.seq;
    }
    if (blockIdx.x == 0) {
      for (int i = t; i < p.num_rows; i += kEpiThreads) {
        wr[kPcIds + i] = __ldcg(p.seq_ids + i);
        wr[kPcLens + i] = __ldcg(p.seq_lens + i);
      }
      for (int i = t; i < 3 * (p.num_rows + 1) + 8; i += kEpiThreads) wr[kPcPlan + i] = plan_mem[i];
      if (t == 0) {
        wr[0] = (int32_t)kPlanCacheMagic;
        wr[1] = (int32_t)args.seq;
        wr[2] = p.num_rows;
        wr[3] = p.max_group_rows;
        wr[4] = p.num_kv_heads;
        wr[5] = p.num_q_heads;
        wr[6] = (int)gridDim.x;
        wr[7] = kPieceCost;
        wr[8] = p.mbs;
        wr[9] = p.bt_rows;
      }
    }
  }
  if (planned && warp >= kSoftmaxWarp0 && warp < kSoftmaxWarp0 + 4)
    write_nan_rows(p, cs.ps, cs.ng, cs.w * 4 + (warp - kSoftmaxWarp0), (long long)gridDim.x * 4);
  const bool work = planned && cs.w < cs.workers;  // uniform over the CTA unless the wait gave up
  if (!work) {
  } else if (warp == kKWarp) {
    producer(cs, &tmap_k, sh->k_full, sh->k_empty, kKOff, kKRing, 1);
  } else if (warp == kVWarp) {
    producer(cs, &tmap_v, sh->v_full, sh->v_empty, kVOff, kVRing, 0);
  } else if (warp == kSWarp) {
    if (lane == 0) s_issuer(cs, &tmap_q);
  } else if (warp == kPVWarp) {
    if (lane == 0) pv_issuer(cs);
  } else if (warp >= kEpiWarp0) {
    epilogue_role(cs);
  } else {
    softmax_role(cs);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kSWarp) tmem_dealloc(sh->tmem_base, kTmemCols);
  if (work && !aborted(sh) && (sh->first_last || sh->last_merge)) finish_units(cs);
}

// ------------------------------------------------------------------ host side
long long verify_workers(int device) { return num_sms(device); }

int verify_max_rows() { return kVerifyMaxRows; }

// Rows of one request per unit.  A unit's rows are cut into four chunks of
// ceil(rows / 4) rows; a chunk's gqa * ceil(rows / 4) query rows must fit the
// 16 lanes of one TMEM quadrant (one softmax warp) and the 16 / gqa rows of
// one Q box, so at most 4 * floor(16 / gqa) rows (64 / gqa rounded down to a
// multiple of 4 rows per chunk: 20 rather than 21 at gqa 3, 4 rather than 7
// at gqa 9).
int verify_group_rows(int gqa) {
  if (gqa < 1 || gqa > kMaxGqa) return 0;
  return 4 * (16 / gqa);
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
              NEB_ERR_INVALID, "group rows exceed what one TMEM quadrant per chunk holds");
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
    // Q as [rows][q heads][128]: a box is one query chunk, gqa heads x (16 / gqa) rows.
    const unsigned long long dims[3] = {128, (unsigned long long)p.num_q_heads, (unsigned long long)p.num_rows};
    const unsigned long long strides[2] = {256, 256ull * p.num_q_heads};
    const unsigned box[3] = {64, (unsigned)gqa, (unsigned)(16 / gqa)};
    int rc = tensor_map(&tq, p.q, 3, dims, strides, box);
    if (rc != NEB_OK) return rc;
  }
  VerifyArgs a;
  a.p = p;
  a.oob_row = (int)rows;
  {
    // Launch number per workspace: calls on one workspace are ordered on one
    // stream, so call n may use the plan left by call n - 1.
    static std::mutex seq_mu;
    static std::unordered_map<const void*, uint32_t> seq_of;
    std::lock_guard<std::mutex> lock(seq_mu);
    a.seq = ++seq_of[p.hdr];
  }
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

}  // namespace neb
