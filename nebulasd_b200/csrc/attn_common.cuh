// Parameters, workspace layout and the split-K merge shared by the attention kernels.
#pragma once

#include "plan.cuh"

namespace neb {

constexpr int kHeadDim = 128;
constexpr int kBlockTokens = 16;
constexpr int kTileHalfs = kBlockTokens * kHeadDim;  // one (block, layer, head) tile: 4 KiB

struct AttnParams {
  const __half* q;
  const __half* k_cache;
  const __half* v_cache;
  const int32_t* block_table;
  int32_t bt_rows;
  int32_t mbs;  // max_blocks_per_seq (row stride of block_table)
  const int32_t* seq_lens;
  const int32_t* seq_ids;
  int32_t num_rows;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int64_t num_blocks;
  int32_t num_layers;
  int32_t cur_layer;
  float scale_log2;  // softmax_scale * log2(e)
  __half* o;
  // workspace
  WorkspaceHeader* hdr;
  int32_t* counters;  // [num_rows * num_kv_heads]
  float* part_lse;    // [2 * workers][nq]
  float* part_o;      // [2 * workers][nq][128]
  int32_t nq;         // partial rows per slot = gqa * max_group_rows
  int32_t max_group_rows;
  int32_t* plan_cache;  // two plan-cache slots (verify kernel)
};

// Workspace: header | counters | plan cache | part_lse | part_o, each 256-byte
// aligned.  The counter region has a fixed size and place whatever the call's
// shape, so the partials of one call can never land where a later call (with
// more rows or heads) keeps counters that must read zero; the plan cache too.
constexpr int kMaxKvHeads = 64;

// Plan cache of the verify kernel: the work plan depends only on the rows'
// seq ids and lengths and the call's shape, which the 36 layer calls of one
// forward share.  A call with launch number n (counted per workspace on the
// host) reads slot (n + 1) % 2, written by call n - 1, and writes slot n % 2;
// a slot is used only when its key, the row arrays and the CTA's own entry
// all match, so a stale or foreign slot just means the plan is rebuilt.
// Slot, in 32-bit words: key [16] | seq ids [kMaxRows] | lengths [kMaxRows] |
// plan arrays as laid out in shared memory [3 * (kMaxRows + 1) + 8] | per
// worker [kPcEntryWords]: {seq, first group, t_begin, t_end} and, from word
// kPcEntryFeed, the block-table entries of its first 96 tiles (64-bit each).
constexpr int kPlanCacheWorkers = 256;
constexpr uint32_t kPlanCacheMagic = 0x4e504331u;
constexpr int kPcIds = 16;
constexpr int kPcLens = kPcIds + kMaxRows;
constexpr int kPcPlan = kPcLens + kMaxRows;
constexpr int kPcWorkers = (kPcPlan + 3 * (kMaxRows + 1) + 8 + 7) & ~7;
constexpr int kPcEntryFeed = 8;
constexpr int kPcEntryWords = 256;
constexpr int kPcSlotWords = ((kPcWorkers + kPlanCacheWorkers * kPcEntryWords) + 63) & ~63;
static_assert(kPcEntryFeed + 2 * 96 <= kPcEntryWords, "a worker's entry holds its 96 tile words");
constexpr size_t kPlanCacheBytes = 2ull * kPcSlotWords * sizeof(int32_t);

struct WorkspaceLayout {
  size_t counters, plan_cache, part_lse, part_o, total;
};

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

__host__ __device__ inline WorkspaceLayout workspace_layout(long long workers, int num_rows,
                                                            int num_kv_heads, int nq) {
  (void)num_rows;
  (void)num_kv_heads;
  WorkspaceLayout L;
  L.counters = sizeof(WorkspaceHeader);
  L.plan_cache = L.counters + align256((size_t)kMaxRows * kMaxKvHeads * sizeof(int32_t));
  L.part_lse = L.plan_cache + align256(kPlanCacheBytes);
  L.part_o = L.part_lse + align256((size_t)2 * workers * nq * sizeof(float));
  L.total = L.part_o + align256((size_t)2 * workers * nq * kHeadDim * sizeof(float));
  return L;
}

__device__ __forceinline__ void record_error(const AttnParams& p, uint32_t bits) {
  atomicOr(&p.hdr->error_bits, bits);
}

// Physical block of logical tile `tile` of sequence `sid`, or -1 (recorded) if
// the table entry, seq_id or tile index is out of range.
__device__ __forceinline__ long long lookup_block(const AttnParams& p, int sid, int tile) {
  if (sid < 0 || sid >= p.bt_rows) return -1;
  if (tile >= p.mbs) {
    record_error(p, kErrTooManyBlocks);
    return -1;
  }
  const long long blk = p.block_table[(long long)sid * p.mbs + tile];
  if (blk < 0 || blk >= p.num_blocks) {
    record_error(p, kErrBlockIndex);
    return -1;
  }
  return blk;
}

// Element offset of the (block, cur_layer, kv_head) tile.
__device__ __forceinline__ long long tile_offset(const AttnParams& p, long long blk, int kv_head) {
  return ((blk * p.num_layers + p.cur_layer) * p.num_kv_heads + kv_head) * (long long)kTileHalfs;
}

// Warp-level log-sum-exp merge of a split unit's partials, in slot order, into
// fp16 output rows.  Unit q-row j = r * gqa + g is row first_row + r, q head
// kv_head * gqa + g.  Pieces whose lse is -inf (no unmasked token) carry no
// weight; if every piece is empty the result is 0/0 = NaN, as in the
// reference's phase 2 (swiftLLM/swiftllm/worker/kernels/paged_attn.py:131-149).
// The warp handles unit rows jbegin, jbegin + jstep, ...
__device__ inline void merge_unit_warp(const AttnParams& p, int first_row, int nrows, int kv_head,
                                       int gqa, long long w0, long long w1, int jbegin = 0, int jstep = 1) {
  const int lane = threadIdx.x & 31;
  const int nqu = nrows * gqa;
  for (int j = jbegin; j < nqu; j += jstep) {
    float mx = neg_inf();
    for (long long w = w0; w <= w1; ++w) {
      const long long slot = piece_slot(w, w0);
      mx = fmaxf(mx, __ldcg(p.part_lse + slot * p.nq + j));
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float den = 0.f;
    if (mx != neg_inf()) {
      for (long long w = w0; w <= w1; ++w) {
        const long long slot = piece_slot(w, w0);
        const float le = __ldcg(p.part_lse + slot * p.nq + j);
        if (le == neg_inf()) continue;
        const float wt = fast_exp2(le - mx);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(p.part_o + (slot * p.nq + j) * kHeadDim) + lane);
        acc.x += wt * v.x; acc.y += wt * v.y; acc.z += wt * v.z; acc.w += wt * v.w;
        den += wt;
      }
    }
    const float inv = 1.f / den;
    const int row = first_row + j / gqa;
    const int head = kv_head * gqa + (j % gqa);
    uint2 out;
    out.x = f2_to_h2(acc.x * inv, acc.y * inv);
    out.y = f2_to_h2(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2*>(p.o + ((long long)row * p.num_q_heads + head) * kHeadDim + lane * 4) = out;
  }
}

// The same merge spread over `nthreads` threads (tid in [0, nthreads)): a
// thread owns (unit row, 4-column chunk) pairs, kQ at a time, and issues the
// loads of all their slots (up to four slots per round) before using any, so
// that a merge costs one memory round trip when nthreads * kQ covers the
// unit.  Slots fold in order with a running maximum; the result does not
// depend on kQ or nthreads.
template <int kQ>
static __device__ __noinline__ void merge_unit_threads(const AttnParams& p, int first_row, int nrows, int kv_head,
                                                       int gqa, long long w0, long long w1, int tid, int nthreads) {
  const int npairs = nrows * gqa * 32;
  for (int base = tid; base < npairs; base += kQ * nthreads) {
    float mx[kQ], den[kQ];
    float4 acc[kQ];
#pragma unroll
    for (int q = 0; q < kQ; ++q) {
      mx[q] = neg_inf();
      den[q] = 0.f;
      acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (long long wb = w0; wb <= w1; wb += 4) {
      float le[kQ][4];
      float4 v[kQ][4];
#pragma unroll
      for (int q = 0; q < kQ; ++q) {
        const int idx = base + q * nthreads;
        const int j = idx >> 5, c = idx & 31;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          le[q][k] = neg_inf();
          v[q][k] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (idx < npairs && wb + k <= w1) {
            const long long slot = piece_slot(wb + k, w0);
            le[q][k] = __ldcg(p.part_lse + slot * p.nq + j);
            v[q][k] = __ldcg(reinterpret_cast<const float4*>(p.part_o + (slot * p.nq + j) * kHeadDim) + c);
          }
        }
      }
#pragma unroll
      for (int q = 0; q < kQ; ++q) {
        const float cm = fmaxf(fmaxf(le[q][0], le[q][1]), fmaxf(le[q][2], le[q][3]));
        if (cm == neg_inf()) continue;
        if (cm > mx[q]) {
          const float sc = fast_exp2(mx[q] - cm);  // 0 while nothing was folded in yet
          acc[q].x *= sc; acc[q].y *= sc; acc[q].z *= sc; acc[q].w *= sc;
          den[q] *= sc;
          mx[q] = cm;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (le[q][k] == neg_inf()) continue;
          const float wt = fast_exp2(le[q][k] - mx[q]);
          acc[q].x += wt * v[q][k].x; acc[q].y += wt * v[q][k].y;
          acc[q].z += wt * v[q][k].z; acc[q].w += wt * v[q][k].w;
          den[q] += wt;
        }
      }
    }
#pragma unroll
    for (int q = 0; q < kQ; ++q) {
      const int idx = base + q * nthreads;
      if (idx >= npairs) continue;
      const int j = idx >> 5, c = idx & 31;
      const float inv = 1.f / den[q];
      const int row = first_row + j / gqa;
      const int head = kv_head * gqa + (j % gqa);
      uint2 out;
      out.x = f2_to_h2(acc[q].x * inv, acc[q].y * inv);
      out.y = f2_to_h2(acc[q].z * inv, acc[q].w * inv);
      *reinterpret_cast<uint2*>(p.o + ((long long)row * p.num_q_heads + head) * kHeadDim + c * 4) = out;
    }
  }
}

// Rows of groups with no tile (every length <= 0) get NaN, like the reference.
static __device__ __noinline__ void write_nan_rows(const AttnParams& p, const PlanSmem& ps, int ng, long long w,
                                      long long workers) {
  const int lane = threadIdx.x & 31;
  const uint2 nan2 = make_uint2(0x7e007e00u, 0x7e007e00u);
  for (long long g = w; g < ng; g += workers) {
    if (ps.gprefix[g + 1] != ps.gprefix[g]) continue;
    for (int r = ps.gfirst[g]; r < ps.gfirst[g + 1]; ++r)
      for (int h = 0; h < p.num_q_heads; ++h)
        *reinterpret_cast<uint2*>(p.o + ((long long)r * p.num_q_heads + h) * kHeadDim + lane * 4) = nan2;
  }
}

}  // namespace neb
