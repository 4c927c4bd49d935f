// Device-side work plan shared by the attention kernels.
//
// Rows are grouped into "groups": maximal runs of adjacent rows with the same
// seq_id, cut every `max_group_rows` rows.  A verify of depth k is lowered by
// the reference into k+1 adjacent rows of one seq_id with lengths L+1..L+k+1
// (nebulasd/src/nebulasd/workers/target/backend.py:102-111), so one group
// streams its KV prefix once for all of its rows; each row keeps its own length
// mask, which is exactly the causality of the reference's independent rows
// (swiftLLM/swiftllm/worker/kernels/paged_attn.py:74-75).
//
// A unit is (group, kv_head); it covers nb = ceil(max_len / 16) KV tiles of
// 16 tokens.  Units are laid end to end (group-major, head-minor) into one
// tile sequence of length T, and worker w of W owns tiles
// [floor(w*T/W), floor((w+1)*T/W)): every worker streams the same number of
// bytes (+-1 tile) whatever the length distribution.  A unit cut by worker
// boundaries is finished by whichever of its workers arrives last, which
// merges the normalised partials by log-sum-exp in a fixed (slot) order.
//
// Every CTA builds the plan redundantly in shared memory from seq_ids and
// seq_lens (R <= kMaxRows); this costs two coalesced reads of R ints and a few
// block scans, and needs no host synchronisation and no extra launch.
#pragma once

#include "neb_common.cuh"

namespace neb {

constexpr int kMaxRows = 4096;

struct PlanSmem {
  int* gfirst;   // [R + 1]  first row of group g; gfirst[NG] = R
  int* gprefix;  // [R + 1]  exclusive prefix of tiles per head; gprefix[NG] = total
  int* misc;     // [8]      misc[0] = NG
  int* gsid;     // [R + 1]  seq id of group g (optional: null when not kept)
};

__host__ __device__ inline size_t plan_smem_bytes(int num_rows, bool with_sid = false) {
  return (size_t)((with_sid ? 3 : 2) * (num_rows + 1) + 8) * sizeof(int);
}

// Block-wide inclusive scan (sum or max) of one value per thread.  `scratch`
// holds >= 32 ints.  All threads of the block must call it.
template <bool kMax>
__device__ __forceinline__ int block_inclusive_scan(int v, int* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v = kMax ? max(v, n) : v + n;
  }
  if (lane == 31) scratch[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int t = lane < nwarps ? scratch[lane] : (kMax ? INT_MIN : 0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int n = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t = kMax ? max(t, n) : t + n;
    }
    scratch[lane] = t;
  }
  __syncthreads();
  if (warp > 0) {
    int prev = scratch[warp - 1];
    v = kMax ? max(v, prev) : v + prev;
  }
  __syncthreads();
  return v;
}

// Builds the plan into `ps`.  `scratch` is 32 ints of shared memory.
// Returns nothing; ps.misc[0] = number of groups.
static __device__ __noinline__ void build_plan(PlanSmem ps, int* scratch, const int32_t* __restrict__ seq_ids,
                                  const int32_t* __restrict__ seq_lens, int num_rows,
                                  int max_group_rows) {
  // Pass 1: group starts and first rows.
  int carry_run = 0, carry_groups = 0;
  for (int base = 0; base < num_rows; base += blockDim.x) {
    const int r = base + threadIdx.x;
    int sid = 0, prev = 0;
    bool seq_start = false;
    if (r < num_rows) {
      sid = seq_ids[r];
      prev = r > 0 ? seq_ids[r - 1] : 0;
      seq_start = (r == 0) || (sid != prev);
      ps.gprefix[r] = seq_lens[r];  // row lengths, read back by pass 2 (one coalesced load)
    }
    int run_start = block_inclusive_scan<true>(seq_start ? r : 0, scratch);
    run_start = max(run_start, carry_run);
    bool gstart = false;
    if (r < num_rows) gstart = seq_start || ((r - run_start) % max_group_rows == 0);
    int gidx = block_inclusive_scan<false>(gstart ? 1 : 0, scratch) + carry_groups - 1;
    if (r < num_rows && gstart) {
      ps.gfirst[gidx] = r;
      if (ps.gsid) ps.gsid[gidx] = sid;
    }
    // carries from the last thread of the chunk
    if (threadIdx.x == blockDim.x - 1) {
      scratch[0] = run_start;
      scratch[1] = gidx + 1;
    }
    __syncthreads();
    carry_run = scratch[0];
    carry_groups = scratch[1];
    __syncthreads();
  }
  const int ng = carry_groups;
  if (threadIdx.x == 0) {
    ps.gfirst[ng] = num_rows;
    ps.misc[0] = ng;
  }
  __syncthreads();
  // Pass 2: tiles per group (max length over its rows) and their exclusive prefix.
  int carry = 0;
  for (int base = 0; base < ng; base += blockDim.x) {
    const int g = base + threadIdx.x;
    int nb = 0;
    if (g < ng) {
      // Lengths of the group's rows (>= g), kept in gprefix by pass 1: every
      // thread reads them before the scan's first barrier and writes only
      // gprefix[g] (< the next chunk's rows) after it.
      int mx = 0;
      for (int r = ps.gfirst[g]; r < ps.gfirst[g + 1]; ++r) mx = max(mx, ps.gprefix[r]);
      nb = (mx + 15) >> 4;
    }
    int incl = block_inclusive_scan<false>(nb, scratch);
    if (g < ng) ps.gprefix[g] = carry + incl - nb;
    if (threadIdx.x == blockDim.x - 1) scratch[0] = carry + incl;
    __syncthreads();
    carry = scratch[0];
    __syncthreads();
  }
  if (threadIdx.x == 0) ps.gprefix[ng] = carry;
  __syncthreads();
}

// The same plan built by one warp (all 32 lanes call it; no block barrier), so
// that the rest of the CTA can be released by an mbarrier as soon as it is in
// shared memory.  Rows go 32 at a time, one per lane: a run of one seq_id
// starts where the id changes (ballot), a group starts there or every
// max_group_rows rows into the run, and group indices come from popcounts.
// Up to four chunks' loads are in flight before the first is used.
static __device__ __noinline__ void build_plan_warp(PlanSmem ps, const int32_t* __restrict__ seq_ids,
                                                    const int32_t* __restrict__ seq_lens, int num_rows,
                                                    int max_group_rows) {
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u, le = lt | (1u << lane);
  int run = 0, groups = 0, last_sid = 0;
  for (int base = 0; base < num_rows; base += 128) {
    int sid[4], len[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int r = base + 32 * k + lane;
      sid[k] = r < num_rows ? __ldg(seq_ids + r) : 0;
      len[k] = r < num_rows ? __ldg(seq_lens + r) : 0;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int b = base + 32 * k;
      if (b >= num_rows) break;
      const int r = b + lane;
      const bool valid = r < num_rows;
      int prev = __shfl_up_sync(0xffffffffu, sid[k], 1);
      if (lane == 0) prev = last_sid;
      const bool seq_start = valid && (r == 0 || sid[k] != prev);
      const unsigned runs = __ballot_sync(0xffffffffu, seq_start) & le;
      const int run_start = runs ? b + 31 - __clz(runs) : run;
      const bool gstart = valid && (seq_start || (r - run_start) % max_group_rows == 0);
      const unsigned gb = __ballot_sync(0xffffffffu, gstart);
      if (gstart) {
        const int gidx = groups + __popc(gb & lt);
        ps.gfirst[gidx] = r;
        if (ps.gsid) ps.gsid[gidx] = sid[k];
      }
      if (valid) ps.gprefix[r] = len[k];  // row lengths, read back below
      run = __shfl_sync(0xffffffffu, run_start, 31);
      last_sid = __shfl_sync(0xffffffffu, sid[k], 31);
      groups += __popc(gb);
    }
  }
  const int ng = groups;
  if (lane == 0) {
    ps.gfirst[ng] = num_rows;
    ps.misc[0] = ng;
  }
  __syncwarp();
  // Tiles per group (max length over its rows) and their exclusive prefix.
  // A chunk reads lengths of rows >= its first group before writing
  // gprefix[g] for its own groups (< the rows of later chunks).
  int carry = 0;
  for (int gb0 = 0; gb0 < ng; gb0 += 32) {
    const int g = gb0 + lane;
    int nb = 0;
    if (g < ng) {
      int mx = 0;
      for (int r = ps.gfirst[g]; r < ps.gfirst[g + 1]; ++r) mx = max(mx, ps.gprefix[r]);
      nb = (mx + 15) >> 4;
    }
    int incl = nb;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    __syncwarp();
    if (g < ng) ps.gprefix[g] = carry + incl - nb;
    carry += __shfl_sync(0xffffffffu, incl, 31);
    __syncwarp();
  }
  if (lane == 0) ps.gprefix[ng] = carry;
  __syncwarp();
}

// Largest group g with hk * gprefix[g] <= t (t < hk * gprefix[ng]); skips empty groups.
__device__ __forceinline__ int find_group(const int* gprefix, int ng, long long t, int hk) {
  int lo = 0, hi = ng;  // invariant: hk*gprefix[lo] <= t < hk*gprefix[hi]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if ((long long)hk * gprefix[mid] <= t) lo = mid; else hi = mid;
  }
  return lo;
}

// Cost-weighted split.  Each unit (group, kv head) counts `pc` extra virtual
// tiles ahead of its own tiles: the fixed cost of starting a piece (its
// epilogue, the pipeline refill).  Unit u = hk*g + h starts at virtual
// position hk*(gprefix[g] + pc*g) + h*(nb_g + pc), and its tile t sits at
// t + pc*(u + 1); V = T + pc*hk*ng.  Workers split [0, V) evenly; a worker's
// tiles are the ones whose virtual positions fall in its share, a contiguous
// range of tiles as with pc = 0 (which reproduces the plain tile split).
struct CostSplit {
  const int* gprefix;
  int ng, hk, pc;
  long long vtotal, workers;

  __device__ __forceinline__ long long vbase(int g) const {
    return (long long)hk * ((long long)gprefix[g] + (long long)pc * g);
  }
  // Virtual position of tile t (t < T).
  __device__ __forceinline__ long long vpos(long long t) const {
    const int g = find_group(gprefix, ng, t, hk);
    const int nb = gprefix[g + 1] - gprefix[g];
    const int h = (int)((t - (long long)hk * gprefix[g]) / nb);
    return t + (long long)pc * ((long long)g * hk + h + 1);
  }
  // First tile whose virtual position is >= v (T when none).
  __device__ __forceinline__ long long tile_at(long long v) const {
    if (v >= vtotal) return (long long)hk * gprefix[ng];
    int lo = 0, hi = ng;  // largest g with vbase(g) <= v
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (vbase(mid) <= v) lo = mid; else hi = mid;
    }
    const int nb = gprefix[lo + 1] - gprefix[lo];
    const long long off = v - vbase(lo);
    const long long h = off / (nb + pc);
    const long long in_unit = off - h * (nb + pc);
    return (long long)hk * gprefix[lo] + h * nb + (in_unit > pc ? in_unit - pc : 0);
  }
  __device__ __forceinline__ long long begin(long long w) const { return tile_at((w * vtotal) / workers); }
  __device__ __forceinline__ long long worker_of_tile(long long t) const {
    return ((vpos(t) + 1) * workers - 1) / vtotal;
  }
};

// Slot of the partial written by worker w for a unit whose first worker is w0.
__host__ __device__ __forceinline__ long long piece_slot(long long w, long long w0) {
  return w == w0 ? 2 * w + 1 : 2 * w;
}

}  // namespace neb
