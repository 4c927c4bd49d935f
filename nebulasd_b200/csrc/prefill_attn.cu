// Causal prefill attention over packed variable-length sequences (tcgen05).
//
// Replaces flash_attn_varlen_func of swiftLLM/swiftllm/worker/layers/
// transformer_layer.py:7-32, which copies cu_seqlens to the host and runs one
// scaled_dot_product_attention per sequence.  q is [T][H][128], k and v are
// [T][Hk][128] (token strides given), sequence s owns tokens cu[s]..cu[s+1]-1
// and row t of it attends to keys 0..t of the same sequence.
//
// Work unit: (sequence, block of TQ = 128 / gqa query tokens, kv head).  Its
// 128 MMA rows are the TQ tokens x gqa q heads of the kv head (row r = token
// r / gqa, head r % gqa), so every K and V tile it reads serves all heads of
// the group.  A unit reads the key tiles 0 .. ceil(last token / 128) of its
// sequence; only the last one needs a mask (the block's tokens all lie in
// it, since TQ divides 128).
//
// Two launches, no host synchronisation:
//   prefill_plan_kernel (one CTA): checks cu_seqlens and lists every unit,
//     the most expensive first (a unit's cost depends only on its block
//     index), as {first token, sequence length, first query token, kv head}.
//   prefill_attn_kernel (one persistent CTA per SM): CTA c takes units
//     c, 2W-1-c, 2W+c, ... of the list (W CTAs), so that every CTA gets a
//     similar mix of long and short units.  Warp roles:
//       warp 0     loads: Q of a unit (two 3D boxes, 16 KB each) into one of
//                  two Q buffers; K and V tiles of 128 keys (two boxes each)
//                  into two-slot K and V rings (TMA, no multicast).
//       warp 1     S issue (one thread): S = Q K^T (M=128, N=128) into one of
//                  three TMEM S buffers, ahead of the softmax.
//       warp 14    P V issue (one thread): O += P V into the TMEM O
//                  accumulator, P from TMEM (A operand), V from shared
//                  memory; an S buffer is reused once its P V has completed.
//       warps 2-9  softmax, two warps per TMEM lane quadrant, 16 rows each
//                  (two rows x 32 columns per thread): the rows' scores from
//                  TMEM, the mask of the last tile, the running max (moved
//                  only when it grows by more than 8 in the exp2 domain, O
//                  then rescaled in TMEM), P = 2^(s - m) as fp16 pairs back
//                  into the S buffer, and the fp32 row sum of exactly those
//                  fp16 values.
//       warps 10-13 epilogue: O / l of a finished unit into registers as
//                  fp16 (O is then free for the next unit), then the output
//                  rows, while the other warps go on with the next unit.
//
// Every wait is bounded (about 2 s); on expiry the kernel records kErrTimeout
// in the workspace header, stops issuing work, waits (bounded) for its own
// copies and MMAs, frees its TMEM and returns.  Launched with programmatic
// stream serialisation: set-up that reads no input overlaps the previous
// launch's tail.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "attn_common.cuh"
#include "sm100.cuh"

namespace neb {
using namespace sm100;

namespace prefill {

constexpr int kThreads = 480;  // 15 warps: 0 loads, 1 S issue, 2-9 softmax, 10-13 epilogue, 14 P V issue
constexpr int kPvWarp = 14;
constexpr int kLoadWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kSoftmaxWarp0 = 2;
constexpr int kSoftmaxWarps = 8;
constexpr int kEpiWarp0 = kSoftmaxWarp0 + kSoftmaxWarps;
constexpr int kRows = 128;     // MMA M: query rows of a unit
constexpr int kKeys = 128;     // keys of a tile: the S tile's N
constexpr uint32_t kTmemCols = 512;
constexpr int kSBufs = 3;        // S (then P) buffers in TMEM: tile G uses columns 128 (G % 3) ..
constexpr uint32_t kOCol = 384;  // the O accumulator: columns 384..511
constexpr long long kWaitLimit = 4000000000LL;

// Shared memory (offsets from a 1024-byte aligned base).
constexpr uint32_t kHalf = kRows * 128;      // 128 rows x 64 fp16 (one swizzled half)
constexpr uint32_t kTile = 2 * kHalf;        // Q of a unit, or K or V of a tile
constexpr uint32_t kQOff = 0;                // two Q buffers
constexpr uint32_t kKOff = kQOff + 2 * kTile;  // K ring, two slots
constexpr uint32_t kVOff = kKOff + 2 * kTile;  // V ring, two slots
constexpr uint32_t kStatOff = kVOff + 2 * kTile;  // row sums of a finished unit: [2 units][128] float
constexpr uint32_t kBarOff = kStatOff + 2 * kRows * 4;
constexpr uint32_t kSmemBytes = kBarOff + 512 + 1024;  // + alignment pad
static_assert(kSmemBytes <= 232448, "fits the 227 KB a CTA may use");

struct Shared {
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[kSBufs], s_empty[kSBufs];
  // Per S buffer (tile G uses buffer G % 3): the softmax may run up to three
  // tiles ahead of P V, so each tile's hand-offs have their own barriers.
  uint64_t p_full[kSBufs], pv_done[kSBufs];
  uint64_t o_full, o_empty;
  uint64_t st_full[2], st_empty[2];
  uint64_t mma_final, pv_final;
  uint32_t tmem_base;
  int32_t abort_flag;
  int32_t num_units;
};
static_assert(sizeof(Shared) <= 512, "barrier block fits its slot");

struct Args {
  const int4* units;   // {first token of the sequence, its length, first query token, kv head}
  const int32_t* num_units;
  WorkspaceHeader* hdr;
  __half* o;
  long long o_stride;  // elements between tokens of o
  int32_t gqa;
  int32_t tq;          // query tokens per unit = 128 / gqa
  int32_t num_q_heads;
  float scale_log2;    // softmax_scale * log2(e)
};

struct Unit {
  int ts, n, qs, h;
};

// Units of this CTA, in order, each loaded one unit ahead of its use.
struct Cursor {
  const int4* units;
  int nu, k;
  int4 nxt;
  __device__ long long index(int i) const {
    const int w = gridDim.x, c = blockIdx.x;
    return (long long)i * w + ((i & 1) ? (w - 1 - c) : c);
  }
  __device__ void init(const int4* u, int n) {
    units = u;
    nu = n;
    k = 0;
    if (index(0) < nu) nxt = __ldg(units + index(0));
  }
  __device__ bool next(Unit& u) {
    if (index(k) >= nu) return false;
    const int4 d = nxt;
    ++k;
    if (index(k) < nu) nxt = __ldg(units + index(k));
    u.ts = d.x;
    u.n = d.y;
    u.qs = d.z;
    u.h = d.w;
    return true;
  }
};

__device__ __forceinline__ int tiles_of(const Unit& u, int tq) { return (min(u.qs + tq, u.n) + kKeys - 1) / kKeys; }

__device__ __forceinline__ bool aborted(Shared* sh) { return *reinterpret_cast<volatile int32_t*>(&sh->abort_flag) != 0; }

__device__ __forceinline__ void raise_abort(Shared* sh, WorkspaceHeader* hdr) {
  if (atomicExch(&sh->abort_flag, 1) == 0) atomicOr(&hdr->error_bits, (uint32_t)kErrTimeout);
}

__device__ __noinline__ bool wait_slow(Shared* sh, WorkspaceHeader* hdr, uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait_sleep(bar, parity, 20000)) {
    if (aborted(sh) || clock64() - t0 > kWaitLimit) {
      raise_abort(sh, hdr);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ bool wt(Shared* sh, WorkspaceHeader* hdr, uint64_t* bar, uint32_t parity) {
  return mbar_try_wait(bar, parity) || wait_slow(sh, hdr, bar, parity);
}

// The same wait by every lane of a warp, with one verdict for all of them.
__device__ __forceinline__ bool wt_warp(Shared* sh, WorkspaceHeader* hdr, uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, wt(sh, hdr, bar, parity));
}

__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// ------------------------------------------------------------------ loads
__device__ __noinline__ void load_role(Shared* sh, const Args& a, uint8_t* smem, const CUtensorMap* tq,
                                       const CUtensorMap* tk, const CUtensorMap* tv) {
  Cursor cur;
  cur.init(a.units, sh->num_units);
  Unit u;
  int nq = 0, nk = 0, nv = 0;  // loads issued (Q: one per unit; K and V: one per tile)
  bool ok = true;
  while (ok && cur.next(u)) {
    const int qb = nq & 1;
    if (!wt(sh, a.hdr, &sh->q_empty[qb], ((nq >> 1) & 1) ^ 1)) {
      ok = false;
      break;
    }
    uint8_t* qdst = smem + kQOff + qb * kTile;
    mbar_arrive_expect_tx(&sh->q_full[qb], kTile);
    tma_load_3d(qdst, tq, &sh->q_full[qb], 0, u.h * a.gqa, u.ts + u.qs);
    tma_load_3d(qdst + kHalf, tq, &sh->q_full[qb], 64, u.h * a.gqa, u.ts + u.qs);
    ++nq;
    const int nt = tiles_of(u, a.tq);
    for (int j = 0; j < nt; ++j) {
      const int key0 = u.ts + j * kKeys;
      if (!wt(sh, a.hdr, &sh->k_empty[nk & 1], ((nk >> 1) & 1) ^ 1)) {
        ok = false;
        break;
      }
      uint8_t* kdst = smem + kKOff + (nk & 1) * kTile;
      mbar_arrive_expect_tx(&sh->k_full[nk & 1], kTile);
      tma_load_3d(kdst, tk, &sh->k_full[nk & 1], 0, u.h, key0);
      tma_load_3d(kdst + kHalf, tk, &sh->k_full[nk & 1], 64, u.h, key0);
      ++nk;
      if (!wt(sh, a.hdr, &sh->v_empty[nv & 1], ((nv >> 1) & 1) ^ 1)) {
        ok = false;
        break;
      }
      uint8_t* vdst = smem + kVOff + (nv & 1) * kTile;
      mbar_arrive_expect_tx(&sh->v_full[nv & 1], kTile);
      tma_load_3d(vdst, tv, &sh->v_full[nv & 1], 0, u.h, key0);
      tma_load_3d(vdst + kHalf, tv, &sh->v_full[nv & 1], 64, u.h, key0);
      ++nv;
    }
  }
  if (ok) return;  // every copy issued was waited for by its consumer
  // After an abort: the copies issued last into each buffer must land before
  // the CTA exits (a slot is reused only after the copy before it landed).
  for (int i = max(0, nq - 2); i < nq; ++i) mbar_wait(&sh->q_full[i & 1], (i >> 1) & 1, kWaitLimit);
  for (int i = max(0, nk - 2); i < nk; ++i) mbar_wait(&sh->k_full[i & 1], (i >> 1) & 1, kWaitLimit);
  for (int i = max(0, nv - 2); i < nv; ++i) mbar_wait(&sh->v_full[i & 1], (i >> 1) & 1, kWaitLimit);
}

// -------------------------------------------------------------- MMA issue
struct PvTile {
  int G, k, j, nt;
};

// O += P V of tile t.G: P (fp16, 64 columns) in the first half of the tile's
// TMEM S buffer, V from shared memory.  The S buffer is free again once this
// P V has completed.
__device__ __forceinline__ bool issue_pv(Shared* sh, const Args& a, uint32_t tmem, uint32_t v_base,
                                         const PvTile& t) {
  const int slot = t.G & 1, sbuf = t.G % kSBufs;
  if (!wt(sh, a.hdr, &sh->p_full[sbuf], (t.G / kSBufs) & 1) || !wt(sh, a.hdr, &sh->v_full[slot], (t.G >> 1) & 1) ||
      (t.j == 0 && !wt(sh, a.hdr, &sh->o_empty, (t.k & 1) ^ 1)))
    return false;
  tc_fence_after();
  const uint32_t idesc = idesc_f16_f32(kRows, 128, false, true);
  const uint64_t vb0 = smem_desc_sw128(v_base + slot * kTile, kHalf, 1024);
  const uint32_t ocol = tmem + kOCol, pcol = tmem + 128u * sbuf;
#pragma unroll
  for (int kb = 0; kb < kKeys / 16; ++kb)
    mma_f16_ta(ocol, pcol + 8u * kb, vb0 + ((kb * 2048) >> 4), idesc, (t.j > 0 || kb > 0) ? 1u : 0u);
  mma_commit(&sh->v_empty[slot]);
  mma_commit(&sh->s_empty[sbuf]);
  mma_commit(&sh->pv_done[sbuf]);
  if (t.j == t.nt - 1) mma_commit(&sh->o_full);
  return true;
}

// S = Q K^T of every tile, into S buffer G % 3 once the P V that last read
// that buffer (tile G - 3) has completed.
__device__ __noinline__ void mma_role(Shared* sh, const Args& a, uint8_t* smem) {
  const uint32_t tmem = sh->tmem_base;
  const uint32_t q_base = smem_u32(smem + kQOff), k_base = smem_u32(smem + kKOff);
  const uint32_t idesc_s = idesc_f16_f32(kRows, kKeys, false, false);
  Cursor cur;
  cur.init(a.units, sh->num_units);
  Unit u;
  bool ok = true;
  int G = 0;
  for (int k = 0; ok && cur.next(u); ++k) {
    const int qb = k & 1, nt = tiles_of(u, a.tq);
    if (!wt(sh, a.hdr, &sh->q_full[qb], (k >> 1) & 1)) break;
    const uint64_t a0 = smem_desc_sw128(q_base + qb * kTile, 16, 1024);
    for (int j = 0; j < nt; ++j, ++G) {
      const int slot = G & 1, sbuf = G % kSBufs;
      if (!wt(sh, a.hdr, &sh->k_full[slot], (G >> 1) & 1) ||
          !wt(sh, a.hdr, &sh->s_empty[sbuf], ((G / kSBufs) & 1) ^ 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t b0 = smem_desc_sw128(k_base + slot * kTile, 16, 1024);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16(tmem + 128u * sbuf, a0 + (((kk >> 2) * kHalf + (kk & 3) * 32) >> 4),
                b0 + (((kk >> 2) * kHalf + (kk & 3) * 32) >> 4), idesc_s, kk > 0 ? 1u : 0u);
      mma_commit(&sh->s_full[sbuf]);
      mma_commit(&sh->k_empty[slot]);
      if (j == nt - 1) mma_commit(&sh->q_empty[qb]);
    }
  }
  // Every MMA issued has completed before the CTA frees its tensor memory.
  mma_commit(&sh->mma_final);
  mbar_wait(&sh->mma_final, 0, kWaitLimit);
}

// O += P V of every tile, by its own thread, so that P V is issued as soon as
// P is written whatever S the other issuer is waiting to issue.
__device__ __noinline__ void pv_role(Shared* sh, const Args& a, uint8_t* smem) {
  const uint32_t tmem = sh->tmem_base;
  const uint32_t v_base = smem_u32(smem + kVOff);
  Cursor cur;
  cur.init(a.units, sh->num_units);
  Unit u;
  int G = 0;
  bool ok = true;
  for (int k = 0; ok && cur.next(u); ++k) {
    const int nt = tiles_of(u, a.tq);
    for (int j = 0; j < nt; ++j, ++G)
      if (!issue_pv(sh, a, tmem, v_base, PvTile{G, k, j, nt})) {
        ok = false;
        break;
      }
  }
  mma_commit(&sh->pv_final);
  mbar_wait(&sh->pv_final, 0, kWaitLimit);
}

// ---------------------------------------------------------------- softmax
// Two warps per TMEM lane quadrant: warp w (quadrant w % 4, h = (w - 2) / 4)
// owns the 16 lanes (rows) 32 (w % 4) + 16 h .. + 15.  In 16x256b loads each
// thread holds 32 columns of two rows, a = base + lane / 4 and b = a + 8:
// element (x, e) of column group R (0..15) is s[4R + 2x + e], at column
// 8R + 2 (lane % 4) + e, so a row's max and sum take two shuffles within its
// four threads and no other warp is waited for.  P goes back into the first
// 64 columns of the tile's S buffer as fp16 pairs (keys 2c and 2c + 1 in
// column c): with the 16x128b store, register 2R (row a) and 2R + 1 (row b)
// land in column 4R + lane % 4, the pair of keys 8R + 2 (lane % 4) + {0, 1}.

// O of this warp's rows times (alpha_a, alpha_b), in TMEM.
__device__ __noinline__ void rescale_o(uint32_t oaddr, float alpha_a, float alpha_b) {
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    uint32_t r[32];
    tmem_ld_16x256b_x8(oaddr + half * 64, r);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      r[4 * i] = __float_as_uint(__uint_as_float(r[4 * i]) * alpha_a);
      r[4 * i + 1] = __float_as_uint(__uint_as_float(r[4 * i + 1]) * alpha_a);
      r[4 * i + 2] = __float_as_uint(__uint_as_float(r[4 * i + 2]) * alpha_b);
      r[4 * i + 3] = __float_as_uint(__uint_as_float(r[4 * i + 3]) * alpha_b);
    }
    tmem_st_16x256b_x8(oaddr + half * 64, r);
  }
  tmem_wait_st();
}

__device__ __noinline__ void softmax_role(Shared* sh, const Args& a, uint8_t* smem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3, half = (warp - kSoftmaxWarp0) >> 2;
  const int base = 32 * quad + 16 * half;  // first TMEM lane (row) of this warp
  const int q4 = lane & 3;
  const int row[2] = {base + (lane >> 2), base + (lane >> 2) + 8};
  const uint32_t tmem = sh->tmem_base + ((uint32_t)base << 16);
  const float sc = a.scale_log2;
  float* stats = reinterpret_cast<float*>(smem + kStatOff);  // [unit parity][row]
  Cursor cur;
  cur.init(a.units, sh->num_units);
  Unit u;
  int G = 0;
  bool ok = true;
  for (int k = 0; ok && cur.next(u); ++k) {
    const int ob = k & 1, nt = tiles_of(u, a.tq);
    int vis[2];  // keys each row sees: its token + 1 (rows past the sequence: all of it)
#pragma unroll
    for (int x = 0; x < 2; ++x) vis[x] = min(u.qs + row[x] / a.gqa + 1, u.n);
    float m[2] = {neg_inf(), neg_inf()}, l[2] = {0.f, 0.f};
    for (int j = 0; j < nt; ++j, ++G) {
      const int sb = G % kSBufs;
      if (!wt_warp(sh, a.hdr, &sh->s_full[sb], (G / kSBufs) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t scol = tmem + 128u * sb;
      uint32_t s[64];
      tmem_ld_16x256b_x8(scol, *reinterpret_cast<uint32_t(*)[32]>(s));
      tmem_ld_16x256b_x8(scol + 64, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
      tmem_wait_ld();
      if (j == nt - 1) {
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const int lim = vis[x] - j * kKeys - 2 * q4;
#pragma unroll
          for (int R = 0; R < 16; ++R)
#pragma unroll
            for (int e = 0; e < 2; ++e)
              if (8 * R + e >= lim) s[4 * R + 2 * x + e] = __float_as_uint(neg_inf());
        }
      }
      // Row a's max then its P, then row b's: row b's max (ALU) can issue
      // while row a's exp2 and packing (XU) are in flight.
      float alpha[2];
      uint32_t pk[32];  // register 2R: row a, 2R + 1: row b (16x128b order)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        float t[4] = {neg_inf(), neg_inf(), neg_inf(), neg_inf()};
#pragma unroll
        for (int R = 0; R < 16; ++R)
          t[R & 3] = fmaxf(t[R & 3], fmaxf(__uint_as_float(s[4 * R + 2 * x]), __uint_as_float(s[4 * R + 2 * x + 1])));
        float mx = fmaxf(fmaxf(t[0], t[1]), fmaxf(t[2], t[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mxs = mx * sc;
        alpha[x] = 1.f;
        if (j == 0) {
          m[x] = mxs;
        } else if (mxs > m[x] + 8.f) {  // lazy: the max moves only when it grew by more than 2^8
          alpha[x] = fast_exp2(m[x] - mxs);
          m[x] = mxs;
        }
        const float negm = -m[x];
        float acc[2] = {0.f, 0.f};
#pragma unroll
        for (int R = 0; R < 16; ++R) {
          const uint32_t h = ex2_f16x2(f2_to_h2(fmaf(__uint_as_float(s[4 * R + 2 * x]), sc, negm),
                                                fmaf(__uint_as_float(s[4 * R + 2 * x + 1]), sc, negm)));
          pk[2 * R + x] = h;
          const float2 f = h2_to_f2(h);
          acc[R & 1] += f.x + f.y;
        }
        l[x] = l[x] * alpha[x] + (acc[0] + acc[1]);
      }
      if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
        // O is complete up to the previous tile once its P V has completed.
        if (!wt_warp(sh, a.hdr, &sh->pv_done[(G - 1) % kSBufs], ((G - 1) / kSBufs) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        rescale_o(tmem + kOCol, alpha[0], alpha[1]);
      }
      tmem_st_16x128b_x16(scol, pk);
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(&sh->p_full[sb]);
    }
    if (!ok) break;
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      l[x] += __shfl_xor_sync(0xffffffffu, l[x], 1);
      l[x] += __shfl_xor_sync(0xffffffffu, l[x], 2);
    }
    if (!wt_warp(sh, a.hdr, &sh->st_empty[ob], ((k >> 1) & 1) ^ 1)) break;
    if (q4 == 0) {
      stats[ob * kRows + row[0]] = l[0];
      stats[ob * kRows + row[1]] = l[1];
    }
    warp_arrive(&sh->st_full[ob]);
  }
}

// --------------------------------------------------------------- epilogue
__device__ __noinline__ void epilogue_role(Shared* sh, const Args& a, uint8_t* smem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3, row = 32 * quad + lane;
  const uint32_t tmem = sh->tmem_base + ((uint32_t)(32 * quad) << 16);
  const int tok_in_unit = row / a.gqa, head_in_unit = row % a.gqa;
  const float* stats = reinterpret_cast<const float*>(smem + kStatOff);
  Cursor cur;
  cur.init(a.units, sh->num_units);
  Unit u;
  for (int k = 0; cur.next(u); ++k) {
    const int ob = k & 1;
    if (!wt_warp(sh, a.hdr, &sh->st_full[ob], (k >> 1) & 1) || !wt_warp(sh, a.hdr, &sh->o_full, k & 1)) break;
    tc_fence_after();
    const float inv = 1.f / stats[ob * kRows + row];
    uint32_t h[64];
#pragma unroll
    for (int c = 0; c < 128; c += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x16(tmem + kOCol + c, r);
      tmem_ld_32x32b_x16(tmem + kOCol + c + 16, r + 16);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; ++i)
        h[c / 2 + i] = f2_to_h2(__uint_as_float(r[2 * i]) * inv, __uint_as_float(r[2 * i + 1]) * inv);
    }
    tc_fence_before();
    warp_arrive(&sh->o_empty);
    warp_arrive(&sh->st_empty[ob]);
    const int t = u.qs + tok_in_unit;
    if (t < u.n) {
      uint4* d4 = reinterpret_cast<uint4*>(a.o + (long long)(u.ts + t) * a.o_stride +
                                           (long long)(u.h * a.gqa + head_in_unit) * kHeadDim);
#pragma unroll
      for (int i = 0; i < 16; ++i) d4[i] = make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                        const __grid_constant__ CUtensorMap tmap_v, const __grid_constant__ Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Shared* sh = reinterpret_cast<Shared*>(smem + kBarOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  grid_launch_dependents();
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh->q_full[i], 1);
      mbar_init(&sh->q_empty[i], 1);
      mbar_init(&sh->k_full[i], 1);
      mbar_init(&sh->k_empty[i], 1);
      mbar_init(&sh->v_full[i], 1);
      mbar_init(&sh->v_empty[i], 1);

      mbar_init(&sh->st_full[i], kSoftmaxWarps);
      mbar_init(&sh->st_empty[i], 4);
    }
    for (int i = 0; i < kSBufs; ++i) {
      mbar_init(&sh->s_full[i], 1);
      mbar_init(&sh->s_empty[i], 1);
      mbar_init(&sh->p_full[i], kSoftmaxWarps);
      mbar_init(&sh->pv_done[i], 1);
    }
    mbar_init(&sh->o_full, 1);
    mbar_init(&sh->o_empty, 4);
    mbar_init(&sh->pv_final, 1);

    mbar_init(&sh->mma_final, 1);
    sh->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&sh->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kLoadWarp && lane == 0) {
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }
  // Inputs (and the unit list of the plan launch) are read only after the
  // previous launch in the stream has completed.
  grid_dependency_wait();
  if (threadIdx.x == 0) sh->num_units = *reinterpret_cast<const volatile int32_t*>(args.num_units);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kLoadWarp) {
    if (lane == 0) load_role(sh, args, smem, &tmap_q, &tmap_k, &tmap_v);
  } else if (warp == kMmaWarp) {
    if (lane == 0) mma_role(sh, args, smem);
  } else if (warp == kPvWarp) {
    if (lane == 0) pv_role(sh, args, smem);
  } else if (warp >= kSoftmaxWarp0 && warp < kEpiWarp0) {
    softmax_role(sh, args, smem);
  } else {
    epilogue_role(sh, args, smem);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(sh->tmem_base, kTmemCols);
}

// ------------------------------------------------------------------ plan
constexpr int kPlanThreads = 1024;

// Inclusive suffix sums a[i] = sum_{j >= i} a[j] of n entries, by one warp.
__device__ void warp_suffix_sum(int* a, int n) {
  const int lane = threadIdx.x & 31;
  int carry = 0;
  for (int base = n - 1; base >= 0; base -= 32) {
    const int i = base - lane;
    int v = i >= 0 ? a[i] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += x;
    }
    if (i >= 0) a[i] = v + carry;
    carry += __shfl_sync(0xffffffffu, v, 31);
  }
}

// Shared memory: hist[L + 2] | cnt[L + 2] | off[L + 2] | cursor[L + 2] | sorted[S].
__global__ void __launch_bounds__(kPlanThreads)
    prefill_plan_kernel(const int32_t* __restrict__ cu, int num_seqs, int total_tokens, int tq, int num_kv_heads,
                        int max_len, int levels, long long capacity, int4* __restrict__ units, int32_t* __restrict__ num_units,
                        WorkspaceHeader* hdr) {
  extern __shared__ int plan_smem[];
  const int L2 = levels + 2;
  int* hist = plan_smem;
  int* cnt = hist + L2;
  int* off = cnt + L2;
  int* cursor = off + L2;
  int* sorted = cursor + L2;
  grid_launch_dependents();
  __shared__ int bad;
  for (int i = threadIdx.x; i < 4 * L2; i += blockDim.x) plan_smem[i] = 0;
  if (threadIdx.x == 0) bad = 0;
  grid_dependency_wait();
  __syncthreads();
  if (threadIdx.x == 0 && num_seqs > 0 && (cu[0] != 0 || cu[num_seqs] != total_tokens)) bad = 1;
  // Blocks per sequence; a sequence with a negative or too large length, or
  // outside the tokens, is recorded and left out.
  for (int s = threadIdx.x; s < num_seqs; s += blockDim.x) {
    const int a = cu[s], b = cu[s + 1], n = b - a;
    int nb = (n + tq - 1) / tq;
    if (a < 0 || b > total_tokens || n < 0 || n > max_len) {
      bad = 1;
      nb = 0;
    }
    atomicAdd(&hist[nb], 1);
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // cnt[b] = sequences with more than b blocks; off[b] = units of the levels above b.
    for (int b = threadIdx.x; b <= levels; b += 32) cnt[b] = b + 1 <= levels ? hist[b + 1] : 0;
    __syncwarp();
    warp_suffix_sum(cnt, levels + 1);
    __syncwarp();
    for (int b = threadIdx.x; b < levels; b += 32) off[b] = b + 1 < levels ? cnt[b + 1] : 0;
    __syncwarp();
    warp_suffix_sum(off, levels);
    __syncwarp();
  }
  __syncthreads();
  // Sequences by block count, most first (counting sort).
  for (int s = threadIdx.x; s < num_seqs; s += blockDim.x) {
    const int a = cu[s], b = cu[s + 1], n = b - a;
    const int nb = (a < 0 || b > total_tokens || n < 0 || n > max_len) ? 0 : (n + tq - 1) / tq;
    if (nb > 0) sorted[cnt[nb] + atomicAdd(&cursor[nb], 1)] = s;
  }
  __syncthreads();
  const long long total = levels > 0 ? (long long)num_kv_heads * (off[0] + cnt[0]) : 0;
  const bool fits = total <= capacity;
  for (long long u = threadIdx.x; fits && u < total; u += blockDim.x) {
    // Level of unit u: the smallest b with Hk * off[b] <= u (off decreases with b).
    int lo = 0, hi = levels - 1;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if ((long long)num_kv_heads * off[mid] <= u) hi = mid;
      else lo = mid + 1;
    }
    const long long i = u - (long long)num_kv_heads * off[lo];
    const int s = sorted[i / num_kv_heads];
    const int a = cu[s];
    units[u] = make_int4(a, cu[s + 1] - a, lo * tq, (int)(i % num_kv_heads));
  }
  if (threadIdx.x == 0) {
    *num_units = fits ? (int32_t)total : 0;
    if (bad || !fits) atomicOr(&hdr->error_bits, (uint32_t)kErrBadSeqlens);
  }
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

// [tokens][heads][128] fp16 with a token stride of `stride` elements, in
// boxes of 64 x box_heads x box_tokens, 128-byte swizzle.
static int token_map(CUtensorMap* map, const void* base, long long tokens, int heads, long long stride,
                     int box_heads, int box_tokens) {
  auto fn = encode_fn();
  NEB_REQUIRE(fn != nullptr, NEB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {128, (cuuint64_t)heads, (cuuint64_t)tokens};
  cuuint64_t strides[2] = {256, (cuuint64_t)stride * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_heads, (cuuint32_t)box_tokens}, estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  NEB_REQUIRE(r == CUDA_SUCCESS, NEB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return NEB_OK;
}

}  // namespace prefill

// Workspace: header | the attention workspace's counter region (kept so that
// neb_workspace_status may clear it) | unit count | units.
static size_t prefill_units_offset() { return workspace_layout(1, 1, 1, 1).plan_cache; }

static long long prefill_capacity(long long tokens, int num_seqs, int num_q_heads, int num_kv_heads) {
  const int gqa = num_q_heads / num_kv_heads;
  const int tq = prefill::kRows / gqa;
  return (long long)num_kv_heads * ((tokens + tq - 1) / tq + num_seqs);
}

static size_t prefill_plan_smem(int levels, int num_seqs) {
  return (size_t)(4 * (levels + 2) + num_seqs) * sizeof(int);
}

}  // namespace neb

using namespace neb;

extern "C" size_t neb_prefill_attention_workspace_bytes(int64_t total_tokens, int32_t num_seqs, int32_t num_q_heads,
                                                        int32_t num_kv_heads) {
  if (total_tokens < 0 || num_seqs < 0 || num_kv_heads <= 0 || num_q_heads < num_kv_heads ||
      num_q_heads % num_kv_heads != 0)
    return 0;
  return prefill_units_offset() + 256 +
         (size_t)prefill_capacity(total_tokens, num_seqs, num_q_heads, num_kv_heads) * sizeof(int4);
}

extern "C" int neb_prefill_attention(const void* q, int64_t q_stride, const void* k, int64_t k_stride, const void* v,
                                     int64_t v_stride, const int32_t* cu_seqlens, int32_t num_seqs,
                                     int64_t total_tokens, int32_t max_seqlen, int32_t num_q_heads,
                                     int32_t num_kv_heads, int32_t head_dim, float softmax_scale, void* o,
                                     int64_t o_stride, void* workspace, size_t workspace_bytes, void* stream) {
  NEB_REQUIRE(q && k && v && cu_seqlens && o && workspace, NEB_ERR_INVALID, "null pointer argument");
  NEB_REQUIRE(head_dim == kHeadDim, NEB_ERR_UNSUPPORTED, "head_dim must be 128 (got %d)", head_dim);
  NEB_REQUIRE(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0, NEB_ERR_INVALID,
              "num_q_heads (%d) must be a multiple of num_kv_heads (%d)", num_q_heads, num_kv_heads);
  const int gqa = num_q_heads / num_kv_heads;
  NEB_REQUIRE(gqa == 1 || gqa == 2 || gqa == 4 || gqa == 8 || gqa == 16, NEB_ERR_UNSUPPORTED,
              "the prefill kernel takes q/kv head ratios 1, 2, 4, 8 and 16 (got %d)", gqa);
  NEB_REQUIRE(num_seqs >= 0 && total_tokens >= 0 && total_tokens < (1ll << 31) && max_seqlen >= 0, NEB_ERR_INVALID,
              "num_seqs, total_tokens and max_seqlen must be non-negative (and total_tokens below 2^31)");
  NEB_REQUIRE(q_stride >= (int64_t)num_q_heads * kHeadDim && o_stride >= (int64_t)num_q_heads * kHeadDim &&
                  k_stride >= (int64_t)num_kv_heads * kHeadDim && v_stride >= (int64_t)num_kv_heads * kHeadDim &&
                  q_stride % 8 == 0 && k_stride % 8 == 0 && v_stride % 8 == 0 && o_stride % 8 == 0,
              NEB_ERR_INVALID, "token strides must cover the heads and be multiples of 8 elements");
  NEB_REQUIRE(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
                reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(workspace)) & 15u) == 0,
              NEB_ERR_INVALID, "q, k, v, o and the workspace must be 16-byte aligned");
  NEB_REQUIRE(workspace_bytes >= neb_prefill_attention_workspace_bytes(total_tokens, num_seqs, num_q_heads,
                                                                       num_kv_heads),
              NEB_ERR_INVALID, "workspace too small (%zu bytes)", workspace_bytes);
  if (num_seqs == 0 || total_tokens == 0) return NEB_OK;
  const int tq = prefill::kRows / gqa;
  const int levels = (max_seqlen + tq - 1) / tq;
  const size_t plan_smem = prefill_plan_smem(levels, num_seqs);
  NEB_REQUIRE(plan_smem <= 200 * 1024, NEB_ERR_UNSUPPORTED,
              "max_seqlen %d with %d sequences exceeds the plan's shared memory", max_seqlen, num_seqs);
  CUtensorMap tq_map, tk_map, tv_map;
  int rc = prefill::token_map(&tq_map, q, total_tokens, num_q_heads, q_stride, gqa, tq);
  if (rc != NEB_OK) return rc;
  rc = prefill::token_map(&tk_map, k, total_tokens, num_kv_heads, k_stride, 1, prefill::kKeys);
  if (rc != NEB_OK) return rc;
  rc = prefill::token_map(&tv_map, v, total_tokens, num_kv_heads, v_stride, 1, prefill::kKeys);
  if (rc != NEB_OK) return rc;

  int device = 0;
  NEB_CUDA(cudaGetDevice(&device));
  NEB_REQUIRE(device >= 0 && device < 64, NEB_ERR_UNSUPPORTED, "device index %d out of range", device);
  static bool attr_set[64] = {};
  static std::mutex attr_mu;
  {
    std::lock_guard<std::mutex> lock(attr_mu);
    if (!attr_set[device]) {
      NEB_CUDA(cudaFuncSetAttribute(prefill::prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)prefill::kSmemBytes));
      NEB_CUDA(cudaFuncSetAttribute(prefill::prefill_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    200 * 1024));
      attr_set[device] = true;
    }
  }
  auto* base = static_cast<uint8_t*>(workspace);
  auto* hdr = reinterpret_cast<WorkspaceHeader*>(base);
  auto* count = reinterpret_cast<int32_t*>(base + prefill_units_offset());
  auto* units = reinterpret_cast<int4*>(base + prefill_units_offset() + 256);
  const long long capacity = prefill_capacity(total_tokens, num_seqs, num_q_heads, num_kv_heads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  NEB_CUDA(launch_pdl(prefill::prefill_plan_kernel, dim3(1), dim3(prefill::kPlanThreads), plan_smem, s, cu_seqlens,
                      num_seqs, (int)total_tokens, tq, num_kv_heads, max_seqlen, levels, capacity, units, count,
                      hdr));
  prefill::Args a;
  a.units = units;
  a.num_units = count;
  a.hdr = hdr;
  a.o = static_cast<__half*>(o);
  a.o_stride = o_stride;
  a.gqa = gqa;
  a.tq = tq;
  a.num_q_heads = num_q_heads;
  a.scale_log2 = softmax_scale * 1.4426950408889634f;
  const long long workers = std::min<long long>(num_sms(device), capacity);
  NEB_CUDA(launch_pdl(prefill::prefill_attn_kernel, dim3((unsigned)workers), dim3(prefill::kThreads),
                      (size_t)prefill::kSmemBytes, s, tq_map, tk_map, tv_map, a));
  return NEB_OK;
}
