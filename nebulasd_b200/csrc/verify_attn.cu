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
// One persistent CTA per SM (plan.cuh gives each an equal share of KV tiles)
// with warp roles:
//   warp 0      TMA producer: per 16-token KV block, two 64-column boxes of K
//               and of V (128-byte swizzle) into a 4-stage ring (64 tokens/stage)
//   warp 1      MMA issuer (one thread): S = Q K^T into a double-buffered TMEM
//               tile (M=128, N=64), then O += P V (V as an MN-major operand) into
//               a TMEM accumulator (M=128, N=128)
//   warps 2..5  softmax / epilogue: read S with tcgen05.ld, masked online
//               softmax in the exp2 domain (lazy rescale of O: only when a row's
//               max grows by more than 2^8), write P (fp16) to shared memory,
//               normalise O at the end of a piece and store it, or store a
//               partial and let the last-arriving CTA of the unit merge.
// Query row j of a unit sits at MMA row 32*(j%4) + j/4, i.e. lanes 0..15 of
// each TMEM lane quadrant, so all four softmax warps share the work and the
// 16x256b TMEM loads give each thread two rows x 16 columns.
//
// Every wait is bounded (about 2 s); on expiry the kernel records an error
// bit, stops issuing work, waits (bounded) for its own copies and MMAs, frees
// its TMEM and returns.  No TMA multicast is used.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "attn_common.cuh"
#include "sm100.cuh"

namespace neb {
using namespace sm100;

// Timeline hooks: empty unless the library is built with -DNEB_TRACE, in which
// case each CTA stamps %globaltimer into a caller-provided buffer (offline
// profiling of the pipeline; the shipped build contains no tracing code).
#ifdef NEB_TRACE
__device__ unsigned long long* g_trace = nullptr;
#define NEB_TRACE_POINT(i)                                                                      \
  do {                                                                                          \
    if (g_trace) {                                                                              \
      unsigned long long t_;                                                                    \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                    \
      g_trace[blockIdx.x * 2048 + (i)] = t_;                                                     \
    }                                                                                           \
  } while (0)
#else
#define NEB_TRACE_POINT(i) \
  do {                     \
  } while (0)
#endif

constexpr int kVThreads = 384;        // 12 warps: 0 TMA, 1 MMA, 2-3 idle, 4-11 softmax
constexpr int kSoftmaxWarp0 = 4;
constexpr int kSoftmaxThreads = 256;
constexpr int kStageBlocks = 4;    // 16-token KV blocks per pipeline stage
constexpr int kStages = 4;         // KV ring depth
constexpr int kMaxQRows = 128;     // query rows per unit: the MMA's M
constexpr uint32_t kTmemCols = 512;  // S: 2 x 64 columns, O: 128 columns, row sums: 16 columns
constexpr uint32_t kOCol = 128;
constexpr uint32_t kSumCol = 256;   // P x ones: every column holds the row's running sum of P

constexpr long long kWaitLimit = 4000000000LL;

// Shared memory map (offsets from a 1024-byte aligned base).
constexpr uint32_t kQOff = 0;                               // 2 d-halves x 128 rows x 128 B
constexpr uint32_t kKVOff = 32768;                          // per stage: K (2 x 8 KiB), V (2 x 8 KiB)
constexpr uint32_t kStageBytes = 32768;
constexpr uint32_t kPOff = kKVOff + kStages * kStageBytes;  // 2 buffers x 128 rows x 128 B
constexpr uint32_t kOnesOff = kPOff + 2 * 16384;            // 16 rows x 128 B of fp16 ones (row-sum MMA)
constexpr uint32_t kBarOff = kOnesOff + 2048;
constexpr uint32_t kPlanOff = kBarOff + 1024;
constexpr int kVerifyMaxRows = 3900;  // keeps the plan arrays inside 227 KiB of shared memory

struct VerifyShared {
  uint64_t kv_full[kStages];   // K and V of a stage landed (softmax reads the block flags)
  uint64_t k_full[kStages];    // K landed
  uint64_t v_full[kStages];    // V landed
  uint64_t k_empty[kStages];   // S of the stage completed: K slot reusable
  uint64_t kv_empty[kStages];  // O += P V of the stage completed: V slot reusable
  uint64_t s_full[2];
  uint64_t s_empty[2];
  uint64_t p_full[2];
  uint64_t pv_done[2];
  uint64_t q_full;
  uint64_t q_empty;
  uint64_t o_empty;
  uint64_t mma_final;
  uint64_t epi_bar;  // bounded barrier of the 128 softmax threads
  uint32_t tmem_base;
  int32_t abort_flag;
  int32_t last_flag;
  int32_t blk[kStages][kStageBlocks];
};
static_assert(sizeof(VerifyShared) <= 1024, "barrier block fits its slot");

__host__ __device__ inline size_t verify_smem_bytes(int num_rows) {
  return 1024 + kPlanOff + plan_smem_bytes(num_rows);
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
  __device__ void init(const PlanSmem* planp, int ngroups, int kvh, long long begin, long long end) {
    ps = planp;
    ng = ngroups;
    hk = kvh;
    t = begin;
    t_end = end;
    g = begin < end ? find_group(ps->gprefix, ng, begin, hk) : 0;
  }
  // Fills (g, kv_head, tile_lo, tile_hi, nb, unit_start); false when done.
  __device__ bool next(int& grp, int& kv_head, int& lo, int& hi, int& nb, long long& unit_start) {
    if (t >= t_end) return false;
    while ((long long)hk * ps->gprefix[g + 1] <= t) ++g;
    nb = ps->gprefix[g + 1] - ps->gprefix[g];
    const long long gbase = (long long)hk * ps->gprefix[g];
    kv_head = (int)((t - gbase) / nb);
    lo = (int)(t - gbase - (long long)kv_head * nb);
    const int cnt = (int)min((long long)(nb - lo), t_end - t);
    hi = lo + cnt;
    unit_start = gbase + (long long)kv_head * nb;
    grp = g;
    t += cnt;
    return true;
  }
};

__device__ __forceinline__ int stages_of(int lo, int hi) { return (hi - lo + kStageBlocks - 1) / kStageBlocks; }

__device__ __forceinline__ void raise_abort(VerifyShared* sh, const AttnParams& p) {
  if (atomicExch(&sh->abort_flag, 1) == 0) record_error(p, kErrTimeout);
}
__device__ __forceinline__ bool aborted(VerifyShared* sh) {
  return *reinterpret_cast<volatile int32_t*>(&sh->abort_flag) != 0;
}
__device__ __forceinline__ bool wait_or_abort(VerifyShared* sh, const AttnParams& p, uint64_t* bar,
                                              uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (aborted(sh) || clock64() - t0 > kWaitLimit) {
      raise_abort(sh, p);
      return false;
    }
  }
  return true;
}

// One arrival per softmax warp (count 4): the warp's lanes are first gathered
// with __syncwarp, which orders their earlier shared/tensor-memory work.
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// Barrier of the 128 softmax threads built on an mbarrier, so that it is bounded.
__device__ __forceinline__ bool epi_sync(VerifyShared* sh, const AttnParams& p, uint32_t& phase) {
  warp_arrive(&sh->epi_bar);
  const bool ok = wait_or_abort(sh, p, &sh->epi_bar, phase & 1);
  ++phase;
  return ok;
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) { return f2_to_h2(a, b); }

__global__ void __launch_bounds__(kVThreads, 1)
    verify_attn_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                       const __grid_constant__ VerifyArgs args) {
  const AttnParams& p = args.p;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  VerifyShared* sh = reinterpret_cast<VerifyShared*>(smem + kBarOff);
  int* plan_mem = reinterpret_cast<int*>(smem + kPlanOff);
  __shared__ int scratch[32];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) NEB_TRACE_POINT(0);
  PlanSmem ps{plan_mem, plan_mem + (p.num_rows + 1), plan_mem + 2 * (p.num_rows + 1)};
  build_plan(ps, scratch, p.seq_ids, p.seq_lens, p.num_rows, p.max_group_rows);
  const int ng = ps.misc[0];
  if (threadIdx.x == 0) NEB_TRACE_POINT(1);
  const int hk = p.num_kv_heads;
  const int gqa = p.num_q_heads / p.num_kv_heads;
  const long long total = (long long)hk * ps.gprefix[ng];
  const long long launched = gridDim.x;
  const long long w = blockIdx.x;
  if (warp >= kSoftmaxWarp0)
    write_nan_rows(p, ps, ng, w * 8 + (warp - kSoftmaxWarp0), launched * 8);
  if (total == 0) return;
  const long long workers = launched < total ? launched : total;
  if (w >= workers) return;
  const long long t_begin = range_begin(w, total, workers);
  const long long t_end = range_begin(w + 1, total, workers);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sh->kv_full[i], 1);
      mbar_init(&sh->k_full[i], 1);
      mbar_init(&sh->v_full[i], 1);
      mbar_init(&sh->k_empty[i], 1);
      mbar_init(&sh->kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh->s_full[i], 1);
      mbar_init(&sh->s_empty[i], 8);
      mbar_init(&sh->p_full[i], 8);
      mbar_init(&sh->pv_done[i], 1);
    }
    mbar_init(&sh->q_full, 8);
    mbar_init(&sh->q_empty, 1);
    mbar_init(&sh->o_empty, 8);
    mbar_init(&sh->mma_final, 1);
    mbar_init(&sh->epi_bar, 8);
    sh->abort_flag = 0;
    sh->last_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sh->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  if (threadIdx.x == 0) NEB_TRACE_POINT(2);
  const uint32_t q_base = smem_u32(smem + kQOff);
  const uint32_t kv_base = smem_u32(smem + kKVOff);
  const uint32_t p_base = smem_u32(smem + kPOff);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // The whole warp looks up 32 block ids at a time (one coalesced read of the
    // block table); lane 0 waits for free slots and issues the copies.
    if (lane == 0) {
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
    }
    PieceCursor cur;
    cur.init(&ps, ng, hk, t_begin, t_end);
    int g, h, lo, hi, nb;
    long long ustart;
    long long G = 0;
    bool ok = true;
    while (ok && cur.next(g, h, lo, hi, nb, ustart)) {
      const int sid = p.seq_ids[ps.gfirst[g]];
      for (int base = lo; base < hi && ok; base += 32) {
        const int tile = base + lane;
        int my_row = args.oob_row, my_valid = 0;
        if (tile < hi) {
          const long long blk = lookup_block(p, sid, tile);
          if (blk >= 0) {
            my_valid = 1;
            my_row = (int)(((blk * p.num_layers + p.cur_layer) * hk + h) * kBlockTokens);
          }
        }
        const int nt = min(32, hi - base);
        for (int s0 = 0; s0 < nt; s0 += kStageBlocks, ++G) {
          const int nblk = min(kStageBlocks, nt - s0);
          const int slot = (int)(G % kStages);
          const uint32_t ph = (uint32_t)(((G / kStages) & 1) ^ 1);
          int rows[kStageBlocks], valid[kStageBlocks];
#pragma unroll
          for (int b = 0; b < kStageBlocks; ++b) {
            rows[b] = __shfl_sync(0xffffffffu, my_row, s0 + b);
            valid[b] = __shfl_sync(0xffffffffu, my_valid, s0 + b);
          }
          int waited = 1;
          if (lane == 0) {
            uint8_t* kst = smem + kKVOff + slot * kStageBytes;
            // K first: its slot frees as soon as S of the stage G-kStages is done.
            waited = wait_or_abort(sh, p, &sh->k_empty[slot], ph);
            if (waited) {
              if (G < 100) NEB_TRACE_POINT(8 + G);
              mbar_arrive_expect_tx(&sh->k_full[slot], (uint32_t)nblk * 2u * 2048u);
              for (int b = 0; b < nblk; ++b) {
                tma_load_2d(kst + b * 2048, &tmap_k, &sh->k_full[slot], 0, rows[b]);
                tma_load_2d(kst + 8192 + b * 2048, &tmap_k, &sh->k_full[slot], 64, rows[b]);
              }
              waited = wait_or_abort(sh, p, &sh->kv_empty[slot], ph);
            }
            if (waited) {
              if (G < 100) NEB_TRACE_POINT(508 + G);
              mbar_arrive_expect_tx(&sh->v_full[slot], (uint32_t)nblk * 2u * 2048u);
              for (int b = 0; b < nblk; ++b) {
                tma_load_2d(kst + 16384 + b * 2048, &tmap_v, &sh->v_full[slot], 0, rows[b]);
                tma_load_2d(kst + 16384 + 8192 + b * 2048, &tmap_v, &sh->v_full[slot], 64, rows[b]);
              }
              // The flags of stage G go in only now: the softmax of stage G - kStages,
              // the previous reader of this slot, finished before its P V completed.
              for (int b = 0; b < nblk; ++b) sh->blk[slot][b] = valid[b];
              mbar_arrive(&sh->kv_full[slot]);
            }
          }
          waited = __shfl_sync(0xffffffffu, waited, 0);
          if (!waited) {
            ok = false;
            break;
          }
          __syncwarp();
        }
      }
    }
    // Wait (bounded) for every copy this CTA issued before the CTA can exit.
    if (lane == 0)
      for (long long Gi = (G > kStages ? G - kStages : 0); Gi < G; ++Gi) {
        mbar_wait(&sh->k_full[Gi % kStages], (uint32_t)((Gi / kStages) & 1), kWaitLimit);
        mbar_wait(&sh->v_full[Gi % kStages], (uint32_t)((Gi / kStages) & 1), kWaitLimit);
      }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    // Polls the barriers and issues whichever is ready first: S(G) for the next
    // stage, or O += P V for the oldest stage whose P is written.  Up to two
    // P V products may be pending, so neither waits for the other's inputs.
    if (lane == 0) {
      PieceCursor cur;
      cur.init(&ps, ng, hk, t_begin, t_end);
      int g, h, lo, hi, nb;
      long long ustart;
      int piece = -1, s_in_piece = 0, nst = 0;
      struct Stage {
        int nblk, first, last, piece;
      };
      auto next_stage = [&](Stage& st) -> bool {
        if (s_in_piece == nst) {
          if (!cur.next(g, h, lo, hi, nb, ustart)) return false;
          ++piece;
          nst = stages_of(lo, hi);
          s_in_piece = 0;
        }
        st.nblk = min(kStageBlocks, hi - (lo + s_in_piece * kStageBlocks));
        st.first = s_in_piece == 0;
        st.last = s_in_piece == nst - 1;
        st.piece = piece;
        ++s_in_piece;
        return true;
      };
      const uint32_t idesc_pv = idesc_f16_f32(128, 128, false, true);
      const uint32_t idesc_sum = idesc_f16_f32(128, 16, false, false);
      const uint32_t ones_base = smem_u32(smem + kOnesOff);
      Stage nxt, pend[2];
      long long pend_g[2] = {0, 0};
      int npend = 0, phead = 0;
      bool have = next_stage(nxt);
      long long Gs = 0;
      long long t_idle = clock64();
      while (have || npend > 0) {
        bool progress = false;
        if (npend > 0) {
          const Stage& st = pend[phead];
          const long long Gp = pend_g[phead];
          bool ready = mbar_test_wait(&sh->p_full[Gp & 1], (uint32_t)((Gp >> 1) & 1)) &&
                       mbar_test_wait(&sh->v_full[Gp % kStages], (uint32_t)((Gp / kStages) & 1));
          if (ready && st.first && st.piece > 0) ready = mbar_test_wait(&sh->o_empty, (uint32_t)((st.piece - 1) & 1));
          if (ready) {
            if (Gp < 100) NEB_TRACE_POINT(208 + Gp);
            tc_fence_after();
            const int sb = (int)(Gp & 1), slot = (int)(Gp % kStages);
            const uint32_t vst = kv_base + slot * kStageBytes + 16384;
            for (int kb = 0; kb < st.nblk; ++kb) {
              const uint64_t a = smem_desc_sw128(p_base + sb * 16384 + kb * 32, 16, 1024);
              const uint64_t b = smem_desc_sw128(vst + kb * 2048, 8192, 1024);
              const uint32_t acc = (st.first && kb == 0) ? 0u : 1u;
              mma_f16(tmem + kOCol, a, b, idesc_pv, acc);
              mma_f16(tmem + kSumCol, a, smem_desc_sw128(ones_base + (kb & 3) * 32, 16, 1024), idesc_sum, acc);
            }
            mma_commit(&sh->kv_empty[slot]);
            mma_commit(&sh->pv_done[sb]);
            phead ^= 1;
            --npend;
            progress = true;
          }
        }
        if (have && npend < 2) {
          bool ready = true;
          if (nxt.first) ready = mbar_test_wait(&sh->q_full, (uint32_t)(nxt.piece & 1));
          ready = ready && mbar_test_wait(&sh->k_full[Gs % kStages], (uint32_t)((Gs / kStages) & 1)) &&
                  mbar_test_wait(&sh->s_empty[Gs & 1], (uint32_t)(((Gs >> 1) & 1) ^ 1));
          if (ready) {
            if (Gs < 100) NEB_TRACE_POINT(108 + Gs);
            tc_fence_after();
            const int sb = (int)(Gs & 1);
            const uint32_t idesc_s = idesc_f16_f32(128, 16 * nxt.nblk, false, false);
            const uint32_t kst = kv_base + (int)(Gs % kStages) * kStageBytes;
            for (int kk = 0; kk < 8; ++kk) {
              const uint64_t a = smem_desc_sw128(q_base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
              const uint64_t b = smem_desc_sw128(kst + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024);
              mma_f16(tmem + sb * 64, a, b, idesc_s, kk > 0 ? 1u : 0u);
            }
            mma_commit(&sh->s_full[sb]);
            mma_commit(&sh->k_empty[Gs % kStages]);
            if (nxt.last) mma_commit(&sh->q_empty);
            const int slot_in = (phead + npend) & 1;
            pend[slot_in] = nxt;
            pend_g[slot_in] = Gs;
            ++npend;
            ++Gs;
            have = next_stage(nxt);
            progress = true;
          }
        }
        if (progress) {
          t_idle = clock64();
        } else if (aborted(sh) || clock64() - t_idle > kWaitLimit) {
          raise_abort(sh, p);
          break;
        } else {
          // Back off: a tight poll of the barriers competes with the softmax
          // warps for the shared-memory pipe.
          __nanosleep(40);
        }
      }
      mma_commit(&sh->mma_final);
      mbar_wait(&sh->mma_final, 0, kWaitLimit);
    }
  } else if (warp >= kSoftmaxWarp0) {
    // ------------------------------------------------- softmax and epilogue
    const int tid = threadIdx.x - kSoftmaxWarp0 * 32;  // 0..255
    const int wg = (warp - kSoftmaxWarp0) >> 2;          // warpgroup: which 16-lane half of the quadrant
    const int qd = warp & 3;                             // TMEM lane quadrant of this warp
    const int q4 = lane & 3;
    const int li_a = lane >> 2, li_b = li_a + 8;           // lanes within the warpgroup's half
    const int ja = (2 * li_a + wg) * 4 + qd, jb = (2 * li_b + wg) * 4 + qd;  // unit query rows
    const int ma = qd * 32 + wg * 16 + li_a, mb = ma + 8;  // MMA rows
    const uint32_t lane_addr = (uint32_t)(qd * 32 + wg * 16) << 16;
    // Clear Q and P once: rows no unit writes must hold finite values.
    for (int i = tid; i < (32768 + 32768) / 16; i += kSoftmaxThreads) {
      uint8_t* dst = i < 2048 ? smem + kQOff + i * 16 : smem + kPOff + (i - 2048) * 16;
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
    named_bar_sync(1, kSoftmaxThreads);
    for (int i = tid; i < 2048 / 16; i += kSoftmaxThreads)
      *reinterpret_cast<uint4*>(smem + kOnesOff + i * 16) = make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);
    PieceCursor cur;
    cur.init(&ps, ng, hk, t_begin, t_end);
    int g, h, lo, hi, nb;
    long long ustart;
    auto load_q = [&](int grp, int kv_head) {
      const int first_row = ps.gfirst[grp];
      const int nq = (ps.gfirst[grp + 1] - first_row) * gqa;
      for (int i = tid; i < nq * 16; i += kSoftmaxThreads) {
        const int j = i >> 4, c = i & 15;
        const int row = first_row + j / gqa;
        const int head = kv_head * gqa + j % gqa;
        uint4 v = *reinterpret_cast<const uint4*>(p.q + ((long long)row * p.num_q_heads + head) * kHeadDim + c * 8);
        // Fold softmax_scale * log2(e) into Q: S then comes out in the exp2 domain.
        uint32_t* w4 = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = h2_to_f2(w4[e]);
          w4[e] = pack_half2(f.x * p.scale_log2, f.y * p.scale_log2);
        }
        const int m = (j & 3) * 32 + ((j >> 2) & 1) * 16 + (j >> 3);
        uint8_t* dst = smem + kQOff + (c >> 3) * 16384 + m * 128 + (((c & 7) ^ (m & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = v;
      }
      fence_proxy_async_smem();
      warp_arrive(&sh->q_full);
    };
    bool have = cur.next(g, h, lo, hi, nb, ustart);
    if (have) load_q(g, h);
    long long G = 0;
    int pi = 0;
    uint32_t epi_phase = 0;
    bool ok = true;
    while (have && ok) {
      const int first_row = ps.gfirst[g];
      const int nrows = ps.gfirst[g + 1] - first_row;
      const int nq = nrows * gqa;
      const int len_a = ja < nq ? p.seq_lens[first_row + ja / gqa] : -1;
      const int len_b = jb < nq ? p.seq_lens[first_row + jb / gqa] : -1;
      // Warp-uniform: does any lane of this warp own a second query row?
      const bool has_b = __any_sync(0xffffffffu, jb < nq);
      float m_a = neg_inf(), m_b = neg_inf();
      const int nst = stages_of(lo, hi);
      for (int s = 0; s < nst; ++s, ++G) {
        const int slot = (int)(G % kStages);
        const int sb = (int)(G & 1);
        if (!wait_or_abort(sh, p, &sh->kv_full[slot], (uint32_t)((G / kStages) & 1)) ||
            !wait_or_abort(sh, p, &sh->s_full[sb], (uint32_t)((G >> 1) & 1))) {
          ok = false;
          break;
        }
        if (tid == 0 && G < 100) NEB_TRACE_POINT(308 + G);
        tc_fence_after();
        uint32_t sr[32];
        tmem_ld_16x256b_x8(tmem + sb * 64 + lane_addr, sr);
        tmem_wait_ld();
        tc_fence_before();
        warp_arrive(&sh->s_empty[sb]);
        const int t0 = lo + s * kStageBlocks;
        const int nblk = min(kStageBlocks, hi - t0);
        const int tok0 = t0 * kBlockTokens;
        float xa[16], xb[16];
        float mxa = neg_inf(), mxb = neg_inf();
        // Interior stages (every block present, every token below both rows'
        // lengths, or the row absent) need no per-element mask.
        bool blocks_ok = true;
        for (int b = 0; b < nblk; ++b) blocks_ok = blocks_ok && sh->blk[slot][b] != 0;
        const int tok_end = tok0 + 16 * nblk;
        const bool fast = __all_sync(0xffffffffu, blocks_ok && nblk == kStageBlocks &&
                                                      (len_a < 0 || tok_end <= len_a) && (len_b < 0 || tok_end <= len_b));
        if (fast && !has_b) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            xa[i] = len_a >= 0 ? __uint_as_float(sr[4 * (i >> 1) + (i & 1)]) : neg_inf();
            mxa = fmaxf(mxa, xa[i]);
          }
        } else if (fast) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int r = i >> 1, e = i & 1;
            xa[i] = len_a >= 0 ? __uint_as_float(sr[4 * r + e]) : neg_inf();
            xb[i] = len_b >= 0 ? __uint_as_float(sr[4 * r + 2 + e]) : neg_inf();
            mxa = fmaxf(mxa, xa[i]);
            mxb = fmaxf(mxb, xb[i]);
          }
        } else {
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const bool blk_ok = (r >> 1) < nblk && sh->blk[slot][r >> 1] != 0;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int tok = tok0 + 8 * r + 2 * q4 + e;
              const bool va = blk_ok && tok < len_a;
              const bool vb = blk_ok && tok < len_b;
              xa[2 * r + e] = va ? __uint_as_float(sr[4 * r + e]) : neg_inf();
              xb[2 * r + e] = vb ? __uint_as_float(sr[4 * r + 2 + e]) : neg_inf();
              mxa = fmaxf(mxa, xa[2 * r + e]);
              mxb = fmaxf(mxb, xb[2 * r + e]);
            }
          }
        }
        mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
        mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
        if (has_b) {
          mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
          mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
        }
        // Lazy rescale: the running max moves only when it grows by more than 8 (x256).
        float alpha_a = 1.f, alpha_b = 1.f;
        if (m_a == neg_inf()) {
          m_a = mxa;
        } else if (mxa > m_a + 8.f) {
          alpha_a = fast_exp2(m_a - mxa);
          m_a = mxa;
        }
        if (m_b == neg_inf()) {
          m_b = mxb;
        } else if (mxb > m_b + 8.f) {
          alpha_b = fast_exp2(m_b - mxb);
          m_b = mxb;
        }
        // P = 2^(s - m) in fp16 pairs (the MMA operand); rows with nothing
        // unmasked yet (m = -inf) get zeros.  Row sums come from the tensor core.
        uint32_t pa[8], pb[8];
        const bool live_a = m_a != neg_inf(), live_b = m_b != neg_inf();
#pragma unroll
        for (int r = 0; r < 8; ++r) pa[r] = live_a ? ex2_f16x2(pack_half2(xa[2 * r] - m_a, xa[2 * r + 1] - m_a)) : 0u;
        if (has_b) {
#pragma unroll
          for (int r = 0; r < 8; ++r) pb[r] = live_b ? ex2_f16x2(pack_half2(xb[2 * r] - m_b, xb[2 * r + 1] - m_b)) : 0u;
        }
        // P buffer sb is free once PV(G-2) completed.
        if (G >= 2 && !wait_or_abort(sh, p, &sh->pv_done[sb], (uint32_t)(((G - 2) >> 1) & 1))) {
          ok = false;
          break;
        }
        const bool rescale = __any_sync(0xffffffffu, alpha_a != 1.f || alpha_b != 1.f) && s > 0;
        if (rescale) {
          if (!wait_or_abort(sh, p, &sh->pv_done[(G - 1) & 1], (uint32_t)(((G - 1) >> 1) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t orr[32];
            const uint32_t oaddr = tmem + kOCol + half * 64 + lane_addr;
            tmem_ld_16x256b_x8(oaddr, orr);
            tmem_wait_ld();
#pragma unroll
            for (int r = 0; r < 8; ++r) {
              orr[4 * r + 0] = __float_as_uint(__uint_as_float(orr[4 * r + 0]) * alpha_a);
              orr[4 * r + 1] = __float_as_uint(__uint_as_float(orr[4 * r + 1]) * alpha_a);
              orr[4 * r + 2] = __float_as_uint(__uint_as_float(orr[4 * r + 2]) * alpha_b);
              orr[4 * r + 3] = __float_as_uint(__uint_as_float(orr[4 * r + 3]) * alpha_b);
            }
            tmem_st_16x256b_x8(oaddr, orr);
          }
          uint32_t srr[8];
          tmem_ld_16x256b_x2(tmem + kSumCol + lane_addr, srr);
          tmem_wait_ld();
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            srr[4 * r + 0] = __float_as_uint(__uint_as_float(srr[4 * r + 0]) * alpha_a);
            srr[4 * r + 1] = __float_as_uint(__uint_as_float(srr[4 * r + 1]) * alpha_a);
            srr[4 * r + 2] = __float_as_uint(__uint_as_float(srr[4 * r + 2]) * alpha_b);
            srr[4 * r + 3] = __float_as_uint(__uint_as_float(srr[4 * r + 3]) * alpha_b);
          }
          tmem_st_16x256b_x2(tmem + kSumCol + lane_addr, srr);
          tmem_wait_st();
        }
        uint8_t* pbuf = smem + kPOff + sb * 16384;
#pragma unroll
        for (int r = 0; r < 8; ++r)
          *reinterpret_cast<uint32_t*>(pbuf + ma * 128 + ((r ^ (ma & 7)) << 4) + q4 * 4) = pa[r];
        if (has_b) {
#pragma unroll
          for (int r = 0; r < 8; ++r)
            *reinterpret_cast<uint32_t*>(pbuf + mb * 128 + ((r ^ (mb & 7)) << 4) + q4 * 4) = pb[r];
        }
        fence_proxy_async_smem();
        tc_fence_before();
        warp_arrive(&sh->p_full[sb]);
        if (tid == 0 && G < 100) NEB_TRACE_POINT(408 + G);
      }
      if (!ok) break;
      // Load the next piece's Q as soon as this piece's S products are done with it.
      int g2, h2, lo2, hi2, nb2;
      long long ustart2;
      const bool have_next = cur.next(g2, h2, lo2, hi2, nb2, ustart2);
      if (have_next) {
        if (!wait_or_abort(sh, p, &sh->q_empty, (uint32_t)(pi & 1))) break;
        load_q(g2, h2);
      }
      // Epilogue of this piece.
      const long long Gl = G - 1;
      if (!wait_or_abort(sh, p, &sh->pv_done[Gl & 1], (uint32_t)((Gl >> 1) & 1))) break;
      tc_fence_after();
      uint32_t o0[32], o1[32], sums[8];
      tmem_ld_16x256b_x8(tmem + kOCol + lane_addr, o0);
      tmem_ld_16x256b_x8(tmem + kOCol + 64 + lane_addr, o1);
      tmem_ld_16x256b_x2(tmem + kSumCol + lane_addr, sums);
      tmem_wait_ld();
      tc_fence_before();
      warp_arrive(&sh->o_empty);
      const float l_a = __uint_as_float(sums[0]), l_b = __uint_as_float(sums[2]);
      const float inv_a = 1.f / l_a, inv_b = 1.f / l_b;
      const bool whole = (lo == 0 && hi == nb);
      const long long unit = (long long)g * hk + h;
      long long w0 = 0, w1 = 0, slot = 0;
      if (!whole) {
        w0 = worker_of(ustart, total, workers);
        w1 = worker_of(ustart + nb - 1, total, workers);
        slot = piece_slot(w, w0);
      }
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int j = x == 0 ? ja : jb;
        if (j >= nq) continue;
        const float inv = x == 0 ? inv_a : inv_b;
        const int row = first_row + j / gqa;
        const int head = h * gqa + j % gqa;
        if (whole) {
          __half* dst = p.o + ((long long)row * p.num_q_heads + head) * kHeadDim;
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const int d = 8 * r + 2 * q4;
            *reinterpret_cast<uint32_t*>(dst + d) =
                pack_half2(__uint_as_float(o0[4 * r + 2 * x]) * inv, __uint_as_float(o0[4 * r + 2 * x + 1]) * inv);
            *reinterpret_cast<uint32_t*>(dst + 64 + d) =
                pack_half2(__uint_as_float(o1[4 * r + 2 * x]) * inv, __uint_as_float(o1[4 * r + 2 * x + 1]) * inv);
          }
        } else {
          float* dst = p.part_o + (slot * p.nq + j) * kHeadDim;
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const int d = 8 * r + 2 * q4;
            __stcg(reinterpret_cast<float2*>(dst + d),
                   make_float2(__uint_as_float(o0[4 * r + 2 * x]) * inv, __uint_as_float(o0[4 * r + 2 * x + 1]) * inv));
            __stcg(reinterpret_cast<float2*>(dst + 64 + d),
                   make_float2(__uint_as_float(o1[4 * r + 2 * x]) * inv, __uint_as_float(o1[4 * r + 2 * x + 1]) * inv));
          }
          if (q4 == 0) {
            const float l = x == 0 ? l_a : l_b;
            const float m = x == 0 ? m_a : m_b;
            __stcg(p.part_lse + slot * p.nq + j, l > 0.f ? m + __log2f(l) : neg_inf());
          }
        }
      }
      if (!whole) {
        __threadfence();
        if (!epi_sync(sh, p, epi_phase)) break;
        if (tid == 0) {
          const int last = atomicAdd(p.counters + unit, 1) == (int)(w1 - w0);
          if (last) p.counters[unit] = 0;  // every piece has arrived: ready for the next call
          sh->last_flag = last;
        }
        if (!epi_sync(sh, p, epi_phase)) break;
        if (sh->last_flag) {
          __threadfence();
          merge_unit_warp(p, first_row, nrows, h, gqa, w0, w1, warp - kSoftmaxWarp0, 8);
        }
      }
      have = have_next;
      g = g2; h = h2; lo = lo2; hi = hi2; nb = nb2; ustart = ustart2;
      ++pi;
    }
  }
  if (warp == 2 && lane == 0) NEB_TRACE_POINT(3);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
  if (threadIdx.x == 0) NEB_TRACE_POINT(4);
}

// ------------------------------------------------------------------ host side
long long verify_workers(int device) { return num_sms(device); }

int verify_group_rows(int gqa) {
  if (gqa < 1 || gqa > 64) return 0;
  return kMaxQRows / gqa;
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

// Tensor map over a cache viewed as [rows = NB*L*Hk*16, 128] fp16 with 64x16 boxes.
static int kv_tensor_map(CUtensorMap* map, const void* base, unsigned long long rows) {
  struct Entry {
    const void* base;
    unsigned long long rows;
    CUtensorMap map;
  };
  static std::mutex mu;
  static Entry cache[16];
  static int next = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (auto& e : cache)
      if (e.base == base && e.rows == rows) {
        *map = e.map;
        return NEB_OK;
      }
  }
  auto fn = encode_fn();
  NEB_REQUIRE(fn != nullptr, NEB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {128, rows};
  cuuint64_t strides[1] = {256};
  cuuint32_t box[2] = {64, 16};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  NEB_REQUIRE(r == CUDA_SUCCESS, NEB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  std::lock_guard<std::mutex> lock(mu);
  cache[next] = Entry{base, rows, *map};
  next = (next + 1) % 16;
  return NEB_OK;
}

int launch_verify(const AttnParams& p, long long workers, cudaStream_t stream) {
  const unsigned long long rows =
      (unsigned long long)p.num_blocks * p.num_layers * p.num_kv_heads * kBlockTokens;
  NEB_REQUIRE(rows + kBlockTokens < (1ull << 31), NEB_ERR_UNSUPPORTED,
              "KV cache of %llu rows exceeds the verify kernel's 2^31-row tensor map", rows);
  NEB_REQUIRE(p.num_rows <= kVerifyMaxRows, NEB_ERR_UNSUPPORTED,
              "verify attention takes at most %d rows per call (got %d)", kVerifyMaxRows, p.num_rows);
  NEB_REQUIRE(p.max_group_rows * (p.num_q_heads / p.num_kv_heads) <= kMaxQRows, NEB_ERR_INVALID,
              "group rows exceed the MMA tile");
  CUtensorMap tk, tv;
  int rc = kv_tensor_map(&tk, p.k_cache, rows);
  if (rc != NEB_OK) return rc;
  rc = kv_tensor_map(&tv, p.v_cache, rows);
  if (rc != NEB_OK) return rc;
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
  verify_attn_kernel<<<(unsigned)workers, kVThreads, smem, stream>>>(tk, tv, a);
  NEB_CUDA(cudaGetLastError());
  return NEB_OK;
}

}  // namespace neb
