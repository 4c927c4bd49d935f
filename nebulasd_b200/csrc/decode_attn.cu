// Draft single-token decode attention: CUDA cores, no tensor cores.
//
// Replaces the reference's two-phase Triton paged decode attention
// (swiftLLM/swiftllm/worker/kernels/paged_attn.py:9-149), which launches one
// single-warp program per (row, q-head, seq-block) and so reads every KV tile
// once per q head of the GQA group, then merges fp32 partials in a second
// launch.  Here one warp streams a KV tile once for all `GQA` q heads of its kv
// head, the split-K merge happens in the same launch, and the work split is
// balanced by bytes (plan.cuh).
//
// Warp layout over one 16x128 fp16 tile (4 KiB): lane l owns the 16-byte
// column chunk dc = l % 16 (8 head-dim values) of tokens tp, tp+2, ..., tp+14
// with tp = l / 16, so each of the 8 128-bit loads of a warp covers 512
// contiguous bytes.  QK partial dots are reduced over the 16 lanes of a token
// with xor shuffles; P.V accumulates per lane in fp32 and the two token halves
// are combined once at the end of a piece.
#include "attn_common.cuh"

namespace neb {

constexpr int kDecodeThreads = 128;
constexpr int kDecodeWarps = kDecodeThreads / 32;

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  float2 a = h2_to_f2(v.x), b = h2_to_f2(v.y), c = h2_to_f2(v.z), d = h2_to_f2(v.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

template <int GQA>
__device__ void decode_piece(const AttnParams& p, int row, int kv_head, int tile_lo, int tile_hi,
                             int nb, long long unit_start, long long unit, long long w,
                             long long workers, long long total) {
  const int lane = threadIdx.x & 31, dc = lane & 15, tp = lane >> 4;
  const int sid = p.seq_ids[row];
  const int len = p.seq_lens[row];
  if ((sid < 0 || sid >= p.bt_rows) && lane == 0) record_error(p, kErrSeqId);

  float qf[GQA][8];
#pragma unroll
  for (int g = 0; g < GQA; ++g) {
    const uint4 v = *reinterpret_cast<const uint4*>(
        p.q + ((long long)row * p.num_q_heads + kv_head * GQA + g) * kHeadDim + dc * 8);
    unpack8(v, qf[g]);
#pragma unroll
    for (int e = 0; e < 8; ++e) qf[g][e] *= p.scale_log2;
  }
  float m[GQA], l[GQA], acc[GQA][8];
#pragma unroll
  for (int g = 0; g < GQA; ++g) {
    m[g] = neg_inf();
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
  }

  for (int tile = tile_lo; tile < tile_hi; ++tile) {
    const long long blk = lookup_block(p, sid, tile);
    uint4 kr[8], vr[8];
    if (blk >= 0) {
      const long long base = tile_offset(p, blk, kv_head) + tp * kHeadDim + dc * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) kr[i] = ld_stream_v4(p.k_cache + base + i * 2 * kHeadDim);
#pragma unroll
      for (int i = 0; i < 8; ++i) vr[i] = ld_stream_v4(p.v_cache + base + i * 2 * kHeadDim);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) kr[i] = vr[i] = make_uint4(0, 0, 0, 0);
    }
    float s[GQA][8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float kf[8];
      unpack8(kr[i], kf);
#pragma unroll
      for (int g = 0; g < GQA; ++g) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) d = fmaf(qf[g][e], kf[e], d);
        s[g][i] = d;
      }
    }
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
#pragma unroll
      for (int g = 0; g < GQA; ++g)
#pragma unroll
        for (int i = 0; i < 8; ++i) s[g][i] += __shfl_xor_sync(0xffffffffu, s[g][i], o);
    }
    const int tok0 = tile * kBlockTokens + tp;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const bool valid = blk >= 0 && (tok0 + 2 * i) < len;
#pragma unroll
      for (int g = 0; g < GQA; ++g) s[g][i] = valid ? s[g][i] : neg_inf();
    }
    // Online softmax: s becomes p = exp2(s - m_new); acc and l are rescaled.
#pragma unroll
    for (int g = 0; g < GQA; ++g) {
      float mt = s[g][0];
#pragma unroll
      for (int i = 1; i < 8; ++i) mt = fmaxf(mt, s[g][i]);
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
      const float mn = fmaxf(m[g], mt);
      float alpha = 1.f;
      if (mn == neg_inf()) {
#pragma unroll
        for (int i = 0; i < 8; ++i) s[g][i] = 0.f;
      } else {
        alpha = fast_exp2(m[g] - mn);
#pragma unroll
        for (int i = 0; i < 8; ++i) s[g][i] = fast_exp2(s[g][i] - mn);
      }
      float ps = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ps += s[g][i];
      l[g] = l[g] * alpha + ps;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] *= alpha;
      m[g] = mn;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float vf[8];
      unpack8(vr[i], vf);
#pragma unroll
      for (int g = 0; g < GQA; ++g)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(s[g][i], vf[e], acc[g][e]);
    }
  }
  // Combine the two token halves (tp = 0 / 1); m is warp-uniform.
#pragma unroll
  for (int g = 0; g < GQA; ++g) {
    l[g] += __shfl_xor_sync(0xffffffffu, l[g], 16);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] += __shfl_xor_sync(0xffffffffu, acc[g][e], 16);
  }
  const bool whole = (tile_lo == 0 && tile_hi == nb);
  if (whole) {
    if (tp == 0) {
#pragma unroll
      for (int g = 0; g < GQA; ++g) {
        const float inv = 1.f / l[g];
        uint4 out;
        out.x = f2_to_h2(acc[g][0] * inv, acc[g][1] * inv);
        out.y = f2_to_h2(acc[g][2] * inv, acc[g][3] * inv);
        out.z = f2_to_h2(acc[g][4] * inv, acc[g][5] * inv);
        out.w = f2_to_h2(acc[g][6] * inv, acc[g][7] * inv);
        *reinterpret_cast<uint4*>(p.o + ((long long)row * p.num_q_heads + kv_head * GQA + g) * kHeadDim + dc * 8) = out;
      }
    }
    return;
  }
  const long long w0 = worker_of(unit_start, total, workers);
  const long long w1 = worker_of(unit_start + nb - 1, total, workers);
  const long long slot = piece_slot(w, w0);
  if (tp == 0) {
#pragma unroll
    for (int g = 0; g < GQA; ++g) {
      const float inv = 1.f / l[g];
      float4* dst = reinterpret_cast<float4*>(p.part_o + (slot * p.nq + g) * kHeadDim + dc * 8);
      __stcg(dst, make_float4(acc[g][0] * inv, acc[g][1] * inv, acc[g][2] * inv, acc[g][3] * inv));
      __stcg(dst + 1, make_float4(acc[g][4] * inv, acc[g][5] * inv, acc[g][6] * inv, acc[g][7] * inv));
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < GQA; ++g)
      __stcg(p.part_lse + slot * p.nq + g, l[g] > 0.f ? m[g] + __log2f(l[g]) : neg_inf());
  }
  __threadfence();
  __syncwarp();
  int last = 0;
  if (lane == 0) last = (atomicAdd(p.counters + unit, 1) == (int)(w1 - w0));
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) {
    __threadfence();
    merge_unit_warp(p, row, 1, kv_head, GQA, w0, w1);
    if (lane == 0) p.counters[unit] = 0;
  }
}

template <int GQA>
__global__ void __launch_bounds__(kDecodeThreads, (GQA <= 2 ? 4 : 2)) decode_attn_kernel(AttnParams p) {
  extern __shared__ int smem[];
  __shared__ int scratch[32];
  pdl_trigger();
  pdl_wait();  // inputs may come from the previous launch in the stream
  PlanSmem ps{smem, smem + (p.num_rows + 1), smem + 2 * (p.num_rows + 1), nullptr};
  build_plan(ps, scratch, p.seq_ids, p.seq_lens, p.num_rows, 1);
  const int ng = ps.misc[0];
  const int hk = p.num_kv_heads;
  const long long total = (long long)hk * ps.gprefix[ng];
  const long long launched = (long long)gridDim.x * kDecodeWarps;
  const long long w = (long long)blockIdx.x * kDecodeWarps + (threadIdx.x >> 5);
  write_nan_rows(p, ps, ng, w, launched);
  if (total == 0) return;
  // Only min(launched, total) workers take part, so every one owns >= 1 tile
  // and all workers w0..w1 of a split unit report to its counter.
  const long long workers = launched < total ? launched : total;
  if (w >= workers) return;
  long long t = range_begin(w, total, workers);
  const long long t_end = range_begin(w + 1, total, workers);
  if (t >= t_end) return;
  int g = find_group(ps.gprefix, ng, t, hk);
  while (t < t_end) {
    while ((long long)hk * ps.gprefix[g + 1] <= t) ++g;
    const int nb = ps.gprefix[g + 1] - ps.gprefix[g];
    const long long gbase = (long long)hk * ps.gprefix[g];
    const int h = (int)((t - gbase) / nb);
    const int off = (int)(t - gbase - (long long)h * nb);
    const int cnt = (int)min((long long)(nb - off), t_end - t);
    decode_piece<GQA>(p, ps.gfirst[g], h, off, off + cnt, nb, gbase + (long long)h * nb,
                      (long long)g * hk + h, w, workers, total);
    t += cnt;
  }
}

// ------------------------------------------------------------------ host side
static int decode_ctas_per_sm(int gqa, int num_rows) {
  int n = 0;
  const size_t smem = plan_smem_bytes(kMaxRows);
  (void)num_rows;
  cudaError_t e = cudaSuccess;
  switch (gqa) {
    case 1: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_attn_kernel<1>, kDecodeThreads, smem); break;
    case 2: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_attn_kernel<2>, kDecodeThreads, smem); break;
    case 4: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_attn_kernel<4>, kDecodeThreads, smem); break;
    case 8: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_attn_kernel<8>, kDecodeThreads, smem); break;
    default: return 0;
  }
  if (e != cudaSuccess || n < 1) return 1;
  return n;
}

long long decode_workers(int device, int gqa) {
  static long long cache[64][9] = {};
  if (device < 0 || device >= 64 || gqa < 1 || gqa > 8) return 0;
  if (cache[device][gqa] == 0) {
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != device) cudaSetDevice(device);
    cache[device][gqa] = (long long)num_sms(device) * decode_ctas_per_sm(gqa, kMaxRows) * kDecodeWarps;
    if (prev != device) cudaSetDevice(prev);
  }
  return cache[device][gqa];
}

int launch_decode(const AttnParams& p, long long workers, cudaStream_t stream) {
  const int grid = (int)(workers / kDecodeWarps);
  const size_t smem = plan_smem_bytes(p.num_rows);
  const int gqa = p.num_q_heads / p.num_kv_heads;
  // Programmatic stream serialisation: the next launch is scheduled as this
  // one starts, and each waits for its predecessor before reading any input,
  // so the launch gap and the previous launch's tail overlap.
  const dim3 g((unsigned)grid), b(kDecodeThreads);
  switch (gqa) {
    case 1: NEB_CUDA(launch_pdl(decode_attn_kernel<1>, g, b, smem, stream, p)); break;
    case 2: NEB_CUDA(launch_pdl(decode_attn_kernel<2>, g, b, smem, stream, p)); break;
    case 4: NEB_CUDA(launch_pdl(decode_attn_kernel<4>, g, b, smem, stream, p)); break;
    case 8: NEB_CUDA(launch_pdl(decode_attn_kernel<8>, g, b, smem, stream, p)); break;
    default: return set_error(NEB_ERR_UNSUPPORTED, "decode attention supports q/kv head ratios 1, 2, 4, 8 (got %d)", gqa);
  }
  return NEB_OK;
}

}  // namespace neb
