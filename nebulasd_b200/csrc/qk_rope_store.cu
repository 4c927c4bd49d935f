// Qwen3 QK-RMSNorm + RoPE + paged KV-store, fused, plus the three separate ops.
//
// Reference semantics (paths relative to the NebulaSD project root):
//   rmsnorm_inplace   swiftLLM/swiftllm/worker/kernels/rmsnorm.py:5-37
//       y = fp16( x32 * (1 / sqrt(sum(x32^2) / n + eps)) * w32 )
//   rotary            swiftLLM/swiftllm/worker/kernels/rotary_emb.py:7-58
//       fp16 arithmetic on the two 64-halves, q handled per GQA group of its kv head
//   store_kvcache     swiftLLM/swiftllm/worker/kernels/kvcache_mgmt.py:10-122
//       decode row r: pos = seq_lens[r] - 1; prefill token i of seq s: pos = i;
//       cache[block_table[seq_id][pos / 16], layer, :, pos % 16, :] = k/v row (bit copy)
//   call order        swiftLLM/swiftllm/worker/layers/transformer_layer.py:114-143
//
// The fused kernel keeps every rounding step of that sequence: the normalised
// value is rounded to fp16 (the reference stores it in place), RoPE multiplies
// and adds in fp16 with round-to-nearest and no contraction (__hmul_rn /
// __hsub_rn / __hadd_rn, the per-operation rounding of the reference's fp16
// expression), and the rotated k is what lands in the cache, bit for bit.
// One warp handles one (token, head) row of 128 values: lane l holds d = 4l..4l+3
// for l < 16 (first half) and the matching second-half values in lane l+16.
#include "neb_common.cuh"

namespace neb {

struct RopeStoreParams {
  __half* q;              // [T, H, 128]   (in place)
  __half* k;              // [T, Hk, 128]  (in place)
  const __half* v;        // [T, Hk, 128]
  const __half* q_w;      // [128] or null (no QK-norm)
  const __half* k_w;
  float eps;
  const __half* cos;      // [T, 64] or null (no RoPE)
  const __half* sin;
  __half* k_cache;        // or null (no store)
  __half* v_cache;
  const int32_t* block_table;
  int32_t bt_rows, mbs;
  const int32_t* seq_ids;         // [num_prefill_seqs + num_decode_rows]
  const int32_t* decode_lens;     // [num_decode_rows]
  const int32_t* prefill_starts;  // [num_prefill_seqs]
  const int32_t* prefill_lens;    // [num_prefill_seqs]
  int32_t num_prefill_seqs, num_prefill_tokens, num_decode_rows;
  int32_t num_tokens, num_q_heads, num_kv_heads;
  int64_t num_blocks;
  int32_t num_layers, cur_layer;
  uint32_t* error_bits;   // optional
};

__device__ __forceinline__ void flag(const RopeStoreParams& p, uint32_t bits) {
  if (p.error_bits) atomicOr(p.error_bits, bits);
}

// Cache slot (element offset of the (block, layer, head 0, pos % 16) row) of token t, or -1.
__device__ __forceinline__ long long token_slot(const RopeStoreParams& p, int t) {
  int sid, pos;
  if (t >= p.num_prefill_tokens) {
    const int r = t - p.num_prefill_tokens;
    sid = p.seq_ids[p.num_prefill_seqs + r];
    pos = p.decode_lens[r] - 1;
  } else {
    if (p.num_prefill_seqs <= 0) return -1;
    int lo = 0, hi = p.num_prefill_seqs;  // last s with start <= t
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (p.prefill_starts[mid] <= t) lo = mid; else hi = mid;
    }
    pos = t - p.prefill_starts[lo];
    if (pos >= p.prefill_lens[lo]) return -1;  // a gap between prefill sequences
    sid = p.seq_ids[lo];
  }
  if (sid < 0 || sid >= p.bt_rows) { flag(p, kErrSeqId); return -1; }
  if (pos < 0) return -1;
  const int tile = pos >> 4;
  if (tile >= p.mbs) { flag(p, kErrTooManyBlocks); return -1; }
  const long long blk = p.block_table[(long long)sid * p.mbs + tile];
  if (blk < 0 || blk >= p.num_blocks) { flag(p, kErrBlockIndex); return -1; }
  return ((blk * p.num_layers + p.cur_layer) * p.num_kv_heads * 16 + (pos & 15)) * 128LL;
}

__device__ __forceinline__ void load4(const __half* src, float (&x)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(src);
  const float2 a = h2_to_f2(u.x), b = h2_to_f2(u.y);
  x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
}

// Normalise (optional) and rotate (optional) one head row held 4 values per lane.
__device__ __forceinline__ uint2 norm_rope_row(const RopeStoreParams& p, const __half* row,
                                               const __half* w, int t) {
  const int lane = threadIdx.x & 31;
  const int d = (lane & 15) * 4 + (lane >> 4) * 64;
  uint2 bits = *reinterpret_cast<const uint2*>(row + d);
  if (w != nullptr) {
    float x[4];
    load4(row + d, x);
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rstd = 1.0f / sqrtf(ss / 128.0f + p.eps);
    float wf[4];
    load4(w + d, wf);
    bits.x = f2_to_h2(x[0] * rstd * wf[0], x[1] * rstd * wf[1]);
    bits.y = f2_to_h2(x[2] * rstd * wf[2], x[3] * rstd * wf[3]);
  }
  if (p.cos != nullptr) {
    const uint2 other = make_uint2(__shfl_xor_sync(0xffffffffu, bits.x, 16),
                                   __shfl_xor_sync(0xffffffffu, bits.y, 16));
    const int c0 = (lane & 15) * 4;
    const uint2 cu = *reinterpret_cast<const uint2*>(p.cos + (long long)t * 64 + c0);
    const uint2 su = *reinterpret_cast<const uint2*>(p.sin + (long long)t * 64 + c0);
    const __half* xs = reinterpret_cast<const __half*>(&bits);
    const __half* os = reinterpret_cast<const __half*>(&other);
    const __half* cs = reinterpret_cast<const __half*>(&cu);
    const __half* sn = reinterpret_cast<const __half*>(&su);
    __half y[4];
    const bool first = lane < 16;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (first) {  // x0' = x0*cos - x1*sin
        y[e] = __hsub_rn(__hmul_rn(xs[e], cs[e]), __hmul_rn(os[e], sn[e]));
      } else {      // x1' = x0*sin + x1*cos
        y[e] = __hadd_rn(__hmul_rn(os[e], sn[e]), __hmul_rn(xs[e], cs[e]));
      }
    }
    bits = *reinterpret_cast<const uint2*>(y);
  }
  return bits;
}

// Items: per token, H q rows, then Hk k rows, then Hk v rows.
__global__ void __launch_bounds__(256) qk_norm_rope_store_kernel(RopeStoreParams p) {
  pdl_trigger();  // the attention launch that follows may start its set-up
  pdl_wait();     // q, k, v come from the previous launch (the QKV projection)
  const int lane = threadIdx.x & 31;
  const int d = (lane & 15) * 4 + (lane >> 4) * 64;
  const int per_tok = p.num_q_heads + 2 * p.num_kv_heads;
  const long long items = (long long)p.num_tokens * per_tok;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long it = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += warps) {
    const int t = (int)(it / per_tok);
    const int j = (int)(it - (long long)t * per_tok);
    if (j < p.num_q_heads) {
      __half* row = p.q + ((long long)t * p.num_q_heads + j) * 128;
      const uint2 y = norm_rope_row(p, row, p.q_w, t);
      *reinterpret_cast<uint2*>(row + d) = y;
    } else if (j < p.num_q_heads + p.num_kv_heads) {
      const int h = j - p.num_q_heads;
      __half* row = p.k + ((long long)t * p.num_kv_heads + h) * 128;
      const uint2 y = norm_rope_row(p, row, p.k_w, t);
      if (p.k_w != nullptr || p.cos != nullptr) *reinterpret_cast<uint2*>(row + d) = y;
      if (p.k_cache != nullptr) {
        const long long slot = token_slot(p, t);
        if (slot >= 0) *reinterpret_cast<uint2*>(p.k_cache + slot + h * 2048LL + d) = y;
      }
    } else if (p.k_cache != nullptr) {
      const int h = j - p.num_q_heads - p.num_kv_heads;
      const uint2 y = *reinterpret_cast<const uint2*>(p.v + ((long long)t * p.num_kv_heads + h) * 128 + d);
      const long long slot = token_slot(p, t);
      if (slot >= 0) *reinterpret_cast<uint2*>(p.v_cache + slot + h * 2048LL + d) = y;
    }
  }
}

// Generic in-place RMSNorm over rows of `hidden` fp16 values (one CTA per row).
__global__ void __launch_bounds__(256) rmsnorm_kernel(__half* x, const __half* w, int hidden, float eps) {
  __shared__ float red[8];
  __half* row = x + (long long)blockIdx.x * hidden;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float v = __half2float(row[i]);
    ss += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float rstd = 1.0f / sqrtf(red[0] / (float)hidden + eps);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x)
    row[i] = __float2half_rn(__half2float(row[i]) * rstd * __half2float(w[i]));
}

static int launch_rope_store(const RopeStoreParams& p, cudaStream_t stream) {
  const long long items = (long long)p.num_tokens * (p.num_q_heads + 2 * p.num_kv_heads);
  if (items == 0) return NEB_OK;
  const long long blocks = (items + 7) / 8;
  const int grid = (int)(blocks < 65535 ? blocks : 65535);
  NEB_CUDA(launch_pdl(qk_norm_rope_store_kernel, dim3((unsigned)grid), dim3(256), 0, stream, p));
  return NEB_OK;
}

static bool al8(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 7u) == 0; }

}  // namespace neb

using namespace neb;

extern "C" {

int neb_qk_norm_rope_store(void* q, void* k, const void* v, const void* q_norm_w, const void* k_norm_w,
                           float eps, const void* cos, const void* sin, void* k_cache, void* v_cache,
                           const int32_t* block_table, int32_t block_table_rows,
                           int32_t max_blocks_per_seq, const int32_t* seq_ids,
                           const int32_t* decode_seq_lens, int32_t num_decode_rows,
                           const int32_t* prefill_start_locs, const int32_t* prefill_seq_lens,
                           int32_t num_prefill_seqs, int32_t num_prefill_tokens,
                           int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                           int32_t block_size, int64_t num_blocks, int32_t num_layers,
                           int32_t cur_layer, uint32_t* error_bits, void* stream) {
  NEB_REQUIRE(head_dim == 128, NEB_ERR_UNSUPPORTED, "head_dim must be 128 (got %d)", head_dim);
  NEB_REQUIRE(block_size == 16, NEB_ERR_UNSUPPORTED, "block_size must be 16 (got %d)", block_size);
  NEB_REQUIRE(num_q_heads > 0 && num_kv_heads > 0, NEB_ERR_INVALID, "head counts must be positive");
  NEB_REQUIRE(num_decode_rows >= 0 && num_prefill_seqs >= 0 && num_prefill_tokens >= 0,
              NEB_ERR_INVALID, "negative row counts");
  NEB_REQUIRE(q && k, NEB_ERR_INVALID, "q and k are required");
  NEB_REQUIRE(al8(q) && al8(k) && (!v || al8(v)), NEB_ERR_INVALID, "q, k, v must be 8-byte aligned");
  NEB_REQUIRE((q_norm_w == nullptr) == (k_norm_w == nullptr), NEB_ERR_INVALID,
              "q_norm_w and k_norm_w must both be given or both be null");
  NEB_REQUIRE((cos == nullptr) == (sin == nullptr), NEB_ERR_INVALID, "cos and sin go together");
  const bool store = k_cache != nullptr;
  if (store) {
    NEB_REQUIRE(v && v_cache && block_table && seq_ids, NEB_ERR_INVALID, "store needs v, caches, block_table, seq_ids");
    NEB_REQUIRE(num_decode_rows == 0 || decode_seq_lens, NEB_ERR_INVALID, "decode rows need decode_seq_lens");
    NEB_REQUIRE(num_prefill_seqs == 0 || (prefill_start_locs && prefill_seq_lens), NEB_ERR_INVALID,
                "prefill rows need start locations and lengths");
    NEB_REQUIRE(num_prefill_tokens == 0 || num_prefill_seqs > 0, NEB_ERR_INVALID,
                "prefill tokens without prefill sequences");
    NEB_REQUIRE(num_layers > 0 && cur_layer >= 0 && cur_layer < num_layers, NEB_ERR_INVALID,
                "cur_layer %d outside [0, %d)", cur_layer, num_layers);
    NEB_REQUIRE(num_blocks > 0 && block_table_rows > 0 && max_blocks_per_seq > 0, NEB_ERR_INVALID,
                "num_blocks, block_table_rows and max_blocks_per_seq must be positive");
  }
  RopeStoreParams p{};
  p.q = static_cast<__half*>(q);
  p.k = static_cast<__half*>(k);
  p.v = static_cast<const __half*>(v);
  p.q_w = static_cast<const __half*>(q_norm_w);
  p.k_w = static_cast<const __half*>(k_norm_w);
  p.eps = eps;
  p.cos = static_cast<const __half*>(cos);
  p.sin = static_cast<const __half*>(sin);
  p.k_cache = static_cast<__half*>(k_cache);
  p.v_cache = static_cast<__half*>(v_cache);
  p.block_table = block_table;
  p.bt_rows = block_table_rows;
  p.mbs = max_blocks_per_seq;
  p.seq_ids = seq_ids;
  p.decode_lens = decode_seq_lens;
  p.prefill_starts = prefill_start_locs;
  p.prefill_lens = prefill_seq_lens;
  p.num_prefill_seqs = num_prefill_seqs;
  p.num_prefill_tokens = num_prefill_tokens;
  p.num_decode_rows = num_decode_rows;
  p.num_tokens = num_prefill_tokens + num_decode_rows;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  p.num_blocks = num_blocks;
  p.num_layers = num_layers;
  p.cur_layer = cur_layer;
  p.error_bits = error_bits;
  return launch_rope_store(p, static_cast<cudaStream_t>(stream));
}

int neb_store_kvcache(const void* k, const void* v, void* k_cache, void* v_cache,
                      const int32_t* block_table, int32_t block_table_rows, int32_t max_blocks_per_seq,
                      const int32_t* seq_ids, const int32_t* decode_seq_lens, int32_t num_decode_rows,
                      const int32_t* prefill_start_locs, const int32_t* prefill_seq_lens,
                      int32_t num_prefill_seqs, int32_t num_prefill_tokens, int32_t num_kv_heads,
                      int32_t head_dim, int32_t block_size, int64_t num_blocks, int32_t num_layers,
                      int32_t cur_layer, uint32_t* error_bits, void* stream) {
  NEB_REQUIRE(k_cache && v_cache, NEB_ERR_INVALID, "caches are required");
  // Store only: q rows = 0, no norm, no rope.  k is read, never written (no transform).
  RopeStoreParams p{};
  NEB_REQUIRE(head_dim == 128, NEB_ERR_UNSUPPORTED, "head_dim must be 128 (got %d)", head_dim);
  NEB_REQUIRE(block_size == 16, NEB_ERR_UNSUPPORTED, "block_size must be 16 (got %d)", block_size);
  NEB_REQUIRE(k && v && block_table && seq_ids, NEB_ERR_INVALID, "null tensor pointer");
  NEB_REQUIRE(al8(k) && al8(v) && al8(k_cache) && al8(v_cache), NEB_ERR_INVALID, "8-byte alignment required");
  NEB_REQUIRE(num_kv_heads > 0 && num_decode_rows >= 0 && num_prefill_seqs >= 0 && num_prefill_tokens >= 0,
              NEB_ERR_INVALID, "bad counts");
  NEB_REQUIRE(num_decode_rows == 0 || decode_seq_lens, NEB_ERR_INVALID, "decode rows need decode_seq_lens");
  NEB_REQUIRE(num_prefill_seqs == 0 || (prefill_start_locs && prefill_seq_lens), NEB_ERR_INVALID,
              "prefill rows need start locations and lengths");
  NEB_REQUIRE(num_prefill_tokens == 0 || num_prefill_seqs > 0, NEB_ERR_INVALID,
              "prefill tokens without prefill sequences");
  NEB_REQUIRE(num_layers > 0 && cur_layer >= 0 && cur_layer < num_layers, NEB_ERR_INVALID,
              "cur_layer %d outside [0, %d)", cur_layer, num_layers);
  NEB_REQUIRE(num_blocks > 0 && block_table_rows > 0 && max_blocks_per_seq > 0, NEB_ERR_INVALID,
              "num_blocks, block_table_rows and max_blocks_per_seq must be positive");
  p.q = nullptr;
  p.k = const_cast<__half*>(static_cast<const __half*>(k));
  p.v = static_cast<const __half*>(v);
  p.k_cache = static_cast<__half*>(k_cache);
  p.v_cache = static_cast<__half*>(v_cache);
  p.block_table = block_table;
  p.bt_rows = block_table_rows;
  p.mbs = max_blocks_per_seq;
  p.seq_ids = seq_ids;
  p.decode_lens = decode_seq_lens;
  p.prefill_starts = prefill_start_locs;
  p.prefill_lens = prefill_seq_lens;
  p.num_prefill_seqs = num_prefill_seqs;
  p.num_prefill_tokens = num_prefill_tokens;
  p.num_decode_rows = num_decode_rows;
  p.num_tokens = num_prefill_tokens + num_decode_rows;
  p.num_q_heads = 0;
  p.num_kv_heads = num_kv_heads;
  p.num_blocks = num_blocks;
  p.num_layers = num_layers;
  p.cur_layer = cur_layer;
  p.error_bits = error_bits;
  return launch_rope_store(p, static_cast<cudaStream_t>(stream));
}

int neb_rmsnorm_inplace(void* x, const void* weight, int64_t num_rows, int32_t hidden, float eps,
                        void* stream) {
  NEB_REQUIRE(x && weight, NEB_ERR_INVALID, "null tensor pointer");
  NEB_REQUIRE(hidden > 0 && num_rows >= 0 && num_rows < (1LL << 31), NEB_ERR_INVALID, "bad shape");
  if (num_rows == 0) return NEB_OK;
  rmsnorm_kernel<<<(unsigned)num_rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__half*>(x), static_cast<const __half*>(weight), hidden, eps);
  NEB_CUDA(cudaGetLastError());
  return NEB_OK;
}

int neb_rotary_inplace(void* q, void* k, const void* cos, const void* sin, int32_t num_tokens,
                       int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, void* stream) {
  NEB_REQUIRE(head_dim == 128, NEB_ERR_UNSUPPORTED, "head_dim must be 128 (got %d)", head_dim);
  NEB_REQUIRE(q && k && cos && sin, NEB_ERR_INVALID, "null tensor pointer");
  NEB_REQUIRE(al8(q) && al8(k) && al8(cos) && al8(sin), NEB_ERR_INVALID, "8-byte alignment required");
  NEB_REQUIRE(num_tokens >= 0 && num_q_heads > 0 && num_kv_heads > 0, NEB_ERR_INVALID, "bad shape");
  RopeStoreParams p{};
  p.q = static_cast<__half*>(q);
  p.k = static_cast<__half*>(k);
  p.cos = static_cast<const __half*>(cos);
  p.sin = static_cast<const __half*>(sin);
  p.num_tokens = num_tokens;
  p.num_prefill_tokens = num_tokens;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  return launch_rope_store(p, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
