// Greedy speculative acceptance on the device.
//
// Replaces the verify-side tail of the reference: `torch.argmax(logits, dim=1)`
// (swiftLLM/swiftllm/worker/layers/post_layer.py:72), the `.tolist()` of the
// posterior tokens (swiftLLM/swiftllm/worker/model.py:465) and the host loop
// of compute_greedy_acceptance (swiftLLM/swiftllm/speculative.py:122-156), so a
// verify forward needs no host synchronisation to know what it accepted.
//
// Phase 1 (every CTA): the arg-max of one chunk of one row's logits.  A CTA
// reads its chunk with 16-byte loads, reduces (value, index) pairs to one
// 64-bit key and folds it into the row's key with one atomicMax.  The key's
// high half orders fp16 values (NaN above everything, -0 as +0, as
// torch.argmax treats them), its low half is ~index, so equal values resolve
// to the lowest index, torch.argmax's choice.
// Phase 2 (the CTA that arrives last): one thread per request compares the
// arg-maxes of its k + 1 rows with its k draft tokens and writes the tokens to
// append (accepted drafts, then the first posterior that differs or the bonus
// token), cut at remaining_output_len and after the first stop token.  It then
// zeroes the row keys and the arrival count, so the workspace is ready for the
// next call.
#include <cuda_fp16.h>

#include "neb_common.cuh"

namespace neb {

constexpr int kAcceptThreads = 256;
constexpr int kChunkHalfs = 16384;  // logits per CTA (32 KB)

struct AcceptParams {
  const __half* logits;
  long long row_stride;  // in halfs
  int vocab, num_rows, num_requests, num_stop, max_out;
  const int32_t* row_start;     // [num_requests + 1]
  const int32_t* draft_tokens;  // [num_rows - num_requests]
  const int32_t* remaining;     // [num_requests] (-1: no limit) or null
  const int32_t* stop_tokens;   // [num_stop]
  int32_t* argmax_out;          // [num_rows] or null
  int32_t* out_tokens;          // [num_requests][max_out]
  int32_t* out_count;           // [num_requests]
  int32_t* out_accepted;        // [num_requests]
  unsigned long long* keys;     // [num_rows], zero between calls
  unsigned int* arrived;        // zero between calls
  unsigned int* error_bits;
  int chunks_per_row;
};

// fp16 bits -> an unsigned order of the values (NaN highest, -0 == +0).
__device__ __forceinline__ unsigned int order_half(unsigned short h) {
  if ((h & 0x7c00u) == 0x7c00u && (h & 0x03ffu)) return 0xffffu;  // NaN
  if (h == 0x8000u) h = 0;                                          // -0
  return (h & 0x8000u) ? (~h & 0xffffu) : (h | 0x8000u);
}

__device__ __forceinline__ unsigned long long make_key(unsigned int ord, int idx) {
  return ((unsigned long long)ord << 32) | (unsigned int)~(unsigned int)idx;
}

__device__ __forceinline__ unsigned long long warp_max_key(unsigned long long k) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long n = __shfl_xor_sync(0xffffffffu, k, o);
    k = n > k ? n : k;
  }
  return k;
}

constexpr int kStageRows = 2048;  // rows whose arg-maxes and drafts phase 2 stages in shared memory

// Phase 2.  `post` holds every row's arg-max (staged in shared memory when it
// fits; null: read the row keys) and `drafts` the draft tokens.
__device__ void accept_requests(const AcceptParams& p, const int32_t* post, const int32_t* drafts) {
  for (int r = threadIdx.x; r < p.num_requests; r += blockDim.x) {
    const int rs = p.row_start[r], re = p.row_start[r + 1];
    const int k = re - rs - 1;
    int32_t* out = p.out_tokens + (long long)r * p.max_out;
    if (k < 0 || k + 1 > p.max_out || rs < 0 || re > p.num_rows) {
      atomicOr(p.error_bits, kErrInvalidRows);
      for (int j = 0; j < p.max_out; ++j) out[j] = -1;
      p.out_count[r] = 0;
      p.out_accepted[r] = 0;
      continue;
    }
    const int32_t* draft = drafts + (rs - r);
    auto posterior = [&](int j) {
      return post ? post[rs + j] : (int)~(unsigned int)(__ldcg(p.keys + rs + j) & 0xffffffffull);
    };
    int n = 0;
    while (n < k && posterior(n) == draft[n]) ++n;
    int len = n + 1;
    const int lim = p.remaining ? p.remaining[r] : -1;
    if (lim >= 0 && lim < len) len = lim;
    if (lim < -1) atomicOr(p.error_bits, kErrInvalidRows);
    for (int j = 0; j < len; ++j) {
      const int tok = j < n ? draft[j] : posterior(n);
      bool stop = false;
      for (int s = 0; s < p.num_stop; ++s) stop |= p.stop_tokens[s] == tok;
      out[j] = tok;
      if (stop) {
        len = j + 1;
        break;
      }
    }
    for (int j = len; j < p.max_out; ++j) out[j] = -1;
    p.out_count[r] = len;
    p.out_accepted[r] = n < len ? n : len;
  }
}

__global__ void __launch_bounds__(kAcceptThreads) greedy_accept_kernel(const AcceptParams p) {
  __shared__ unsigned long long red[kAcceptThreads / 32];
  __shared__ bool last;
  const int row = blockIdx.x / p.chunks_per_row;
  const int chunk = blockIdx.x - row * p.chunks_per_row;
  const int lo = chunk * kChunkHalfs;
  const int hi = min(p.vocab, lo + kChunkHalfs);
  const __half* x = p.logits + (long long)row * p.row_stride;
  unsigned long long best = 0;
  // 8 halfs per 16-byte load when the row is 16-byte aligned; else halfs one by one.
  const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) && (lo % 8 == 0);
  if (vec) {
    const int vhi = lo + ((hi - lo) & ~7);
    // The thread's kWords 16-byte words are all in flight before any is used;
    // words past the chunk read as -inf.  Its maximum comes from packed fp16
    // max (NaN propagating), then the first of its logits equal to it (or the
    // first NaN) gives the index: about one instruction per two logits.
    constexpr int kWords = kChunkHalfs / (8 * kAcceptThreads), kStep = 8 * kAcceptThreads;
    static_assert(kWords * 8 * kAcceptThreads == kChunkHalfs, "whole words per thread");
    const int i0 = lo + 8 * threadIdx.x;
    uint4 v[kWords];
#pragma unroll
    for (int u = 0; u < kWords; ++u)
      v[u] = i0 + u * kStep < vhi ? __ldcs(reinterpret_cast<const uint4*>(x + i0 + u * kStep))
                                  : make_uint4(0xfc00fc00u, 0xfc00fc00u, 0xfc00fc00u, 0xfc00fc00u);
    if (i0 < vhi) {
      __half2 m2 = __halves2half2(__ushort_as_half(0xfc00u), __ushort_as_half(0xfc00u));
#pragma unroll
      for (int u = 0; u < kWords; ++u) {
        const uint4 w = v[u];
        m2 = __hmax2_nan(m2, *reinterpret_cast<const __half2*>(&w.x));
        m2 = __hmax2_nan(m2, *reinterpret_cast<const __half2*>(&w.y));
        m2 = __hmax2_nan(m2, *reinterpret_cast<const __half2*>(&w.z));
        m2 = __hmax2_nan(m2, *reinterpret_cast<const __half2*>(&w.w));
      }
      const __half mx = __hmax_nan(__low2half(m2), __high2half(m2));
      const bool is_nan = __hisnan(mx);
      const __half2 mx2 = __half2half2(mx);
      int idx = i0;
      bool found = false;
#pragma unroll
      for (int u = 0; u < kWords; ++u) {
        const unsigned int w4[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const __half2 h = *reinterpret_cast<const __half2*>(&w4[q]);
          // NaN halves are the ones not equal to themselves.
          const unsigned int hit = is_nan ? __heq2_mask(h, h) ^ 0xffffffffu : __heq2_mask(h, mx2);
          if (!found && hit) {
            found = true;
            idx = i0 + u * kStep + 2 * q + ((hit & 0xffffu) ? 0 : 1);
          }
        }
      }
      best = make_key(order_half(__half_as_ushort(mx)), idx);
    }
    for (int j = vhi + threadIdx.x; j < hi; j += kAcceptThreads) {
      const unsigned long long key = make_key(order_half(__half_as_ushort(x[j])), j);
      best = key > best ? key : best;
    }
  } else {
    for (int i = lo + threadIdx.x; i < hi; i += kAcceptThreads) {
      const unsigned long long key = make_key(order_half(__half_as_ushort(x[i])), i);
      best = key > best ? key : best;
    }
  }
  best = warp_max_key(best);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    unsigned long long b = threadIdx.x < kAcceptThreads / 32 ? red[threadIdx.x] : 0;
    b = warp_max_key(b);
    if (threadIdx.x == 0) {
      atomicMax(p.keys + row, b);
      __threadfence();
      last = atomicAdd(p.arrived, 1u) == gridDim.x - 1;
    }
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // Every row's arg-max (and the drafts) in one round of loads, then the
  // per-request loops read shared memory.
  __shared__ int32_t s_post[kStageRows], s_draft[kStageRows];
  const bool staged = p.num_rows <= kStageRows;
  for (int r = threadIdx.x; r < p.num_rows; r += kAcceptThreads) {
    const int a = (int)~(unsigned int)(__ldcg(p.keys + r) & 0xffffffffull);
    if (p.argmax_out) p.argmax_out[r] = a;
    if (staged) {
      s_post[r] = a;
      if (r < p.num_rows - p.num_requests) s_draft[r] = p.draft_tokens[r];
    }
  }
  __syncthreads();
  if (staged) {
    accept_requests(p, s_post, s_draft);
  } else {
    accept_requests(p, nullptr, p.draft_tokens);
  }
  __syncthreads();
  for (int r = threadIdx.x; r < p.num_rows; r += kAcceptThreads) p.keys[r] = 0;
  if (threadIdx.x == 0) *p.arrived = 0;
}

}  // namespace neb

using namespace neb;

extern "C" size_t neb_greedy_accept_workspace_bytes(int32_t num_rows) {
  return num_rows < 0 ? 0 : 256 + align_up((size_t)num_rows * sizeof(unsigned long long), 256);
}

extern "C" int neb_greedy_accept(const void* logits, int64_t row_stride, int32_t vocab, int32_t num_rows,
                                 const int32_t* row_start, int32_t num_requests, const int32_t* draft_tokens,
                                 const int32_t* remaining, const int32_t* stop_tokens, int32_t num_stop,
                                 int32_t max_out, int32_t* argmax_out, int32_t* out_tokens, int32_t* out_count,
                                 int32_t* out_accepted, void* workspace, size_t workspace_bytes, void* stream) {
  NEB_REQUIRE(num_rows >= 0 && num_requests >= 0 && vocab > 0 && num_stop >= 0 && max_out >= 1, NEB_ERR_INVALID,
              "invalid sizes");
  NEB_REQUIRE(row_stride >= vocab, NEB_ERR_INVALID, "row stride %lld is shorter than the vocabulary %d",
              (long long)row_stride, vocab);
  NEB_REQUIRE(num_requests <= num_rows, NEB_ERR_INVALID, "every request needs at least one row");
  if (num_rows == 0) return NEB_OK;
  NEB_REQUIRE(logits && row_start && out_tokens && out_count && out_accepted && workspace, NEB_ERR_INVALID,
              "null argument");
  NEB_REQUIRE(num_rows == num_requests || draft_tokens, NEB_ERR_INVALID, "draft tokens are null");
  NEB_REQUIRE(num_stop == 0 || stop_tokens, NEB_ERR_INVALID, "stop tokens are null");
  NEB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0, NEB_ERR_WORKSPACE,
              "workspace must be 256-byte aligned");
  NEB_REQUIRE(workspace_bytes >= neb_greedy_accept_workspace_bytes(num_rows), NEB_ERR_WORKSPACE,
              "workspace of %zu bytes is smaller than the %zu required", workspace_bytes,
              neb_greedy_accept_workspace_bytes(num_rows));
  AcceptParams p;
  p.logits = static_cast<const __half*>(logits);
  p.row_stride = row_stride;
  p.vocab = vocab;
  p.num_rows = num_rows;
  p.num_requests = num_requests;
  p.num_stop = num_stop;
  p.max_out = max_out;
  p.row_start = row_start;
  p.draft_tokens = draft_tokens;
  p.remaining = remaining;
  p.stop_tokens = stop_tokens;
  p.argmax_out = argmax_out;
  p.out_tokens = out_tokens;
  p.out_count = out_count;
  p.out_accepted = out_accepted;
  char* base = static_cast<char*>(workspace);
  p.error_bits = reinterpret_cast<unsigned int*>(base);
  p.arrived = reinterpret_cast<unsigned int*>(base + 4);
  p.keys = reinterpret_cast<unsigned long long*>(base + 256);
  p.chunks_per_row = (vocab + kChunkHalfs - 1) / kChunkHalfs;
  const long long blocks = (long long)num_rows * p.chunks_per_row;
  NEB_REQUIRE(blocks < (1ll << 31), NEB_ERR_UNSUPPORTED, "too many logits");
  greedy_accept_kernel<<<(unsigned)blocks, kAcceptThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  NEB_CUDA(cudaGetLastError());
  return NEB_OK;
}
