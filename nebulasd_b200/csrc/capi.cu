// C ABI: argument validation, workspace sizing and dispatch of the attention kernels.
#include <cstdarg>
#include <cstring>

#include "attn_common.cuh"

namespace neb {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  // The failure is reported through the return code; clear the runtime's
  // record of it (non-sticky errors only), so that a later launch check on
  // this thread does not report it again.
  (void)cudaGetLastError();
  return set_error(NEB_ERR_CUDA, "%s failed: %s (%d)", what, cudaGetErrorString(e), (int)e);
}

int num_sms(int device) {
  static int cache[64] = {};
  if (device < 0 || device >= 64) return 0;
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    cache[device] = n;
  }
  return cache[device];
}

long long decode_workers(int device, int gqa);
int launch_decode(const AttnParams& p, long long workers, cudaStream_t stream);
long long verify_workers(int device);
int verify_group_rows(int gqa);
int launch_verify(const AttnParams& p, long long workers, cudaStream_t stream);
int verify_max_rows();
namespace vlong {
long long verify_workers(int device);
int verify_group_rows(int gqa);
int launch_verify(const AttnParams& p, long long workers, cudaStream_t stream);
int verify_max_rows();
}  // namespace vlong

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// Validates the common attention arguments and fills everything but the workspace.
static int attention_params(AttnParams& p, const void* q, const void* k_cache, const void* v_cache,
                            const int32_t* block_table, int32_t block_table_rows,
                            int32_t max_blocks_per_seq, const int32_t* seq_lens,
                            const int32_t* seq_ids, int32_t num_rows, int32_t num_q_heads,
                            int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                            int64_t num_blocks, int32_t num_layers, int32_t cur_layer,
                            float softmax_scale, void* o) {
  NEB_REQUIRE(head_dim == kHeadDim, NEB_ERR_UNSUPPORTED, "head_dim must be 128 (got %d)", head_dim);
  NEB_REQUIRE(block_size == kBlockTokens, NEB_ERR_UNSUPPORTED, "block_size must be 16 (got %d)", block_size);
  NEB_REQUIRE(num_rows >= 0 && num_rows <= kMaxRows, NEB_ERR_UNSUPPORTED,
              "num_rows must be in [0, %d] (got %d)", kMaxRows, num_rows);
  NEB_REQUIRE(num_kv_heads > 0 && num_kv_heads <= kMaxKvHeads, NEB_ERR_UNSUPPORTED,
              "num_kv_heads must be in [1, %d] (got %d)", kMaxKvHeads, num_kv_heads);
  NEB_REQUIRE(num_kv_heads > 0 && num_q_heads > 0 && num_q_heads % num_kv_heads == 0,
              NEB_ERR_INVALID, "num_q_heads (%d) must be a positive multiple of num_kv_heads (%d)",
              num_q_heads, num_kv_heads);
  NEB_REQUIRE(num_layers > 0 && cur_layer >= 0 && cur_layer < num_layers, NEB_ERR_INVALID,
              "cur_layer %d outside [0, %d)", cur_layer, num_layers);
  NEB_REQUIRE(num_blocks > 0 && block_table_rows > 0 && max_blocks_per_seq > 0, NEB_ERR_INVALID,
              "num_blocks, block_table_rows and max_blocks_per_seq must be positive");
  NEB_REQUIRE(q && k_cache && v_cache && block_table && seq_lens && seq_ids && o, NEB_ERR_INVALID,
              "null tensor pointer");
  NEB_REQUIRE(aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && aligned16(o),
              NEB_ERR_INVALID, "q, caches and o must be 16-byte aligned");
  NEB_REQUIRE(softmax_scale > 0.f, NEB_ERR_INVALID, "softmax_scale must be positive");
  std::memset(&p, 0, sizeof(p));
  p.q = static_cast<const __half*>(q);
  p.k_cache = static_cast<const __half*>(k_cache);
  p.v_cache = static_cast<const __half*>(v_cache);
  p.block_table = block_table;
  p.bt_rows = block_table_rows;
  p.mbs = max_blocks_per_seq;
  p.seq_lens = seq_lens;
  p.seq_ids = seq_ids;
  p.num_rows = num_rows;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  p.num_blocks = num_blocks;
  p.num_layers = num_layers;
  p.cur_layer = cur_layer;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.o = static_cast<__half*>(o);
  return NEB_OK;
}

static int bind_workspace(AttnParams& p, void* workspace, size_t workspace_bytes, long long workers,
                          int nq) {
  const WorkspaceLayout L = workspace_layout(workers, p.num_rows, p.num_kv_heads, nq);
  NEB_REQUIRE(workspace != nullptr, NEB_ERR_WORKSPACE, "workspace is null");
  NEB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0, NEB_ERR_WORKSPACE,
              "workspace must be 256-byte aligned");
  NEB_REQUIRE(workspace_bytes >= L.total, NEB_ERR_WORKSPACE,
              "workspace of %zu bytes is smaller than the %zu required", workspace_bytes, L.total);
  char* base = static_cast<char*>(workspace);
  p.hdr = reinterpret_cast<WorkspaceHeader*>(base);
  p.counters = reinterpret_cast<int32_t*>(base + L.counters);
  p.part_lse = reinterpret_cast<float*>(base + L.part_lse);
  p.part_o = reinterpret_cast<float*>(base + L.part_o);
  p.plan_cache = reinterpret_cast<int32_t*>(base + L.plan_cache);
  p.nq = nq;
  return NEB_OK;
}

static int attention_workers(int kernel, int device, int gqa, long long* workers, int* nq,
                             int* group_rows) {
  if (kernel == NEB_ATTN_DECODE) {
    NEB_REQUIRE(gqa == 1 || gqa == 2 || gqa == 4 || gqa == 8, NEB_ERR_UNSUPPORTED,
                "decode attention supports q/kv head ratios 1, 2, 4, 8 (got %d)", gqa);
    *workers = decode_workers(device, gqa);
    *group_rows = 1;
  } else if (kernel == NEB_ATTN_VERIFY) {
    *group_rows = verify_group_rows(gqa);
    NEB_REQUIRE(*group_rows > 0, NEB_ERR_UNSUPPORTED,
                "verify attention supports q/kv head ratios 1..16 (got %d)", gqa);
    *workers = verify_workers(device);
  } else if (kernel == NEB_ATTN_VERIFY_LONG) {
    *group_rows = vlong::verify_group_rows(gqa);
    NEB_REQUIRE(*group_rows > 0, NEB_ERR_UNSUPPORTED,
                "long-context verify attention supports q/kv head ratios 1..64 (got %d)", gqa);
    *workers = vlong::verify_workers(device);
  } else {
    return set_error(NEB_ERR_INVALID, "unknown attention kernel %d", kernel);
  }
  NEB_REQUIRE(*workers > 0, NEB_ERR_CUDA, "could not size the grid for device %d", device);
  *nq = gqa * *group_rows;
  return NEB_OK;
}

}  // namespace neb

using namespace neb;

extern "C" {

int neb_version(void) { return 100; }

const char* neb_last_error(void) { return g_last_error; }

int neb_attention_max_rows(int kernel) {
  if (kernel == NEB_ATTN_VERIFY) return verify_max_rows();
  if (kernel == NEB_ATTN_VERIFY_LONG) return vlong::verify_max_rows();
  return kernel == NEB_ATTN_DECODE ? kMaxRows : 0;
}

size_t neb_attention_workspace_bytes(int kernel, int device, int num_rows, int num_q_heads,
                                     int num_kv_heads) {
  if (num_kv_heads <= 0 || num_kv_heads > kMaxKvHeads || num_q_heads <= 0 || num_q_heads % num_kv_heads ||
      num_rows < 0)
    return 0;
  long long workers = 0;
  int nq = 0, group_rows = 0;
  if (attention_workers(kernel, device, num_q_heads / num_kv_heads, &workers, &nq, &group_rows) != NEB_OK)
    return 0;
  return workspace_layout(workers, num_rows > 0 ? num_rows : 1, num_kv_heads, nq).total;
}

static int paged_attention_impl(int kernel, const void* q, const void* k_cache, const void* v_cache,
                                const int32_t* block_table, int32_t block_table_rows,
                                int32_t max_blocks_per_seq, const int32_t* seq_lens,
                                const int32_t* seq_ids, int32_t num_rows, int32_t num_q_heads,
                                int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                int64_t num_blocks, int32_t num_layers, int32_t cur_layer,
                                float softmax_scale, void* o, void* workspace,
                                size_t workspace_bytes, void* stream) {
  AttnParams p;
  int rc = attention_params(p, q, k_cache, v_cache, block_table, block_table_rows, max_blocks_per_seq,
                            seq_lens, seq_ids, num_rows, num_q_heads, num_kv_heads, head_dim,
                            block_size, num_blocks, num_layers, cur_layer, softmax_scale, o);
  if (rc != NEB_OK) return rc;
  if (num_rows == 0) return NEB_OK;
  int device = 0;
  NEB_CUDA(cudaGetDevice(&device));
  long long workers = 0;
  int nq = 0, group_rows = 0;
  rc = attention_workers(kernel, device, num_q_heads / num_kv_heads, &workers, &nq, &group_rows);
  if (rc != NEB_OK) return rc;
  rc = bind_workspace(p, workspace, workspace_bytes, workers, nq);
  if (rc != NEB_OK) return rc;
  p.max_group_rows = group_rows;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (kernel == NEB_ATTN_DECODE) return launch_decode(p, workers, s);
  return kernel == NEB_ATTN_VERIFY ? launch_verify(p, workers, s) : vlong::launch_verify(p, workers, s);
}

int neb_paged_attention_decode(const void* q, const void* k_cache, const void* v_cache,
                               const int32_t* block_table, int32_t block_table_rows,
                               int32_t max_blocks_per_seq, const int32_t* seq_lens,
                               const int32_t* seq_ids, int32_t num_rows, int32_t num_q_heads,
                               int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                               int64_t num_blocks, int32_t num_layers, int32_t cur_layer,
                               float softmax_scale, void* o, void* workspace,
                               size_t workspace_bytes, void* stream) {
  return paged_attention_impl(NEB_ATTN_DECODE, q, k_cache, v_cache, block_table, block_table_rows,
                              max_blocks_per_seq, seq_lens, seq_ids, num_rows, num_q_heads,
                              num_kv_heads, head_dim, block_size, num_blocks, num_layers, cur_layer,
                              softmax_scale, o, workspace, workspace_bytes, stream);
}

int neb_paged_attention_verify(const void* q, const void* k_cache, const void* v_cache,
                               const int32_t* block_table, int32_t block_table_rows,
                               int32_t max_blocks_per_seq, const int32_t* seq_lens,
                               const int32_t* seq_ids, int32_t num_rows, int32_t num_q_heads,
                               int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                               int64_t num_blocks, int32_t num_layers, int32_t cur_layer,
                               float softmax_scale, void* o, void* workspace,
                               size_t workspace_bytes, void* stream) {
  return paged_attention_impl(NEB_ATTN_VERIFY, q, k_cache, v_cache, block_table, block_table_rows,
                              max_blocks_per_seq, seq_lens, seq_ids, num_rows, num_q_heads,
                              num_kv_heads, head_dim, block_size, num_blocks, num_layers, cur_layer,
                              softmax_scale, o, workspace, workspace_bytes, stream);
}

int neb_paged_attention_verify_long(const void* q, const void* k_cache, const void* v_cache,
                                    const int32_t* block_table, int32_t block_table_rows,
                                    int32_t max_blocks_per_seq, const int32_t* seq_lens,
                                    const int32_t* seq_ids, int32_t num_rows, int32_t num_q_heads,
                                    int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                    int64_t num_blocks, int32_t num_layers, int32_t cur_layer,
                                    float softmax_scale, void* o, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  return paged_attention_impl(NEB_ATTN_VERIFY_LONG, q, k_cache, v_cache, block_table, block_table_rows,
                              max_blocks_per_seq, seq_lens, seq_ids, num_rows, num_q_heads,
                              num_kv_heads, head_dim, block_size, num_blocks, num_layers, cur_layer,
                              softmax_scale, o, workspace, workspace_bytes, stream);
}

}  // extern "C"

namespace neb {

// Reads and clears the error bits of a workspace (or of the static scratch)
// whose calls are ordered on `s`.  A call that gave up on a bounded wait
// (kErrTimeout) stops without counting its split pieces in, so the arrival
// counters it shared with other CTAs may be left above zero; they are cleared
// here, before any later call can merge against them.
static int read_and_clear_status(void* base, uint32_t* error_bits, cudaStream_t s) {
  WorkspaceHeader h;
  NEB_CUDA(cudaMemcpyAsync(&h, base, sizeof(h), cudaMemcpyDeviceToHost, s));
  NEB_CUDA(cudaStreamSynchronize(s));
  *error_bits = h.error_bits;
  if (h.error_bits) {
    NEB_CUDA(cudaMemsetAsync(base, 0, sizeof(uint32_t), s));
    if (h.error_bits & kErrTimeout) {
      const WorkspaceLayout L = workspace_layout(1, 1, 1, 1);
      NEB_CUDA(cudaMemsetAsync(static_cast<char*>(base) + L.counters, 0, L.plan_cache - L.counters, s));
    }
    NEB_CUDA(cudaStreamSynchronize(s));
  }
  return NEB_OK;
}

}  // namespace neb

extern "C" int neb_workspace_status(void* workspace, uint32_t* error_bits, void* stream) {
  NEB_REQUIRE(workspace && error_bits, NEB_ERR_INVALID, "null argument");
  return read_and_clear_status(workspace, error_bits, static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------- allocation-free decode attention
// For callers that cannot allocate device memory: the split-K scratch of the
// decode kernel lives in one statically sized __device__ array of this
// library instead of a caller-provided workspace.  See the declaration of
// neb_paged_attention_decode_noalloc in include/nebula_b200.h for the contract.
#include <mutex>

namespace neb {

// Holds the header, the arrival counters and the partials of one decode call.
// The call uses as many decode workers as fit (at most the workspace entry's
// count), so every q/kv head ratio the decode kernel supports fits.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mutex;
static void* g_noalloc_address[64] = {};

// Device address of the static scratch on `device`, which must be current.
// In host code `g_noalloc_scratch` names a host-side stand-in, not device
// memory, so the address is looked up once per device and kept (the library
// must not outlive a reset of that device's context).  The first lookup also
// clears the header and the counters on `s`.
static int noalloc_scratch_address(int device, cudaStream_t s, void** address) {
  NEB_REQUIRE(device >= 0 && device < 64, NEB_ERR_UNSUPPORTED, "device index %d out of range", device);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_address[device] == nullptr) {
    void* ptr = nullptr;
    NEB_CUDA(cudaGetSymbolAddress(&ptr, g_noalloc_scratch));
    const WorkspaceLayout L = workspace_layout(1, 1, 1, 1);
    NEB_CUDA(cudaMemsetAsync(ptr, 0, L.part_lse, s));
    g_noalloc_address[device] = ptr;
  }
  *address = g_noalloc_address[device];
  return NEB_OK;
}

// Decode workers whose partials fit the static scratch next to its header and
// counters (a multiple of the kernel's warps per CTA).
static long long noalloc_workers(long long workers, int nq) {
  const WorkspaceLayout L0 = workspace_layout(0, 1, 1, nq);
  const size_t per_worker = (size_t)2 * nq * (kHeadDim + 1) * sizeof(float);
  long long fit = (long long)((kNoAllocScratchBytes - L0.total - 512) / per_worker);
  fit -= fit % 4;
  return workers < fit ? workers : fit;
}

}  // namespace neb

extern "C" int neb_paged_attention_decode_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const int32_t* block_table,
    int32_t block_table_rows, int32_t max_blocks_per_seq, const int32_t* seq_lens, const int32_t* seq_ids,
    int32_t num_rows, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
    int64_t num_blocks, int32_t num_layers, int32_t cur_layer, float softmax_scale, void* o, void* stream) {
  AttnParams p;
  int rc = attention_params(p, q, k_cache, v_cache, block_table, block_table_rows, max_blocks_per_seq,
                            seq_lens, seq_ids, num_rows, num_q_heads, num_kv_heads, head_dim, block_size,
                            num_blocks, num_layers, cur_layer, softmax_scale, o);
  if (rc != NEB_OK) return rc;
  if (num_rows == 0) return NEB_OK;
  int device = 0;
  NEB_CUDA(cudaGetDevice(&device));
  long long workers = 0;
  int nq = 0, group_rows = 0;
  rc = attention_workers(NEB_ATTN_DECODE, device, num_q_heads / num_kv_heads, &workers, &nq, &group_rows);
  if (rc != NEB_OK) return rc;
  workers = noalloc_workers(workers, nq);
  const WorkspaceLayout L = workspace_layout(workers, num_rows, num_kv_heads, nq);
  NEB_REQUIRE(workers >= 4 && L.total <= kNoAllocScratchBytes, NEB_ERR_WORKSPACE,
              "this call needs %zu bytes of scratch; the static scratch holds %zu", L.total,
              kNoAllocScratchBytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  rc = noalloc_scratch_address(device, s, &scratch);
  if (rc != NEB_OK) return rc;
  // The array keeps the previous call's bytes.  The counters this call can
  // touch must start at zero; the partials are written before they are read.
  // The header's error bits are left to accumulate until
  // neb_paged_attention_noalloc_status reads and clears them.
  NEB_CUDA(cudaMemsetAsync(static_cast<char*>(scratch) + L.counters, 0,
                           (size_t)num_rows * num_kv_heads * sizeof(int32_t), s));
  rc = bind_workspace(p, scratch, kNoAllocScratchBytes, workers, nq);
  if (rc != NEB_OK) return rc;
  p.max_group_rows = group_rows;
  return launch_decode(p, workers, s);
}

extern "C" int neb_paged_attention_noalloc_status(uint32_t* error_bits, void* stream) {
  NEB_REQUIRE(error_bits, NEB_ERR_INVALID, "null argument");
  int device = 0;
  NEB_CUDA(cudaGetDevice(&device));
  NEB_REQUIRE(device >= 0 && device < 64, NEB_ERR_UNSUPPORTED, "device index %d out of range", device);
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    scratch = g_noalloc_address[device];
  }
  *error_bits = 0;
  if (scratch == nullptr) return NEB_OK;  // no allocation-free call ran on this device
  return read_and_clear_status(scratch, error_bits, static_cast<cudaStream_t>(stream));
}
