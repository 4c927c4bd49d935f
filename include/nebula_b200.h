/*
 * nebula_b200.h -- C ABI of the B200-native swiftLLM attention hot path.
 *
 * Every entry point takes plain device/host pointers, sizes and a
 * cudaStream_t passed as `void*`, launches asynchronously on that stream and
 * returns an int status (NEB_OK = 0).  neb_last_error() gives the message of
 * the last failure on the calling thread.  Tensors are owned by the caller.
 *
 * Layout contract (fixed by the reference's callers):
 *   q / o        [num_rows, num_q_heads, head_dim]                     fp16
 *   k/v cache    [num_blocks, num_layers, num_kv_heads, block_size, head_dim] fp16
 *   block_table  [block_table_rows, max_blocks_per_seq]                int32
 *   seq_lens / seq_ids  [num_rows]                                     int32
 * head_dim must be 128 and block_size 16 (the Qwen3 / swiftLLM configuration).
 *
 * Reference interfaces replaced (paths relative to the NebulaSD project root):
 *   swiftLLM/swiftllm/worker/kernels/paged_attn.py:152-222      paged_attention
 *   swiftLLM/swiftllm/worker/kernels/kvcache_mgmt.py:81-122     store_kvcache
 *   swiftLLM/swiftllm/worker/kernels/rotary_emb.py:44-58        rotary_embedding_inplace
 *   swiftLLM/swiftllm/worker/kernels/rmsnorm.py:26-37           rmsnorm_inplace
 *   nebulasd/src/nebulasd/kv/cuda_transfer.py:78-108            CudaCopyBackend.launch
 *   swiftLLM/csrc/src/block_swapping.cpp:22-85                  swap_blocks
 */
#ifndef NEBULA_B200_H
#define NEBULA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NEB_OK 0
#define NEB_ERR_INVALID 1      /* bad argument (shape, pointer, size) */
#define NEB_ERR_UNSUPPORTED 2  /* valid but unsupported configuration */
#define NEB_ERR_CUDA 3         /* a CUDA runtime/driver call failed */
#define NEB_ERR_WORKSPACE 4    /* workspace missing or too small */
#define NEB_ERR_DEVICE 5       /* the kernel recorded an error (see neb_workspace_status) */

/* Library version (major*10000 + minor*100 + patch). */
int neb_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* neb_last_error(void);

/* ------------------------------------------------------------------ attention
 * Paged attention over decode rows.  Row r attends q[r] to the first
 * seq_lens[r] tokens of sequence seq_ids[r]; token t of a sequence lives in
 * cache[block_table[seq_id][t / 16], cur_layer, kv_head, t % 16, :].  Adjacent
 * rows with the same seq_id (a verify of depth k lowers to k+1 such rows with
 * lengths L+1..L+k+1) share one read of their KV prefix.  Output o is fp16,
 * accumulated in fp32.  A row with seq_len <= 0 gets NaN, as the reference's
 * 0/0 normalisation does.
 *
 * workspace: device scratch of at least neb_attention_workspace_bytes(...)
 * bytes, zero-filled once before its first use and then reused by calls that
 * are ordered on one stream (the kernels leave its counters at zero).  Calls
 * that may overlap on the GPU need distinct workspaces.
 *
 * Replaces paged_attention, swiftLLM/swiftllm/worker/kernels/paged_attn.py:152-222
 * (phase 1 :9-108, phase 2 :111-149), whose fp32 mid_o / mid_o_logexpsum
 * buffers (:170-180) this workspace stands in for.
 */
#define NEB_ATTN_DECODE 0       /* CUDA-core kernel: 128-bit loads, warp shuffles */
#define NEB_ATTN_VERIFY 1       /* tcgen05 kernel: GQA x rows packed into MMA tiles */
#define NEB_ATTN_VERIFY_LONG 2  /* tcgen05 kernel for long prefixes: KV tokens on the MMA's M */

size_t neb_attention_workspace_bytes(int kernel, int device, int num_rows, int num_q_heads,
                                     int num_kv_heads);

/* Largest num_rows one call of `kernel` accepts (the plan of a call lives in
 * shared memory); larger batches are split by the caller or go to the other
 * kernel.  The reference has no such bound. */
int neb_attention_max_rows(int kernel);

int neb_paged_attention_decode(const void* q, const void* k_cache, const void* v_cache,
                               const int32_t* block_table, int32_t block_table_rows,
                               int32_t max_blocks_per_seq, const int32_t* seq_lens,
                               const int32_t* seq_ids, int32_t num_rows, int32_t num_q_heads,
                               int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                               int64_t num_blocks, int32_t num_layers, int32_t cur_layer,
                               float softmax_scale, void* o, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Target verify attention on tcgen05 tensor cores: the GQA group and up to
 * 64 / gqa adjacent rows of one seq_id (the k+1 verify rows) form the M
 * dimension of one MMA tile, so each KV tile is staged once (TMA) for all of
 * them.  Same arguments, semantics and workspace contract as the decode entry.
 * Replaces the same reference function: paged_attn.py:152-222, as called for
 * Target verify rows from nebulasd/src/nebulasd/workers/target/backend.py:102-111. */
int neb_paged_attention_verify(const void* q, const void* k_cache, const void* v_cache,
                               const int32_t* block_table, int32_t block_table_rows,
                               int32_t max_blocks_per_seq, const int32_t* seq_lens,
                               const int32_t* seq_ids, int32_t num_rows, int32_t num_q_heads,
                               int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                               int64_t num_blocks, int32_t num_layers, int32_t cur_layer,
                               float softmax_scale, void* o, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Decode attention that allocates nothing.  It has no counterpart in the
 * reference.  Some callers cannot call cudaMalloc: a worker whose device
 * memory was claimed up front by its KV-cache pool (swiftLLM sizes the pool
 * from the free memory left after profiling), a host that forbids calls which
 * may synchronise the device while copies and compute overlap on other
 * streams, or an FFI host with no device allocator of its own.  This entry
 * takes the same arguments as neb_paged_attention_decode minus the workspace:
 * its split-K scratch is a 16 MiB static __device__ array inside this library
 * (held on every GPU that loads the library until the process exits).  A call
 * uses as many split-K workers as the array holds partials for (on a B200 at
 * q/kv head ratio 8, fewer than the workspace entry uses), so every ratio the
 * decode kernel supports fits; a call that would still need more fails with
 * NEB_ERR_WORKSPACE.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current and clears its
 * header and counters, so make that first call before any stream capture.
 * Every call clears the counters it needs to start at zero, on `stream`, and
 * allocates nothing.  The error bits the kernel records (the bits of
 * neb_workspace_status) accumulate in the array's header until
 * neb_paged_attention_noalloc_status reads and clears them.  All calls share
 * the one array: calls that may overlap on the GPU (different streams without
 * ordering between them) race and must not be made.  The library keeps the
 * array's address per device, so it must not outlive a reset of the device. */
int neb_paged_attention_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                       const int32_t* block_table, int32_t block_table_rows,
                                       int32_t max_blocks_per_seq, const int32_t* seq_lens,
                                       const int32_t* seq_ids, int32_t num_rows, int32_t num_q_heads,
                                       int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                       int64_t num_blocks, int32_t num_layers, int32_t cur_layer,
                                       float softmax_scale, void* o, void* stream);

/* Status of the allocation-free entry on the current device: synchronises
 * `stream`, then reads and clears the error bits its calls recorded since the
 * last read (0 when no such call ran on the device).  Allocates nothing.  It
 * has no counterpart in the reference (whose kernels record no errors). */
int neb_paged_attention_noalloc_status(uint32_t* error_bits, void* stream);

/* Target verify attention for long prefixes (thousands of tokens per request
 * and kv head), on tcgen05 tensor cores in the other orientation: 128 KV
 * tokens are the M dimension of S^T = K Q^T and of O^T += V^T P^T, and the GQA
 * heads x adjacent rows of one request (up to 64 query columns) the N
 * dimension, so that a 64 KB stage of K and V costs eight MMAs per issuing
 * thread.  Faster than neb_paged_attention_verify once the steady state
 * dominates (prefixes of about 8 K tokens and more); slower for short ones,
 * whose fixed per-launch costs it does not reduce.  Same arguments, semantics
 * and workspace contract as the decode entry; q/kv head ratios 1..64.
 * Replaces the same reference function: paged_attn.py:152-222. */
int neb_paged_attention_verify_long(const void* q, const void* k_cache, const void* v_cache,
                                    const int32_t* block_table, int32_t block_table_rows,
                                    int32_t max_blocks_per_seq, const int32_t* seq_lens,
                                    const int32_t* seq_ids, int32_t num_rows, int32_t num_q_heads,
                                    int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                    int64_t num_blocks, int32_t num_layers, int32_t cur_layer,
                                    float softmax_scale, void* o, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* Synchronises `stream`, then reads the error bits the attention kernels
 * recorded in `workspace` (bit 0: block index out of range, bit 1: seq_id out
 * of range, bit 2: sequence longer than max_blocks_per_seq, bit 3: a bounded
 * wait gave up, bit 4: invalid accept rows, bit 5: invalid prefill
 * cu_seqlens) and clears them.  After bit 3 it also clears the workspace's
 * split-K arrival counters (the call that gave up left some of them counted),
 * so call it before reusing a workspace whose last call may have failed. */
int neb_workspace_status(void* workspace, uint32_t* error_bits, void* stream);

/* ---------------------------------------------------------------- greedy accept
 * Greedy speculative acceptance on the device.  Replaces the verify-side tail
 * of the reference: torch.argmax of the logits
 * (swiftLLM/swiftllm/worker/layers/post_layer.py:72), the .tolist() of the
 * posterior tokens (swiftLLM/swiftllm/worker/model.py:465) and
 * compute_greedy_acceptance (swiftLLM/swiftllm/speculative.py:122-156), with
 * no host synchronisation.  No reference function takes these arguments; the
 * Python face is nebulasd_b200.accept.greedy_accept.
 *
 * logits        fp16 [num_rows][row_stride], the first `vocab` of each row used
 * row_start     [num_requests + 1]: request r owns rows row_start[r] ..
 *               row_start[r+1]-1 (k + 1 rows for k draft tokens)
 * draft_tokens  [num_rows - num_requests]: request r's k drafts start at
 *               row_start[r] - r
 * remaining     [num_requests] output budget (-1: none) or NULL
 * stop_tokens   [num_stop]
 * out_tokens    [num_requests][max_out]: the tokens to append, then -1
 * out_count     [num_requests]: how many; out_accepted: accepted drafts
 * argmax_out    [num_rows] arg-max per row (ties: lowest index; NaN counts as
 *               the largest value), or NULL
 * All arrays are device memory.  The workspace
 * (neb_greedy_accept_workspace_bytes) is zero-filled once and left zero by
 * every call; calls sharing it must be ordered on one stream.  Invalid rows or
 * budgets are recorded as error bit 4 (read with neb_workspace_status). */
size_t neb_greedy_accept_workspace_bytes(int32_t num_rows);
int neb_greedy_accept(const void* logits, int64_t row_stride, int32_t vocab, int32_t num_rows,
                      const int32_t* row_start, int32_t num_requests, const int32_t* draft_tokens,
                      const int32_t* remaining, const int32_t* stop_tokens, int32_t num_stop, int32_t max_out,
                      int32_t* argmax_out, int32_t* out_tokens, int32_t* out_count, int32_t* out_accepted,
                      void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------ prefill attention
 * Causal attention within each sequence of a packed prefill batch.  Replaces
 * flash_attn_varlen_func (swiftLLM/swiftllm/worker/layers/transformer_layer.py:7-32,
 * called at :154-164 with q and k covering the same sequences, causal=True),
 * without its copy of cu_seqlens to the host.
 *
 * q            fp16 [total_tokens][num_q_heads][128], q_stride elements between tokens
 * k, v         fp16 [total_tokens][num_kv_heads][128], k_stride / v_stride likewise
 * cu_seqlens   int32 [num_seqs + 1] on the device: sequence s is tokens
 *              cu_seqlens[s] .. cu_seqlens[s+1]-1 (cu_seqlens[0] = 0,
 *              cu_seqlens[num_seqs] = total_tokens)
 * max_seqlen   an upper bound of the sequence lengths (the reference's max_seqlen_q)
 * o            fp16 [total_tokens][num_q_heads][128], o_stride elements between tokens
 * q/kv head ratios 1, 2, 4, 8 and 16; head_dim 128; strides multiples of 8
 * elements; every pointer 16-byte aligned.  The workspace
 * (neb_prefill_attention_workspace_bytes) is zero-filled once; calls sharing
 * it must be ordered on one stream.  A cu_seqlens that is not a split of the
 * tokens, or a sequence longer than max_seqlen, is recorded as error bit 5
 * (read with neb_workspace_status) and its sequences are left out. */
size_t neb_prefill_attention_workspace_bytes(int64_t total_tokens, int32_t num_seqs, int32_t num_q_heads,
                                             int32_t num_kv_heads);
int neb_prefill_attention(const void* q, int64_t q_stride, const void* k, int64_t k_stride, const void* v,
                          int64_t v_stride, const int32_t* cu_seqlens, int32_t num_seqs, int64_t total_tokens,
                          int32_t max_seqlen, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                          float softmax_scale, void* o, int64_t o_stride, void* workspace,
                          size_t workspace_bytes, void* stream);

/* ------------------------------------------------ QK-norm, RoPE and KV store
 * Token layout of one forward (the reference's): prefill tokens first
 * (sequence s occupies [prefill_start_locs[s], +prefill_seq_lens[s]) with
 * seq_id seq_ids[s]), then num_decode_rows decode tokens (row r has seq_id
 * seq_ids[num_prefill_seqs + r] and position decode_seq_lens[r] - 1).
 * Out-of-range block ids / seq ids are skipped and OR-ed into *error_bits
 * (optional device word; same bits as neb_workspace_status). */

/* Fused Qwen3 QK-RMSNorm + RoPE + paged KV store, in one launch:
 *   q, k <- RoPE(RMSNorm(x) rounded to fp16)   (in place; norm skipped when the
 *                                               weights are null, RoPE when cos is null)
 *   k_cache/v_cache[slot(token)] <- k, v       (skipped when k_cache is null)
 * Replaces the call sequence swiftLLM/swiftllm/worker/layers/transformer_layer.py:114-143
 * (rmsnorm_inplace x2 rmsnorm.py:26-37, rotary_embedding_inplace rotary_emb.py:44-58,
 * store_kvcache kvcache_mgmt.py:81-122). */
int neb_qk_norm_rope_store(void* q, void* k, const void* v, const void* q_norm_w,
                           const void* k_norm_w, float eps, const void* cos, const void* sin,
                           void* k_cache, void* v_cache, const int32_t* block_table,
                           int32_t block_table_rows, int32_t max_blocks_per_seq,
                           const int32_t* seq_ids, const int32_t* decode_seq_lens,
                           int32_t num_decode_rows, const int32_t* prefill_start_locs,
                           const int32_t* prefill_seq_lens, int32_t num_prefill_seqs,
                           int32_t num_prefill_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                           int32_t head_dim, int32_t block_size, int64_t num_blocks,
                           int32_t num_layers, int32_t cur_layer, uint32_t* error_bits,
                           void* stream);

/* Paged KV store only (bit copies).  Replaces store_kvcache,
 * swiftLLM/swiftllm/worker/kernels/kvcache_mgmt.py:81-122 (kernels :10-79). */
int neb_store_kvcache(const void* k, const void* v, void* k_cache, void* v_cache,
                      const int32_t* block_table, int32_t block_table_rows,
                      int32_t max_blocks_per_seq, const int32_t* seq_ids,
                      const int32_t* decode_seq_lens, int32_t num_decode_rows,
                      const int32_t* prefill_start_locs, const int32_t* prefill_seq_lens,
                      int32_t num_prefill_seqs, int32_t num_prefill_tokens, int32_t num_kv_heads,
                      int32_t head_dim, int32_t block_size, int64_t num_blocks, int32_t num_layers,
                      int32_t cur_layer, uint32_t* error_bits, void* stream);

/* In-place RMSNorm of num_rows rows of `hidden` fp16 values.  Replaces
 * rmsnorm_inplace, swiftLLM/swiftllm/worker/kernels/rmsnorm.py:26-37. */
int neb_rmsnorm_inplace(void* x, const void* weight, int64_t num_rows, int32_t hidden, float eps,
                        void* stream);

/* In-place rotate-half RoPE of q [T, Hq, 128] and k [T, Hk, 128] with fp16
 * cos/sin rows [T, 64], in the reference's fp16 arithmetic.  Replaces
 * rotary_embedding_inplace, swiftLLM/swiftllm/worker/kernels/rotary_emb.py:44-58. */
int neb_rotary_inplace(void* q, void* k, const void* cos, const void* sin, int32_t num_tokens,
                       int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, void* stream);

/* ------------------------------------------------------------ HostKV copies
 * direction 0 = D2H (writeback), 1 = H2D (restore).  regions: host array of
 * num_regions triples (host_block, gpu_block, block_count), host_block
 * already including the extent offset; each block moves block_bytes bytes of
 * the K plane and of the V plane.  Destination ranges must not overlap.
 * mode 0: one cudaMemcpyAsync per merged run of adjacent regions and plane;
 * mode 1: one copy kernel for the whole plan (host planes must be pinned and
 * mapped; pass their device addresses, see neb_host_device_pointer).
 * Replaces CudaCopyBackend.launch, nebulasd/src/nebulasd/kv/cuda_transfer.py:78-108,
 * and swap_blocks, swiftLLM/csrc/src/block_swapping.cpp:22-85. */
int neb_hostkv_copy(int direction, const void* host_k_plane, const void* host_v_plane,
                    void* k_cache, void* v_cache, int64_t block_bytes, const int64_t* regions,
                    int32_t num_regions, int32_t mode, void* stream);

/* Same-role KV migration as a direct GPU-to-GPU copy: regions are triples
 * (src_block, dst_block, block_count) between two caches of one layout; run
 * on the destination device (mode 1 reads the peer cache from a kernel over
 * NVLink; enable access first with neb_enable_peer_access).  Replaces the
 * writeback + restore through HostKV of nebulasd/docs/current/KV.md:3-22. */
int neb_kv_peer_copy(const void* src_k_cache, const void* src_v_cache, void* dst_k_cache,
                     void* dst_v_cache, int64_t block_bytes, const int64_t* regions,
                     int32_t num_regions, int32_t mode, void* stream);

/* Device address of pinned, mapped host memory (cudaHostGetDevicePointer). */
int neb_host_device_pointer(void* host_ptr, void** device_ptr);

/* Lets the current device read `peer_device`'s memory (idempotent). */
int neb_enable_peer_access(int peer_device);

#ifdef __cplusplus
}
#endif
#endif /* NEBULA_B200_H */
