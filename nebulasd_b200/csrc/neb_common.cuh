// Shared helpers of the NebulaSD B200 attention-path library (sm_100a only).
#pragma once

#include <climits>
#include <cstdint>
#include <cstdio>
#include <utility>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/nebula_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "nebula_b200 is built for sm_100a only"
#endif

namespace neb {

// ---------------------------------------------------------------- host errors
// Each C entry point returns an int status (0 = ok).  The message of the last
// failure on the calling host thread is kept for neb_last_error().
int set_error(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);

#define NEB_REQUIRE(cond, code, ...)                      \
  do {                                                    \
    if (!(cond)) return ::neb::set_error((code), __VA_ARGS__); \
  } while (0)

#define NEB_CUDA(call)                                    \
  do {                                                    \
    cudaError_t _e = (call);                              \
    if (_e != cudaSuccess) return ::neb::check_cuda(_e, #call); \
  } while (0)

int num_sms(int device);

// ------------------------------------------------------------- device helpers
// Device-side error bits recorded in the workspace header (never a trap).
enum DeviceError : uint32_t {
  kErrBlockIndex = 1u << 0,   // block_table entry outside [0, num_blocks)
  kErrSeqId = 1u << 1,        // seq_id outside [0, block_table_rows)
  kErrTooManyBlocks = 1u << 2,  // sequence needs more than max_blocks_per_seq blocks
  kErrTimeout = 1u << 3,      // a bounded wait gave up
  kErrInvalidRows = 1u << 4,  // greedy accept: a request's rows or output limit are invalid
  kErrBadSeqlens = 1u << 5,   // prefill: cu_seqlens not a valid split of the tokens (or past max_seqlen)
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Programmatic dependent launch: let the next kernel in the stream be
// scheduled (pdl_trigger), and wait until the previous one has completed and
// its memory is visible (pdl_wait; a no-op when the launch did not ask for
// programmatic serialisation).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launches `kernel` on `stream` with programmatic stream serialisation.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Workspace header shared by the attention kernels (first 256 bytes).
struct WorkspaceHeader {
  uint32_t error_bits;
  uint32_t timeout_site;
  uint32_t reserved[62];
};
static_assert(sizeof(WorkspaceHeader) == 256, "header is 256 bytes");

__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t u) {
  __half2 h = *reinterpret_cast<__half2*>(&u);
  return __half22float2(h);
}

__device__ __forceinline__ uint32_t f2_to_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000u); }

// Units per worker of the balanced split: worker w owns tiles [a_w, a_{w+1})
// with a_w = floor(w * T / W).  worker_of(t) inverts it.
__host__ __device__ __forceinline__ long long range_begin(long long w, long long total, long long workers) {
  return (w * total) / workers;
}
__host__ __device__ __forceinline__ long long worker_of(long long t, long long total, long long workers) {
  return ((t + 1) * workers - 1) / total;
}

}  // namespace neb
