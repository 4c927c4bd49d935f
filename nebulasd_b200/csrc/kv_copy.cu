// HostKV restore/writeback block copies and same-role KV migration.
//
// Reference: nebulasd/src/nebulasd/kv/cuda_transfer.py:78-108 issues, per
// region and per plane (K then V), one cudaMemcpyAsync of
// block_count * block_bytes bytes between
//   host = arena + plane_offset + (extent.offset_blocks + host_begin) * block_bytes
//   gpu  = cache + gpu_begin * block_bytes
// on the backend's stream; swiftLLM/csrc/src/block_swapping.cpp:22-85 does the
// same for the legacy swap path after merging runs of consecutive block ids.
//
// Here one launch moves every region of a plan, both planes, as a byte stream
// cut into equal 64 KiB chunks (the region list rides in the kernel
// parameters, so no descriptor upload is needed).  Each thread keeps four
// 16-byte loads in flight before storing, which is what hides the ~1-2 us
// latency of host memory reads across PCIe.  The same kernel runs device ->
// device across NVLink for migration, reading the peer's cache through its
// unified address.  A copy-engine mode merges adjacent regions and issues one
// cudaMemcpyAsync per merged run and plane, like the reference, for callers
// whose host memory is not mapped into the device address space.
#include <algorithm>
#include <vector>

#include "neb_common.cuh"

namespace neb {

constexpr int kMaxCopyRegions = 1024;
constexpr long long kChunkBytes = 64 * 1024;
constexpr int kCopyThreads = 256;

struct CopyRegions {
  const char* src[2];  // K plane, V plane
  char* dst[2];
  long long block_bytes;
  int num_regions;
  long long total_bytes_per_plane;
  long long src_block[kMaxCopyRegions / 2];
  long long dst_block[kMaxCopyRegions / 2];
  long long first_byte[kMaxCopyRegions / 2 + 1];  // prefix of region bytes within a plane
};
constexpr int kRegionsPerLaunch = kMaxCopyRegions / 2;
static_assert(sizeof(CopyRegions) < 32000, "kernel parameter block must stay under 32 KB");

__global__ void __launch_bounds__(kCopyThreads) copy_regions_kernel(const __grid_constant__ CopyRegions r) {
  const long long per_plane = r.total_bytes_per_plane;
  const long long chunks_per_plane = (per_plane + kChunkBytes - 1) / kChunkBytes;
  for (long long c = blockIdx.x; c < 2 * chunks_per_plane; c += gridDim.x) {
    const int plane = (int)(c / chunks_per_plane);
    const long long lo = (c - plane * chunks_per_plane) * kChunkBytes;
    const long long hi = min(lo + kChunkBytes, per_plane);
    // region containing byte `lo`
    int a = 0, b = r.num_regions;
    while (b - a > 1) {
      const int m = (a + b) >> 1;
      if (r.first_byte[m] <= lo) a = m; else b = m;
    }
    long long pos = lo;
    int reg = a;
    while (pos < hi) {
      while (r.first_byte[reg + 1] <= pos) ++reg;
      const long long seg_end = min(hi, r.first_byte[reg + 1]);
      const long long off = pos - r.first_byte[reg];
      const uint4* s = reinterpret_cast<const uint4*>(r.src[plane] + r.src_block[reg] * r.block_bytes + off);
      uint4* d = reinterpret_cast<uint4*>(r.dst[plane] + r.dst_block[reg] * r.block_bytes + off);
      const long long n = (seg_end - pos) >> 4;
      long long i = threadIdx.x;
      for (; i + 3 * kCopyThreads < n; i += 4 * kCopyThreads) {
        const uint4 v0 = __ldcv(s + i);
        const uint4 v1 = __ldcv(s + i + kCopyThreads);
        const uint4 v2 = __ldcv(s + i + 2 * kCopyThreads);
        const uint4 v3 = __ldcv(s + i + 3 * kCopyThreads);
        __stcs(d + i, v0);
        __stcs(d + i + kCopyThreads, v1);
        __stcs(d + i + 2 * kCopyThreads, v2);
        __stcs(d + i + 3 * kCopyThreads, v3);
      }
      for (; i < n; i += kCopyThreads) __stcs(d + i, __ldcv(s + i));
      pos = seg_end;
    }
  }
}

// regions: n triples (src_block, dst_block, block_count), host memory.
static int copy_regions(const void* src_k, const void* src_v, void* dst_k, void* dst_v,
                        long long block_bytes, const int64_t* regions, int n, int mode,
                        cudaStream_t stream) {
  NEB_REQUIRE(block_bytes > 0 && block_bytes % 16 == 0, NEB_ERR_INVALID,
              "block_bytes must be a positive multiple of 16 (got %lld)", block_bytes);
  NEB_REQUIRE(n >= 0 && (n == 0 || regions), NEB_ERR_INVALID, "bad region list");
  NEB_REQUIRE(src_k && src_v && dst_k && dst_v, NEB_ERR_INVALID, "null plane pointer");
  for (int i = 0; i < n; ++i)
    NEB_REQUIRE(regions[3 * i] >= 0 && regions[3 * i + 1] >= 0 && regions[3 * i + 2] >= 0,
                NEB_ERR_INVALID, "negative copy range in region %d", i);
  {
    // Regions run concurrently in the kernel path, so destinations must not
    // overlap (HostKV plans name distinct extents and bank ranges).
    std::vector<std::pair<long long, long long>> iv;
    for (int i = 0; i < n; ++i)
      if (regions[3 * i + 2] > 0) iv.emplace_back(regions[3 * i + 1], regions[3 * i + 1] + regions[3 * i + 2]);
    std::sort(iv.begin(), iv.end());
    for (size_t i = 1; i < iv.size(); ++i)
      NEB_REQUIRE(iv[i].first >= iv[i - 1].second, NEB_ERR_INVALID,
                  "copy regions overlap at destination block %lld", iv[i].first);
  }
  if (mode == 0) {
    // Copy engines: merge runs that are contiguous on both sides (order kept).
    const char* src[2] = {static_cast<const char*>(src_k), static_cast<const char*>(src_v)};
    char* dst[2] = {static_cast<char*>(dst_k), static_cast<char*>(dst_v)};
    int i = 0;
    while (i < n) {
      long long s0 = regions[3 * i], d0 = regions[3 * i + 1], cnt = regions[3 * i + 2];
      int j = i + 1;
      while (j < n && regions[3 * j] == s0 + cnt && regions[3 * j + 1] == d0 + cnt) {
        cnt += regions[3 * j + 2];
        ++j;
      }
      if (cnt > 0)
        for (int pl = 0; pl < 2; ++pl)
          NEB_CUDA(cudaMemcpyAsync(dst[pl] + d0 * block_bytes, src[pl] + s0 * block_bytes,
                                   (size_t)(cnt * block_bytes), cudaMemcpyDefault, stream));
      i = j;
    }
    return NEB_OK;
  }
  NEB_REQUIRE(mode == 1, NEB_ERR_INVALID, "copy mode must be 0 (copy engines) or 1 (kernel)");
  NEB_REQUIRE(((reinterpret_cast<uintptr_t>(src_k) | reinterpret_cast<uintptr_t>(src_v) |
                reinterpret_cast<uintptr_t>(dst_k) | reinterpret_cast<uintptr_t>(dst_v)) & 15u) == 0,
              NEB_ERR_INVALID, "kernel copies need 16-byte aligned planes");
  int dev = 0;
  NEB_CUDA(cudaGetDevice(&dev));
  const int sms = num_sms(dev);
  for (int base = 0; base < n; base += kRegionsPerLaunch) {
    CopyRegions r;
    r.src[0] = static_cast<const char*>(src_k);
    r.src[1] = static_cast<const char*>(src_v);
    r.dst[0] = static_cast<char*>(dst_k);
    r.dst[1] = static_cast<char*>(dst_v);
    r.block_bytes = block_bytes;
    int m = 0;
    long long acc = 0;
    for (int i = base; i < n && m < kRegionsPerLaunch; ++i) {
      if (regions[3 * i + 2] == 0) continue;
      r.src_block[m] = regions[3 * i];
      r.dst_block[m] = regions[3 * i + 1];
      r.first_byte[m] = acc;
      acc += regions[3 * i + 2] * block_bytes;
      ++m;
    }
    r.first_byte[m] = acc;
    r.num_regions = m;
    r.total_bytes_per_plane = acc;
    if (m == 0) continue;
    const long long chunks = 2 * ((acc + kChunkBytes - 1) / kChunkBytes);
    const int grid = (int)std::min<long long>(chunks, (long long)sms * 8);
    copy_regions_kernel<<<grid, kCopyThreads, 0, stream>>>(r);
    NEB_CUDA(cudaGetLastError());
  }
  return NEB_OK;
}

}  // namespace neb

using namespace neb;

extern "C" {

int neb_hostkv_copy(int direction, const void* host_k_plane, const void* host_v_plane, void* k_cache,
                    void* v_cache, int64_t block_bytes, const int64_t* regions, int32_t num_regions,
                    int32_t mode, void* stream) {
  NEB_REQUIRE(direction == 0 || direction == 1, NEB_ERR_INVALID, "direction must be 0 (D2H) or 1 (H2D)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (direction == 1)  // H2D: host block -> gpu block
    return copy_regions(host_k_plane, host_v_plane, k_cache, v_cache, block_bytes, regions, num_regions, mode, s);
  // D2H: swap columns so the source is the GPU cache.
  std::vector<int64_t> swapped(3 * (size_t)std::max(num_regions, 0));
  for (int i = 0; i < num_regions; ++i) {
    swapped[3 * i] = regions[3 * i + 1];
    swapped[3 * i + 1] = regions[3 * i];
    swapped[3 * i + 2] = regions[3 * i + 2];
  }
  return copy_regions(k_cache, v_cache, const_cast<void*>(host_k_plane), const_cast<void*>(host_v_plane),
                      block_bytes, swapped.data(), num_regions, mode, s);
}

int neb_kv_peer_copy(const void* src_k_cache, const void* src_v_cache, void* dst_k_cache, void* dst_v_cache,
                     int64_t block_bytes, const int64_t* regions, int32_t num_regions, int32_t mode,
                     void* stream) {
  return copy_regions(src_k_cache, src_v_cache, dst_k_cache, dst_v_cache, block_bytes, regions, num_regions,
                      mode, static_cast<cudaStream_t>(stream));
}

int neb_host_device_pointer(void* host_ptr, void** device_ptr) {
  NEB_REQUIRE(host_ptr && device_ptr, NEB_ERR_INVALID, "null argument");
  NEB_CUDA(cudaHostGetDevicePointer(device_ptr, host_ptr, 0));
  return NEB_OK;
}

int neb_enable_peer_access(int peer_device) {
  int dev = 0, can = 0;
  NEB_CUDA(cudaGetDevice(&dev));
  NEB_REQUIRE(peer_device != dev, NEB_ERR_INVALID, "peer device equals the current device");
  NEB_CUDA(cudaDeviceCanAccessPeer(&can, dev, peer_device));
  NEB_REQUIRE(can, NEB_ERR_UNSUPPORTED, "device %d cannot access device %d", dev, peer_device);
  cudaError_t e = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return NEB_OK;
  }
  NEB_CUDA(e);
  return NEB_OK;
}

}  // extern "C"
