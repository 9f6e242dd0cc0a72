// kvx_swap_noalloc: the per-tensor swap (kvx_swap semantics, SM zero-copy
// path) for callers that cannot allocate GPU memory.
//
// Some callers must not call cudaMalloc or any allocating library routine
// while they move KV blocks: a runtime that owns every byte of HBM through its
// own arena (the reference's worker carves its KV cache out of one big arena
// and expects nothing else to appear next to it), a process that swaps while
// it is close to the memory limit during a model switch, or code running
// where an allocation would synchronise the device or fail.  The regular
// entry points keep their work-item tables in a device ring the library
// allocates on first use; this one instead keeps its scratch (the id lists of
// the call) in a fixed, file-scope device array.  Every GPU that loads
// libkvx.so holds that array (KVX_NOALLOC_MAX_IDS * 16 bytes = 1 MiB) until
// the process exits.
//
// The caller still provides the inputs and outputs (cache, page-locked host
// buffer, id lists).  Nothing here calls cudaMalloc, cudaFree, cudaHostAlloc
// or a library routine that allocates; host-side scratch is static storage.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/kvx.h"
#include "kvx_kernels.cuh"

namespace kvx {
void record_error(const std::string& msg);  // kvx_runtime.cu

namespace {

constexpr int64_t kMaxIds = KVX_NOALLOC_MAX_IDS;
constexpr uint32_t kTileShift = 15;  // 32 KiB tiles, as the regular SM path

// The scratch: source ids in [0, kMaxIds), target ids in [kMaxIds, 2*kMaxIds).
// Host code must not use this name as an address (it is a host-side stand-in);
// it obtains the device address with cudaGetSymbolAddress.
static __device__ __align__(256) int64_t g_noalloc_ids[2 * kMaxIds];

// Host-side static work areas (no heap use), guarded by g_mu.
std::mutex g_mu;
struct Pair {
  int64_t target;
  int64_t index;
};
Pair g_pairs[kMaxIds];
int64_t g_upload[2 * kMaxIds];
int64_t* g_scratch_ptr[64] = {};  // per device, set once

int fail(int code, const char* msg) {
  record_error(msg);  // shown by kvx_last_error()
  return code;
}

// Ids are read from the scratch; block b of a buffer is [b*B, (b+1)*B).
template <int kSrc>
__global__ void __launch_bounds__(kVecThreads)
    kvx_copy_ids(const int64_t* __restrict__ ids, uint32_t m, uint64_t block_bytes,
                 uint64_t src_base, uint64_t dst_base, uint32_t tiles_per_block) {
  uint32_t t0, t1;
  cta_span(m * tiles_per_block, &t0, &t1);
  for (uint32_t t = t0; t < t1; ++t) {
    const uint32_t i = t / tiles_per_block;
    const uint64_t off = uint64_t(t % tiles_per_block) << kTileShift;
    const uint64_t n = min(block_bytes - off, uint64_t(1) << kTileShift);
    const uint64_t s = src_base + uint64_t(ids[i]) * block_bytes + off;
    const uint64_t d = dst_base + uint64_t(ids[kMaxIds + i]) * block_bytes + off;
    cta_copy<kSrc>(reinterpret_cast<const char*>(s), reinterpret_cast<char*>(d), uint32_t(n));
  }
}

// Device address of the scratch on `device` (which is current); looked up once.
int scratch_for(int device, int64_t** out) {
  if (device < 0 || device >= 64) return fail(KVX_ERR_INVALID_ARGUMENT, "device index out of range");
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_ids);
    if (e != cudaSuccess)
      return fail(KVX_ERR_CUDA, (std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e)).c_str());
    g_scratch_ptr[device] = static_cast<int64_t*>(p);
  }
  *out = g_scratch_ptr[device];
  return KVX_OK;
}

}  // namespace
}  // namespace kvx

using namespace kvx;

extern "C" {

int kvx_swap_noalloc(const int64_t* source_block_ids, const int64_t* target_block_ids,
                     int64_t num_ids, int is_swap_in, void* kv_cache, uint64_t kv_cache_bytes,
                     uint64_t block_bytes, void* kv_swap, uint64_t kv_swap_bytes, void* stream) {
  record_error("");
  if (num_ids < 0) return fail(KVX_ERR_INVALID_ARGUMENT, "negative id count");
  if (num_ids > kMaxIds)
    return fail(KVX_ERR_INVALID_ARGUMENT,
                "kvx_swap_noalloc: more ids than KVX_NOALLOC_MAX_IDS (65536) in one call");
  if (num_ids == 0 || block_bytes == 0) return KVX_OK;
  if (!source_block_ids || !target_block_ids || !kv_cache || !kv_swap)
    return fail(KVX_ERR_INVALID_ARGUMENT, "null argument");
  if ((block_bytes >> kTileShift) >= (1ull << 20))
    return fail(KVX_ERR_INVALID_ARGUMENT, "block_bytes too large");
  const uint64_t cache_blocks = kv_cache_bytes / block_bytes;
  const uint64_t swap_blocks = kv_swap_bytes / block_bytes;
  for (int64_t i = 0; i < num_ids; ++i) {
    const int64_t dev = is_swap_in ? target_block_ids[i] : source_block_ids[i];
    const int64_t slot = is_swap_in ? source_block_ids[i] : target_block_ids[i];
    if (dev < 0 || uint64_t(dev) >= cache_blocks)
      return fail(KVX_ERR_BLOCK_ID, "kv_cache block id out of range");
    if (slot < 0 || uint64_t(slot) >= swap_blocks)
      return fail(KVX_ERR_BLOCK_ID, "kv_swap block id out of range");
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The ids travel through static host storage that the next call reuses, so
  // a copy recorded into a graph would read whatever a later call left there:
  // a capturing stream is refused before anything is queued.
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(s, &capture);
  if (e != cudaSuccess) return fail(KVX_ERR_CUDA, "cudaStreamIsCapturing failed");
  if (capture != cudaStreamCaptureStatusNone)
    return fail(KVX_ERR_INVALID_ARGUMENT,
                "kvx_swap_noalloc: the stream is capturing; call it on a stream that is not");
  int device = 0;
  e = cudaGetDevice(&device);
  if (e != cudaSuccess) return fail(KVX_ERR_CUDA, "cudaGetDevice failed");
  // Memory kinds as kvx_swap accepts them: the cache in device or managed
  // memory of this device, the host side page-locked and mapped, or managed.
  cudaPointerAttributes ca, ha;
  if (cudaPointerGetAttributes(&ca, kv_cache) != cudaSuccess ||
      !(ca.type == cudaMemoryTypeManaged ||
        (ca.type == cudaMemoryTypeDevice && ca.device == device))) {
    cudaGetLastError();
    return fail(KVX_ERR_INVALID_ARGUMENT,
                "kv_cache is not device (or managed) memory of the current device");
  }
  uint64_t host_dev = 0;
  if (cudaPointerGetAttributes(&ha, kv_swap) != cudaSuccess) {
    cudaGetLastError();
  } else if (ha.type == cudaMemoryTypeHost && ha.devicePointer) {
    host_dev = reinterpret_cast<uint64_t>(ha.devicePointer);
  } else if (ha.type == cudaMemoryTypeManaged) {
    host_dev = reinterpret_cast<uint64_t>(kv_swap);
  }
  if (!host_dev)
    return fail(KVX_ERR_HOST_MEMORY,
                "kv_swap must be page-locked host memory mapped for the device "
                "(cudaHostAlloc or cudaHostRegister) or managed memory");
  const uint32_t tiles_per_block = uint32_t((block_bytes + (1u << kTileShift) - 1) >> kTileShift);
  if (uint64_t(num_ids) * tiles_per_block > 0xffffffffull)
    return fail(KVX_ERR_INVALID_ARGUMENT, "request too large for one call");
  std::lock_guard<std::mutex> g(g_mu);
  int64_t* scratch = nullptr;
  int rc = scratch_for(device, &scratch);
  if (rc) return rc;
  // Keep the last copy per target (what in-order copies leave behind); the
  // survivors have distinct targets, so they may run in any order.
  for (int64_t i = 0; i < num_ids; ++i) g_pairs[i] = Pair{target_block_ids[i], i};
  std::sort(g_pairs, g_pairs + num_ids, [](const Pair& a, const Pair& b) {
    return a.target != b.target ? a.target < b.target : a.index < b.index;
  });
  int64_t m = 0;
  for (int64_t k = 0; k < num_ids; ++k) {
    if (k + 1 < num_ids && g_pairs[k + 1].target == g_pairs[k].target) continue;
    g_upload[m] = source_block_ids[g_pairs[k].index];
    g_upload[kMaxIds + m] = g_pairs[k].target;
    ++m;
  }
  // g_upload is pageable.  The runtime's documented behaviour for an
  // asynchronous copy from pageable host memory to the device is to copy the
  // source into its own staging memory before the call returns, so g_upload
  // may be rewritten by the next call as soon as these return.
  e = cudaMemcpyAsync(scratch, g_upload, size_t(m) * sizeof(int64_t), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(scratch + kMaxIds, g_upload + kMaxIds, size_t(m) * sizeof(int64_t),
                        cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return fail(KVX_ERR_CUDA, "id upload failed");
  const uint64_t tiles = uint64_t(m) * tiles_per_block;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const uint32_t grid = uint32_t(std::min<uint64_t>(tiles, host_path_ctas(sms, !is_swap_in)));
  const uint64_t cache = reinterpret_cast<uint64_t>(kv_cache);
  if (is_swap_in)
    kvx_copy_ids<kSrcHost><<<grid, kVecThreads, 0, s>>>(scratch, uint32_t(m), block_bytes,
                                                         host_dev, cache, tiles_per_block);
  else
    kvx_copy_ids<kSrcDevice><<<grid, kVecThreads, 0, s>>>(scratch, uint32_t(m), block_bytes,
                                                           cache, host_dev, tiles_per_block);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(KVX_ERR_CUDA, cudaGetErrorString(e));
  return KVX_OK;
}

}  // extern "C"
