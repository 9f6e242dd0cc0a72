// Copy kernels for KV-block movement on sm_100a.
//
// Both kernels walk a work list: an item list (kvx::Item: source,
// destination, length, first tile) or a grid list (entries x segments,
// kvx_worklist.h).  The launch-wide tile sequence is split into one
// contiguous span per CTA, so every CTA moves the same number of tiles and
// streams through memory in order; a CTA finds its first record by binary
// search and then advances record by record.
//
//  * kvx_copy_vec  : 32-byte vector loads and stores where source, destination
//                    and length allow (16-byte and byte fallbacks), 128 bytes
//                    in flight per thread (32 KiB per 256-thread CTA).  Works
//                    on any memory the SM can address: local HBM,
//                    device-mapped page-locked host memory (PCIe) and
//                    IPC-mapped peer HBM (NVLink).
//                    kvx_copy_vec_inline is the same kernel with a small grid
//                    list passed by value in its parameters.
//  * kvx_copy_bulk : local HBM only.  One elected thread runs a ring of TMA
//                    bulk copies (cp.async.bulk global->shared completing on
//                    an mbarrier, then shared->global in bulk groups).  Every
//                    mbarrier wait is bounded by a %globaltimer deadline; on
//                    expiry the kernel records KVX_ERR_DEVICE_TIMEOUT in the
//                    device status word, drains its own bulk stores (also
//                    bounded) and returns.  No multicast form is used.
#pragma once

#include <cstdint>

#include "kvx_plan.h"
#include "kvx_worklist.h"

namespace kvx {

constexpr int kVecThreads = 256;
constexpr int kVecUnroll = 8;  // 256 threads x 8 x 16 B = 32 KiB per pass

enum SrcKind : int { kSrcDevice = 0, kSrcHost = 1 };

// CTAs of a vector-kernel launch with a host side.  Swap-out and swap-in
// kernels run at the same time and must fit on the SMs together (two CTAs
// per SM in all): 3/4 of the SM count for writes to host memory, 5/4 for
// reads from it.  One direction alone moves the same bytes per second with
// writes at 1/2 to 1 CTA per SM and reads at 3/4 to 3/2; with both
// directions at once this split moves 0.80 of the bidirectional link where
// one CTA per SM each way moves 0.70 (scattered 896 KiB host rows).
inline uint32_t host_path_ctas(int sms, bool to_host) {
  const int ctas = to_host ? sms * 3 / 4 : sms * 5 / 4;
  return uint32_t(ctas > 0 ? ctas : 1);
}

__device__ __forceinline__ uint4 ld_dev16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ld_host16(const void* p) {
  uint4 r;
  asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void st16(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// 32-byte accesses (sm_100 256-bit global loads / stores).
struct V32 {
  uint4 a, b;
};

__device__ __forceinline__ V32 ld_dev32(const void* p) {
  V32 r;
  asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r.a.x), "=r"(r.a.y), "=r"(r.a.z), "=r"(r.a.w), "=r"(r.b.x),
                 "=r"(r.b.y), "=r"(r.b.z), "=r"(r.b.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ V32 ld_host32(const void* p) {
  V32 r;
  asm volatile("ld.global.cs.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r.a.x), "=r"(r.a.y), "=r"(r.a.z), "=r"(r.a.w), "=r"(r.b.x),
                 "=r"(r.b.y), "=r"(r.b.z), "=r"(r.b.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void st32(void* p, const V32& v) {
  asm volatile("st.global.cs.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v.a.x),
               "r"(v.a.y), "r"(v.a.z), "r"(v.a.w), "r"(v.b.x), "r"(v.b.y), "r"(v.b.z),
               "r"(v.b.w)
               : "memory");
}

// Largest i with items[i].tile_begin <= t (items sorted, items[0].tile_begin == 0).
__device__ __forceinline__ uint32_t find_item(const Item* __restrict__ items,
                                              uint32_t n_items, uint32_t t) {
  uint32_t lo = 0, hi = n_items - 1;
  while (lo < hi) {
    const uint32_t mid = (lo + hi + 1) >> 1;
    if (items[mid].tile_begin <= t)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void cta_span(uint32_t n_tiles, uint32_t* t0,
                                         uint32_t* t1) {
  const uint32_t g = gridDim.x, b = blockIdx.x;
  const uint32_t per = n_tiles / g, rem = n_tiles % g;
  *t0 = b * per + min(b, rem);
  *t1 = *t0 + per + (b < rem ? 1u : 0u);
}

template <int kSrc>
__device__ __forceinline__ void cta_copy32(const char* __restrict__ s, char* __restrict__ d,
                                           uint32_t n) {
  constexpr int kU = kVecUnroll / 2;  // same bytes in flight per thread as 8 x 16 B
  const uint32_t n32 = n >> 5;
  for (uint32_t base = threadIdx.x; base < n32; base += kVecThreads * kU) {
    V32 r[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const uint32_t k = base + u * kVecThreads;
      if (k < n32) r[u] = kSrc == kSrcHost ? ld_host32(s + 32ull * k) : ld_dev32(s + 32ull * k);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const uint32_t k = base + u * kVecThreads;
      if (k < n32) st32(d + 32ull * k, r[u]);
    }
  }
}

template <int kSrc, int kVec = 16>
__device__ __forceinline__ void cta_copy(const char* __restrict__ s,
                                         char* __restrict__ d, uint32_t n) {
  if (kVec == 32 && ((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d) | n) &
                     31u) == 0) {
    cta_copy32<kSrc>(s, d, n);
  } else if (((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d) | n) &
       15u) == 0) {
    const uint32_t n16 = n >> 4;
    const uint4* s16 = reinterpret_cast<const uint4*>(s);
    uint4* d16 = reinterpret_cast<uint4*>(d);
    for (uint32_t base = threadIdx.x; base < n16;
         base += kVecThreads * kVecUnroll) {
      uint4 r[kVecUnroll];
#pragma unroll
      for (int u = 0; u < kVecUnroll; ++u) {
        const uint32_t k = base + u * kVecThreads;
        if (k < n16) r[u] = kSrc == kSrcHost ? ld_host16(s16 + k) : ld_dev16(s16 + k);
      }
#pragma unroll
      for (int u = 0; u < kVecUnroll; ++u) {
        const uint32_t k = base + u * kVecThreads;
        if (k < n16) st16(d16 + k, r[u]);
      }
    }
  } else {
    for (uint32_t k = threadIdx.x; k < n; k += kVecThreads) d[k] = s[k];
  }
}

// A work list maps a tile index to (source, destination, length).  seek()
// positions a cursor on the first tile of a CTA's span; get() advances the
// cursor monotonically.
struct ItemList {
  const Item* items;
  uint32_t n;
  __device__ __forceinline__ uint32_t seek(uint32_t t) const { return find_item(items, n, t); }
  __device__ __forceinline__ void get(uint32_t& cur, uint32_t t, uint32_t shift, uint64_t* src,
                                      uint64_t* dst, uint32_t* len) const {
    while (cur + 1 < n && items[cur + 1].tile_begin <= t) ++cur;
    const Item it = items[cur];
    const uint64_t off = uint64_t(t - it.tile_begin) << shift;
    *len = uint32_t(min(uint64_t(it.len) - off, uint64_t(1) << shift));
    *src = it.src + off;
    *dst = it.dst + off;
  }
};

struct GridList {
  const GridEntry* entries;
  uint32_t n;
  const GridSeg* segs;
  __device__ __forceinline__ uint32_t seek(uint32_t t) const { return grid_find(entries, n, t); }
  __device__ __forceinline__ void get(uint32_t& cur, uint32_t t, uint32_t shift, uint64_t* src,
                                      uint64_t* dst, uint32_t* len) const {
    while (cur + 1 < n && entries[cur + 1].tile_begin <= t) ++cur;
    grid_resolve(entries[cur], segs, t, shift, src, dst, len);
  }
};

// A grid list carried in the kernel's parameter space instead of a device
// table: small requests launch without a descriptor upload.  Entries occupy
// records [0, n), the segment table records [n, n + n_segs); both are 32-byte
// records.  Three capacities: 124 records (the parameter block within 4 KiB),
// 508 (16 KiB) and 1020 (within the 32,764-byte limit that sm_70 and later
// accept since CUDA 12.1); a launch uses the smallest that holds its plan, so
// it sends no more parameter bytes than it needs.
constexpr uint32_t kInlineRecords = 124;
constexpr uint32_t kInlineRecordsMid = 508;
constexpr uint32_t kInlineRecordsMax = 1020;

template <uint32_t kCap>
struct InlineGridListT {
  uint32_t n = 0;       // entries
  uint32_t n_segs = 0;  // segments
  uint32_t pad[2] = {};
  uint4 rec[2 * kCap];
  __host__ __device__ __forceinline__ const GridEntry* entries() const {
    return reinterpret_cast<const GridEntry*>(rec);
  }
  __host__ __device__ __forceinline__ const GridSeg* segs() const {
    return reinterpret_cast<const GridSeg*>(rec + 2 * n);
  }
  __device__ __forceinline__ uint32_t seek(uint32_t t) const { return grid_find(entries(), n, t); }
  __device__ __forceinline__ void get(uint32_t& cur, uint32_t t, uint32_t shift, uint64_t* src,
                                      uint64_t* dst, uint32_t* len) const {
    const GridEntry* e = entries();
    while (cur + 1 < n && e[cur + 1].tile_begin <= t) ++cur;
    grid_resolve(e[cur], segs(), t, shift, src, dst, len);
  }
};
using InlineGridList = InlineGridListT<kInlineRecords>;
using InlineGridListMid = InlineGridListT<kInlineRecordsMid>;
using InlineGridListMax = InlineGridListT<kInlineRecordsMax>;
// the list plus the kernel's two 32-bit arguments
static_assert(sizeof(InlineGridList) + 8 <= 4096, "inline list exceeds 4 KiB");
static_assert(sizeof(InlineGridListMid) + 8 <= 16384, "inline list exceeds 16 KiB");
static_assert(sizeof(InlineGridListMax) + 8 <= 32764, "inline list exceeds the parameter limit");

template <int kSrc, int kVec, class List>
__device__ __forceinline__ void copy_tiles(const List& list, uint32_t n_tiles,
                                           uint32_t tile_shift) {
  uint32_t t0, t1;
  cta_span(n_tiles, &t0, &t1);
  if (t0 >= t1) return;
  uint32_t cur = list.seek(t0);
  for (uint32_t t = t0; t < t1; ++t) {
    uint64_t src, dst;
    uint32_t n;
    list.get(cur, t, tile_shift, &src, &dst, &n);
    cta_copy<kSrc, kVec>(reinterpret_cast<const char*>(src), reinterpret_cast<char*>(dst), n);
  }
}

template <int kSrc, class List, int kVec = 16>
__global__ void __launch_bounds__(kVecThreads)
    kvx_copy_vec(List list, uint32_t n_tiles, uint32_t tile_shift) {
  copy_tiles<kSrc, kVec>(list, n_tiles, tile_shift);
}

// Same copy with the work list read in place from the parameter space
// (__grid_constant__: no per-thread copy of the list).
template <int kSrc, int kVec, class InlineList>
__global__ void __launch_bounds__(kVecThreads)
    kvx_copy_vec_inline(const __grid_constant__ InlineList list, uint32_t n_tiles,
                        uint32_t tile_shift) {
  copy_tiles<kSrc, kVec>(list, n_tiles, tile_shift);
}

// ---- TMA bulk copy (local HBM only) ----------------------------------------

// Device error word: set by kernels whose bounded waits gave up.
static __device__ int g_kvx_device_status;

constexpr int kBulkStages = 6;
constexpr uint32_t kBulkShift = 14;
constexpr uint32_t kBulkChunk = 1u << kBulkShift;  // one tile per stage
constexpr uint32_t kBulkSmem = kBulkStages * kBulkChunk + kBulkStages * 8;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per wait

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait; false when the deadline passed.
__device__ __forceinline__ bool mbar_wait_for(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t start = global_ns();
  while (!mbar_try(bar, parity))
    if (global_ns() - start > limit_ns) return false;
  return true;
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  return mbar_wait_for(bar, parity, kWaitLimitNs);
}

// Self-test of the bounded wait: waits on an mbarrier that nothing arrives on;
// the wait gives up after limit_ns and the kernel records the timeout in the
// device status word, exactly as the copy kernel does.
static __global__ void __launch_bounds__(32) kvx_wait_selftest(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  const uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(&bar));
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(b) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  if (!mbar_wait_for(b, 0, limit_ns)) atomicExch(&g_kvx_device_status, 8 /* timeout */);
}

__device__ __forceinline__ void bulk_load(uint32_t smem, const void* src,
                                          uint32_t bytes, uint32_t bar) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
      "r"(bytes)
      : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(smem),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void bulk_store(void* dst, uint32_t smem,
                                           uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                   dst),
               "r"(smem), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_read_le1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Requires every copy 16-byte aligned in address and length (the host checks)
// and a tile size of kBulkChunk.
template <class List>
__global__ void __launch_bounds__(32) kvx_copy_bulk(List list, uint32_t n_tiles) {
  extern __shared__ __align__(128) unsigned char smem[];
  if (threadIdx.x != 0) return;
  uint32_t t0, t1;
  cta_span(n_tiles, &t0, &t1);
  if (t0 >= t1) return;
  const uint32_t T = t1 - t0;
  const uint32_t buf0 = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const uint32_t bar0 = buf0 + kBulkStages * kBulkChunk;
  for (int s = 0; s < kBulkStages; ++s)
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8 * s)
                 : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

  uint64_t st_dst[kBulkStages];
  uint32_t st_len[kBulkStages];
  uint32_t cur = list.seek(t0);  // load-side cursor
  uint32_t next_load = 0;        // chunks issued so far
  auto issue_load = [&]() {
    const uint32_t k = next_load++;
    uint64_t src, dst;
    uint32_t n;
    list.get(cur, t0 + k, kBulkShift, &src, &dst, &n);
    const int s = int(k % kBulkStages);
    st_dst[s] = dst;
    st_len[s] = n;
    bulk_load(buf0 + s * kBulkChunk, reinterpret_cast<const void*>(src), n, bar0 + 8 * s);
  };

  while (next_load < T && next_load < uint32_t(kBulkStages)) issue_load();
  bool ok = true;
  uint32_t k = 0;
  for (; k < T; ++k) {
    const int s = int(k % kBulkStages);
    if (!mbar_wait(bar0 + 8 * s, (k / kBulkStages) & 1u)) {
      ok = false;
      break;
    }
    bulk_store(reinterpret_cast<void*>(st_dst[s]), buf0 + s * kBulkChunk, st_len[s]);
    // Refill the stage of chunk k-1 once its store has read shared memory
    // (every bulk group but the newest, store k, has finished reading).
    if (k >= 1 && next_load < T) {
      bulk_wait_read_le1();
      issue_load();
    }
  }
  bulk_wait_all();
  if (!ok) {
    atomicExch(&g_kvx_device_status, 8 /* KVX_ERR_DEVICE_TIMEOUT */);
    // Let the loads still in flight into shared memory land, bounded.
    for (uint32_t j = k; j < next_load; ++j)
      if (!mbar_wait(bar0 + 8 * int(j % kBulkStages), (j / kBulkStages) & 1u)) break;
  }
}

}  // namespace kvx
