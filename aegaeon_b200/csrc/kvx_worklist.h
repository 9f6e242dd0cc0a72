// Work lists of the copy kernels, shared by device code and host code.
//
// A launch moves a sequence of tiles.  Two encodings of that sequence exist:
//
//  * item list  : one record per contiguous copy (kvx::Item); used for any
//                 request, in particular ones with overlapping destinations
//                 (ordered waves), mixed page sizes or partial host runs.
//  * grid list  : one record per entry (a block id pair with its live byte
//                 extent) plus a table of segments (base and stride of the
//                 source and destination side).  The copy of entry e in
//                 segment s is
//                    src = seg[s].src_base + e.src_id * seg[s].src_stride + e.off
//                    dst = seg[s].dst_base + e.dst_id * seg[s].dst_stride + e.off
//                 over e.len bytes.  Host planning is O(entries + segments)
//                 instead of O(entries x segments); the kernel expands it.
//
// Tiles of a grid entry run segment after segment (entry-major), so one CTA
// writes a host row front to back.  The resolvers below are the only place
// that maps a tile to addresses; the host uses the same functions to expand a
// plan for tests.
#pragma once

#include <cstdint>

#ifdef __CUDACC__
#define KVX_HD __host__ __device__ __forceinline__
#else
#define KVX_HD inline
#endif

namespace kvx {

struct GridEntry {
  int64_t src_id;
  int64_t dst_id;
  uint32_t off;            // byte offset of the live extent inside a page
  uint32_t len;            // bytes of the live extent (> 0)
  uint32_t tile_begin;     // first tile of this entry
  uint32_t tiles_per_seg;  // ceil(len / tile)
};
static_assert(sizeof(GridEntry) == 32, "GridEntry must stay 32 bytes");

struct GridSeg {
  uint64_t src_base;
  uint64_t src_stride;
  uint64_t dst_base;
  uint64_t dst_stride;
};
static_assert(sizeof(GridSeg) == 32, "GridSeg must stay 32 bytes");

// Largest i with e[i].tile_begin <= t (e sorted by tile_begin, e[0] starts at 0).
KVX_HD uint32_t grid_find(const GridEntry* e, uint32_t n, uint32_t t) {
  uint32_t lo = 0, hi = n - 1;
  while (lo < hi) {
    const uint32_t mid = (lo + hi + 1) >> 1;
    if (e[mid].tile_begin <= t)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

// Addresses and length of tile t of entry `en` (t inside the entry's range).
KVX_HD void grid_resolve(const GridEntry& en, const GridSeg* segs, uint32_t t,
                         uint32_t tile_shift, uint64_t* src, uint64_t* dst,
                         uint32_t* len) {
  const uint32_t local = t - en.tile_begin;
  const uint32_t s = local / en.tiles_per_seg;
  const uint32_t c = local - s * en.tiles_per_seg;
  const uint32_t done = c << tile_shift;
  const uint32_t left = en.len - done;
  const uint32_t tile = 1u << tile_shift;
  *len = left < tile ? left : tile;
  const GridSeg g = segs[s];
  *src = g.src_base + uint64_t(en.src_id) * g.src_stride + en.off + done;
  *dst = g.dst_base + uint64_t(en.dst_id) * g.dst_stride + en.off + done;
}

}  // namespace kvx
