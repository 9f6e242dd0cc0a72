// Host-side planning for KV-block movement: validation, extent arithmetic,
// ordering ("waves"), coalescing and work-item tables for the copy kernels.
// Pure C++ (no CUDA calls), so every rule here is testable without a GPU.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "kvx_worklist.h"

namespace kvx {

// One byte-range copy. Addresses are absolute (device-visible for the kernel
// path, or the caller's host address for the copy-engine path).
struct Copy {
  uint64_t src;
  uint64_t dst;
  uint64_t len;
};

// Work item read by the copy kernels: a copy with the index of its first tile
// in the launch-wide tile sequence.  24 bytes, 8-byte aligned.
struct Item {
  uint64_t src;
  uint64_t dst;
  uint32_t len;         // bytes, <= kMaxItemBytes
  uint32_t tile_begin;  // first tile of this item
};
static_assert(sizeof(Item) == 24, "Item must stay 24 bytes");

constexpr uint64_t kMaxItemBytes = 1ull << 30;

struct Error {
  int code = 0;
  std::string msg;
  bool ok() const { return code == 0; }
};

// Layout of one GPU's composite KV block and its host pool (see kvx.h).
struct Layout {
  int device = 0;
  std::vector<uint64_t> seg_pages;       // device address of page 0
  std::vector<uint64_t> seg_page_bytes;
  std::vector<uint64_t> seg_num_blocks;
  std::vector<uint64_t> seg_cpu_offset;
  std::vector<uint64_t> seg_owner_mask;
  std::vector<int64_t> group_ratio;      // kernel blocks per physical block
  uint64_t host_pool = 0;                // caller's host address (0: none)
  uint64_t host_pool_dev = 0;            // device-visible address (0: not mapped)
  uint64_t host_pool_bytes = 0;
  uint64_t host_row_bytes = 0;
  uint64_t host_row_offset = 0;
  uint64_t host_num_rows = 0;
};

Error validate_layout(const Layout& L);

// a3: byte_extent_for_kernel_blocks (cache_transfer.py:113-165).
Error byte_extent(uint64_t page_bytes, int64_t kernel_blocks_per_page,
                  int64_t first, int64_t count, uint64_t* off, uint64_t* len);

struct Entries {
  int64_t n = 0;
  const int64_t* src = nullptr;
  const int64_t* dst = nullptr;
  const int64_t* group = nullptr;
  const int64_t* first = nullptr;
  const int64_t* valid = nullptr;
};

enum class Side { kDevice, kHost };

// Copies of a segmented swap in the reference's issue order (segment-major,
// then entry order; worker.py:2272-2329).  Host addresses use `host_base`
// (the caller's host address or the device-mapped one).
Error plan_swap_blocks(const Layout& L, const Entries& e, bool is_swap_in,
                       uint64_t host_base, std::vector<Copy>* out,
                       uint64_t* copied_bytes);

// Copies of a GPU->GPU migration between two layouts with equal segment
// tables.  Issue order as above.
Error plan_migrate(const Layout& S, const Layout& T, const Entries& e,
                   std::vector<Copy>* out, uint64_t* copied_bytes);

// a1: per-tensor swap (ops/swap.cu:34-58).
Error plan_swap(const int64_t* src_ids, const int64_t* dst_ids, int64_t n,
                bool is_swap_in, uint64_t cache, uint64_t cache_bytes,
                uint64_t block_bytes, uint64_t swap, uint64_t swap_bytes,
                std::vector<Copy>* out);

// Split an ordered copy list into consecutive waves such that, inside a
// wave, no copy's destination overlaps another copy's source or destination.
// Running the waves in order with full parallelism inside each reproduces the
// bytes of executing the list sequentially.  Returns wave end indices.
std::vector<size_t> split_waves(const std::vector<Copy>& copies);

// Merge neighbours that are contiguous on both sides (in list order).
void coalesce(std::vector<Copy>* copies);

// Build the kernel item table for `copies` with the given tile size (power of
// two).  Copies longer than kMaxItemBytes are split.  Returns the tile count.
uint64_t build_items(const std::vector<Copy>& copies, uint32_t tile_bytes,
                     std::vector<Item>* items);

// Copy-engine staging plan for one direction.  `host_is_src` selects whether
// the host side is the source (swap-in) or destination (swap-out).  The copies
// are reordered by host address and cut into chunks of at most
// staging_bytes; within a chunk staging offsets follow host order.
struct StagedChunk {
  std::vector<Copy> device_moves;  // device <-> staging (staging as offsets)
  std::vector<Copy> host_runs;     // host <-> staging (staging as offsets)
  uint64_t bytes = 0;
};
void plan_staged(const std::vector<Copy>& copies, bool host_is_src,
                 uint64_t staging_bytes, std::vector<StagedChunk>* chunks);

// Mean length of host-contiguous runs (after sorting by host address).
uint64_t mean_host_run(const std::vector<Copy>& copies, bool host_is_src);

// ---- grid plans (entries x segments expanded on the device) ----------------
// A grid plan exists when every segment has the same page size, every
// segment is owned by every cache group the entries use, the target ids of
// the copying entries are distinct and the source and destination memory do
// not overlap.  Then no two copies conflict and host work is O(entries).
// The grid_* builders return false when those conditions do not hold or any
// check fails: the item planner then runs and reports the canonical error.
struct GridPlan {
  std::vector<GridEntry> entries;
  std::vector<GridSeg> segs;
  uint64_t copied = 0;   // payload bytes
  uint64_t extents = 0;  // entry x segment copies
  // Host side, for swaps (0 for migrations): 1 = source, 2 = destination.
  int host_side = 0;
  uint64_t row_base = 0;    // host address of row 0 of this GPU's bytes
  uint64_t row_stride = 0;  // host row pitch
  uint64_t row_span = 0;    // S * page when every entry writes its whole,
                            // gap-free composite span (copy-engine staging), else 0
};

bool grid_swap_blocks(const Layout& L, const Entries& e, bool is_swap_in,
                      uint64_t host_base, GridPlan* out);
bool grid_migrate(const Layout& S, const Layout& T, const Entries& e, GridPlan* out);
bool grid_swap(const int64_t* src_ids, const int64_t* dst_ids, int64_t n, bool is_swap_in,
               uint64_t cache, uint64_t cache_bytes, uint64_t block_bytes, uint64_t swap,
               uint64_t swap_bytes, GridPlan* out);

// Fill tile_begin / tiles_per_seg for a tile size of 1 << tile_shift and
// return the tile count (> 0xffffffff: too large for one launch).
uint64_t grid_finalize(GridPlan* p, uint32_t tile_shift);

// The copies a finalized grid plan performs, tile by tile, through the same
// resolver the kernels use (host emulation; tiles of one copy are merged).
void grid_expand(const GridPlan& p, uint32_t tile_shift, std::vector<Copy>* out);

}  // namespace kvx
