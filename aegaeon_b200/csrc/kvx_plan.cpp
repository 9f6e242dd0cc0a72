// Host-side planning for KV-block movement.  See kvx_plan.h.
//
// The rules below restate, in C++, the validation and address arithmetic of
// the reference's swap path:
//   * per-tensor swap            ops/swap.cu:34-58
//   * segmented swap loop        aegaeon/worker.py:2230-2329
//   * extent arithmetic          aegaeon/cache_transfer.py:113-165
// Validation is complete before any copy is produced: a failing request
// yields no copies at all (the reference raises midway through its loop, after
// some copies were already queued).
#include "kvx_plan.h"

#include <algorithm>
#include <cstdio>
#include <iterator>
#include <map>
#include <numeric>

namespace kvx {
namespace {

constexpr int64_t kIdLimit = int64_t(1) << 48;  // keeps all products in range

Error fail(int code, const char* fmt, long long a = 0, long long b = 0,
           long long c = 0) {
  char buf[320];
  std::snprintf(buf, sizeof(buf), fmt, a, b, c);
  Error e;
  e.code = code;
  e.msg = buf;
  return e;
}

// kvx.h status codes (kept numeric here so this file needs no CUDA header).
constexpr int kInvalid = 1, kGroup = 3, kExtent = 4, kBlockId = 5,
              kHostMemory = 6, kLayoutMismatch = 9;

// prefix_bytes_for_kernel_blocks, cache_transfer.py:113-135.
Error prefix_bytes(uint64_t page, int64_t ratio, int64_t valid, uint64_t* out) {
  if (page == 0) return fail(kExtent, "page_size_bytes must be positive, got 0");
  if (ratio <= 0)
    return fail(kExtent, "kernel_blocks_per_page must be positive, got %lld",
                ratio);
  if (valid < 0 || valid > ratio)
    return fail(kExtent, "valid kernel blocks %lld outside [0, %lld]", valid,
                ratio);
  if (page % uint64_t(ratio))
    return fail(kExtent,
                "Backing page size %lld is not divisible by %lld kernel blocks",
                (long long)page, ratio);
  *out = page / uint64_t(ratio) * uint64_t(valid);
  return Error{};
}

}  // namespace

// byte_extent_for_kernel_blocks, cache_transfer.py:138-165 (same check order).
Error byte_extent(uint64_t page_bytes, int64_t ratio, int64_t first,
                  int64_t count, uint64_t* off, uint64_t* len) {
  if (first < 0)
    return fail(kExtent, "first_kernel_block must be non-negative, got %lld",
                first);
  if (first > kIdLimit || count > kIdLimit || count < -kIdLimit)
    return fail(kExtent, "kernel-block extent [%lld, +%lld) out of range",
                first, count);
  const int64_t end = first + count;
  if (end > ratio)
    return fail(kExtent, "Kernel-block extent [%lld, %lld) exceeds page size %lld",
                first, end, ratio);
  Error e = prefix_bytes(page_bytes, ratio, first, off);
  if (!e.ok()) return e;
  return prefix_bytes(page_bytes, ratio, count, len);
}

Error validate_layout(const Layout& L) {
  const size_t ns = L.seg_pages.size();
  if (L.seg_page_bytes.size() != ns || L.seg_num_blocks.size() != ns ||
      L.seg_cpu_offset.size() != ns || L.seg_owner_mask.size() != ns)
    return fail(kInvalid, "segment tables differ in length");
  const size_t ng = L.group_ratio.size();
  if (ng > 64) return fail(kInvalid, "at most 64 cache groups, got %lld", ng);
  for (size_t g = 0; g < ng; ++g)
    if (L.group_ratio[g] <= 0 || L.group_ratio[g] > kIdLimit)
      return fail(kInvalid, "group %lld: kernel blocks per block must be positive, got %lld",
                  (long long)g, L.group_ratio[g]);
  const uint64_t valid_mask = ng == 64 ? ~0ull : ((1ull << ng) - 1);
  for (size_t s = 0; s < ns; ++s) {
    if (L.seg_page_bytes[s] == 0)
      return fail(kInvalid, "segment %lld: page size must be positive", (long long)s);
    if (L.seg_pages[s] == 0 && L.seg_num_blocks[s] != 0)
      return fail(kInvalid, "segment %lld: null page pointer", (long long)s);
    if (L.seg_num_blocks[s] > uint64_t(kIdLimit) ||
        L.seg_page_bytes[s] > (1ull << 40))
      return fail(kInvalid, "segment %lld: size out of range", (long long)s);
    const uint64_t m = L.seg_owner_mask[s];
    if (m == 0)
      return fail(kInvalid, "Cache segment %lld is not owned by any KV-cache group",
                  (long long)s);
    if (m & ~valid_mask)
      return fail(kInvalid, "segment %lld: owner mask names a group >= %lld",
                  (long long)s, (long long)ng);
    if (L.host_pool) {
      const uint64_t end = L.host_row_offset + L.seg_cpu_offset[s] + L.seg_page_bytes[s];
      if (end > L.host_row_bytes)
        return fail(kInvalid,
                    "segment %lld: host bytes end at %lld, beyond the %lld-byte row",
                    (long long)s, (long long)end, (long long)L.host_row_bytes);
    }
  }
  if (L.host_pool) {
    if (L.host_row_bytes == 0) return fail(kInvalid, "host_row_bytes must be positive");
    if (L.host_num_rows != L.host_pool_bytes / L.host_row_bytes)
      return fail(kInvalid, "host row count inconsistent with the pool size");
  }
  return Error{};
}

namespace {

Error check_groups(const Layout& L, const Entries& e) {
  if (e.n < 0) return fail(kInvalid, "negative entry count %lld", e.n);
  if (e.n > 0 && (!e.src || !e.dst || !e.group || !e.first || !e.valid))
    return fail(kInvalid, "null entry array");
  const int64_t ng = int64_t(L.group_ratio.size());
  for (int64_t i = 0; i < e.n; ++i)  // worker.py:2244-2246, before any copy
    if (e.group[i] < 0 || e.group[i] >= ng)
      return fail(kGroup, "Invalid swap cache-group id %lld", e.group[i]);
  return Error{};
}

}  // namespace

Error plan_swap_blocks(const Layout& L, const Entries& e, bool is_swap_in,
                       uint64_t host_base, std::vector<Copy>* out,
                       uint64_t* copied_bytes) {
  out->clear();
  uint64_t copied = 0;
  if (!L.host_pool || !host_base)
    return fail(kHostMemory, "layout has no host pool");
  Error err = check_groups(L, e);
  if (!err.ok()) return err;
  const size_t ns = L.seg_pages.size();
  out->reserve(ns * size_t(e.n));
  for (size_t s = 0; s < ns; ++s) {
    const uint64_t page = L.seg_page_bytes[s];
    const uint64_t owners = L.seg_owner_mask[s];
    for (int64_t i = 0; i < e.n; ++i) {
      const int64_t g = e.group[i];
      if (!((owners >> g) & 1)) continue;  // worker.py:2292-2293
      uint64_t off = 0, len = 0;
      err = byte_extent(page, L.group_ratio[g], e.first[i], e.valid[i], &off, &len);
      if (!err.ok()) return err;
      if (len == 0) continue;  // worker.py:2300-2301
      const int64_t dev_id = is_swap_in ? e.dst[i] : e.src[i];
      const int64_t row = is_swap_in ? e.src[i] : e.dst[i];
      if (dev_id < 0 || uint64_t(dev_id) >= L.seg_num_blocks[s])
        return fail(kBlockId, "GPU block id %lld outside [0, %lld) of segment %lld",
                    dev_id, (long long)L.seg_num_blocks[s], (long long)s);
      if (row < 0 || uint64_t(row) >= L.host_num_rows)
        return fail(kBlockId, "CPU block id %lld outside [0, %lld)", row,
                    (long long)L.host_num_rows);
      const uint64_t dev = L.seg_pages[s] + uint64_t(dev_id) * page + off;
      const uint64_t host = host_base + uint64_t(row) * L.host_row_bytes +
                            L.host_row_offset + L.seg_cpu_offset[s] + off;
      out->push_back(is_swap_in ? Copy{host, dev, len} : Copy{dev, host, len});
      copied += len;
    }
  }
  if (copied_bytes) *copied_bytes = copied;
  return Error{};
}

Error plan_migrate(const Layout& S, const Layout& T, const Entries& e,
                   std::vector<Copy>* out, uint64_t* copied_bytes) {
  out->clear();
  uint64_t copied = 0;
  const size_t ns = S.seg_pages.size();
  if (T.seg_pages.size() != ns)
    return fail(kLayoutMismatch, "source has %lld segments, target %lld",
                (long long)ns, (long long)T.seg_pages.size());
  if (S.group_ratio != T.group_ratio)
    return fail(kLayoutMismatch, "cache-group tables differ");
  for (size_t s = 0; s < ns; ++s)
    if (S.seg_page_bytes[s] != T.seg_page_bytes[s] ||
        S.seg_owner_mask[s] != T.seg_owner_mask[s])
      return fail(kLayoutMismatch, "segment %lld differs between the layouts",
                  (long long)s);
  Error err = check_groups(S, e);
  if (!err.ok()) return err;
  for (size_t s = 0; s < ns; ++s) {
    const uint64_t page = S.seg_page_bytes[s];
    const uint64_t owners = S.seg_owner_mask[s];
    for (int64_t i = 0; i < e.n; ++i) {
      const int64_t g = e.group[i];
      if (!((owners >> g) & 1)) continue;
      uint64_t off = 0, len = 0;
      err = byte_extent(page, S.group_ratio[g], e.first[i], e.valid[i], &off, &len);
      if (!err.ok()) return err;
      if (len == 0) continue;
      if (e.src[i] < 0 || uint64_t(e.src[i]) >= S.seg_num_blocks[s])
        return fail(kBlockId, "source block id %lld outside [0, %lld) of segment %lld",
                    e.src[i], (long long)S.seg_num_blocks[s], (long long)s);
      if (e.dst[i] < 0 || uint64_t(e.dst[i]) >= T.seg_num_blocks[s])
        return fail(kBlockId, "target block id %lld outside [0, %lld) of segment %lld",
                    e.dst[i], (long long)T.seg_num_blocks[s], (long long)s);
      out->push_back(Copy{S.seg_pages[s] + uint64_t(e.src[i]) * page + off,
                          T.seg_pages[s] + uint64_t(e.dst[i]) * page + off, len});
      copied += len;
    }
  }
  if (copied_bytes) *copied_bytes = copied;
  return Error{};
}

Error plan_swap(const int64_t* src_ids, const int64_t* dst_ids, int64_t n,
                bool is_swap_in, uint64_t cache, uint64_t cache_bytes,
                uint64_t block_bytes, uint64_t swap, uint64_t swap_bytes,
                std::vector<Copy>* out) {
  out->clear();
  if (n < 0) return fail(kInvalid, "negative id count %lld", n);
  if (n > 0 && (!src_ids || !dst_ids)) return fail(kInvalid, "null id array");
  if (n > 0 && block_bytes > 0 && (!cache || !swap))
    return fail(kInvalid, "null kv_cache or kv_swap");
  if (block_bytes == 0) return Error{};  // zero-byte copies: nothing to do
  const uint64_t cache_blocks = cache_bytes / block_bytes;
  const uint64_t swap_blocks = swap_bytes / block_bytes;
  out->reserve(size_t(n));
  for (int64_t i = 0; i < n; ++i) {
    const int64_t dev_id = is_swap_in ? dst_ids[i] : src_ids[i];
    const int64_t slot = is_swap_in ? src_ids[i] : dst_ids[i];
    if (dev_id < 0 || uint64_t(dev_id) >= cache_blocks)
      return fail(kBlockId, "kv_cache block id %lld outside [0, %lld)", dev_id,
                  (long long)cache_blocks);
    if (slot < 0 || uint64_t(slot) >= swap_blocks)
      return fail(kBlockId, "kv_swap block id %lld outside [0, %lld)", slot,
                  (long long)swap_blocks);
    const uint64_t d = cache + uint64_t(dev_id) * block_bytes;
    const uint64_t h = swap + uint64_t(slot) * block_bytes;
    out->push_back(is_swap_in ? Copy{h, d, block_bytes} : Copy{d, h, block_bytes});
  }
  return Error{};
}

namespace {

// Disjoint interval set keyed by start.
struct IntervalSet {
  std::map<uint64_t, uint64_t> iv;  // start -> end
  bool overlaps(uint64_t b, uint64_t e) const {
    if (b >= e) return false;
    auto it = iv.upper_bound(b);
    if (it != iv.begin()) {
      auto p = std::prev(it);
      if (p->second > b) return true;
    }
    return it != iv.end() && it->first < e;
  }
  void insert(uint64_t b, uint64_t e) {  // merges with neighbours
    if (b >= e) return;
    auto it = iv.upper_bound(b);
    if (it != iv.begin()) {
      auto p = std::prev(it);
      if (p->second >= b) {
        b = p->first;
        e = std::max(e, p->second);
        it = iv.erase(p);
      }
    }
    while (it != iv.end() && it->first <= e) {
      e = std::max(e, it->second);
      it = iv.erase(it);
    }
    iv.emplace(b, e);
  }
  void clear() { iv.clear(); }
};

}  // namespace

std::vector<size_t> split_waves(const std::vector<Copy>& copies) {
  std::vector<size_t> ends;
  const size_t n = copies.size();
  if (n == 0) return ends;
  // Fast path: destinations pairwise disjoint and the source / destination
  // hulls disjoint -> a single wave.
  uint64_t smin = ~0ull, smax = 0, dmin = ~0ull, dmax = 0;
  for (const Copy& c : copies) {
    if (c.len == 0) continue;
    smin = std::min(smin, c.src);
    smax = std::max(smax, c.src + c.len);
    dmin = std::min(dmin, c.dst);
    dmax = std::max(dmax, c.dst + c.len);
  }
  const bool hulls_disjoint = smax <= dmin || dmax <= smin;
  if (hulls_disjoint) {
    std::vector<size_t> order(n);
    std::iota(order.begin(), order.end(), size_t(0));
    std::sort(order.begin(), order.end(), [&](size_t a, size_t b) {
      return copies[a].dst < copies[b].dst;
    });
    bool clash = false;
    uint64_t reach = 0;
    bool any = false;
    for (size_t k : order) {
      const Copy& c = copies[k];
      if (c.len == 0) continue;
      if (any && c.dst < reach) { clash = true; break; }
      reach = std::max(reach, c.dst + c.len);
      any = true;
    }
    if (!clash) { ends.push_back(n); return ends; }
  }
  IntervalSet wdst, wsrc;
  for (size_t i = 0; i < n; ++i) {
    const Copy& c = copies[i];
    const uint64_t sb = c.src, se = c.src + c.len, db = c.dst, de = c.dst + c.len;
    if (wdst.overlaps(db, de) || wdst.overlaps(sb, se) || wsrc.overlaps(db, de)) {
      ends.push_back(i);
      wdst.clear();
      wsrc.clear();
    }
    wdst.insert(db, de);
    wsrc.insert(sb, se);
  }
  ends.push_back(n);
  return ends;
}

void coalesce(std::vector<Copy>* copies) {
  std::vector<Copy>& v = *copies;
  size_t w = 0;
  for (size_t i = 0; i < v.size(); ++i) {
    if (v[i].len == 0) continue;
    if (w > 0 && v[w - 1].src + v[w - 1].len == v[i].src &&
        v[w - 1].dst + v[w - 1].len == v[i].dst) {
      v[w - 1].len += v[i].len;
    } else {
      v[w++] = v[i];
    }
  }
  v.resize(w);
}

uint64_t build_items(const std::vector<Copy>& copies, uint32_t tile_bytes,
                     std::vector<Item>* items) {
  items->clear();
  uint64_t tiles = 0;
  for (const Copy& c : copies) {
    uint64_t done = 0;
    while (done < c.len) {
      const uint64_t len = std::min<uint64_t>(c.len - done, kMaxItemBytes);
      Item it;
      it.src = c.src + done;
      it.dst = c.dst + done;
      it.len = uint32_t(len);
      it.tile_begin = uint32_t(tiles);
      items->push_back(it);
      tiles += (len + tile_bytes - 1) / tile_bytes;
      done += len;
    }
  }
  return tiles;
}

namespace {
inline uint64_t host_addr(const Copy& c, bool host_is_src) {
  return host_is_src ? c.src : c.dst;
}
inline uint64_t dev_addr(const Copy& c, bool host_is_src) {
  return host_is_src ? c.dst : c.src;
}
}  // namespace

void plan_staged(const std::vector<Copy>& copies, bool host_is_src,
                 uint64_t staging_bytes, std::vector<StagedChunk>* chunks) {
  chunks->clear();
  std::vector<size_t> order(copies.size());
  std::iota(order.begin(), order.end(), size_t(0));
  std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) {
    return host_addr(copies[a], host_is_src) < host_addr(copies[b], host_is_src);
  });
  StagedChunk cur;
  auto flush = [&]() {
    if (cur.bytes) {
      coalesce(&cur.device_moves);
      chunks->push_back(std::move(cur));
    }
    cur = StagedChunk{};
  };
  for (size_t k : order) {
    const Copy& c = copies[k];
    uint64_t h = host_addr(c, host_is_src), d = dev_addr(c, host_is_src);
    uint64_t left = c.len;
    while (left) {
      if (cur.bytes == staging_bytes) flush();
      const uint64_t take = std::min(left, staging_bytes - cur.bytes);
      const uint64_t pos = cur.bytes;
      if (host_is_src) {
        cur.device_moves.push_back(Copy{pos, d, take});
        if (!cur.host_runs.empty() &&
            cur.host_runs.back().src + cur.host_runs.back().len == h &&
            cur.host_runs.back().dst + cur.host_runs.back().len == pos)
          cur.host_runs.back().len += take;
        else
          cur.host_runs.push_back(Copy{h, pos, take});
      } else {
        cur.device_moves.push_back(Copy{d, pos, take});
        if (!cur.host_runs.empty() &&
            cur.host_runs.back().dst + cur.host_runs.back().len == h &&
            cur.host_runs.back().src + cur.host_runs.back().len == pos)
          cur.host_runs.back().len += take;
        else
          cur.host_runs.push_back(Copy{pos, h, take});
      }
      cur.bytes += take;
      h += take;
      d += take;
      left -= take;
    }
  }
  flush();
}

uint64_t mean_host_run(const std::vector<Copy>& copies, bool host_is_src) {
  if (copies.empty()) return 0;
  std::vector<std::pair<uint64_t, uint64_t>> hv;
  hv.reserve(copies.size());
  uint64_t total = 0;
  for (const Copy& c : copies) {
    if (!c.len) continue;
    hv.emplace_back(host_addr(c, host_is_src), c.len);
    total += c.len;
  }
  if (hv.empty()) return 0;
  std::sort(hv.begin(), hv.end());
  uint64_t runs = 1;
  for (size_t i = 1; i < hv.size(); ++i)
    if (hv[i - 1].first + hv[i - 1].second != hv[i].first) ++runs;
  return total / runs;
}

namespace {

struct Range {
  uint64_t b, e;
};

// True when no range of `a` intersects a range of `b`.
bool disjoint_sets(std::vector<Range> a, std::vector<Range> b) {
  auto by_begin = [](const Range& x, const Range& y) { return x.b < y.b; };
  std::sort(a.begin(), a.end(), by_begin);
  std::sort(b.begin(), b.end(), by_begin);
  size_t i = 0, j = 0;
  while (i < a.size() && j < b.size()) {
    if (a[i].b >= a[i].e) { ++i; continue; }
    if (b[j].b >= b[j].e) { ++j; continue; }
    if (a[i].b < b[j].e && b[j].b < a[i].e) return false;
    if (a[i].e <= b[j].e) ++i; else ++j;
  }
  return true;
}

bool unique_ids(std::vector<int64_t> ids) {
  std::sort(ids.begin(), ids.end());
  return std::adjacent_find(ids.begin(), ids.end()) == ids.end();
}

// True when no two non-empty ranges of `a` intersect.
bool pairwise_disjoint(std::vector<Range> a) {
  std::sort(a.begin(), a.end(), [](const Range& x, const Range& y) { return x.b < y.b; });
  uint64_t end = 0;
  bool any = false;
  for (const Range& r : a) {
    if (r.b >= r.e) continue;
    if (any && r.b < end) return false;
    end = any ? std::max(end, r.e) : r.e;
    any = true;
  }
  return true;
}

// Entry-level checks shared by the segmented grid builders: uniform page,
// owners, groups, extents.  Fills out->entries (ids raw, extents set) and
// returns false when the grid form does not apply.
bool grid_entries(const Layout& L, const Entries& e, GridPlan* out, uint64_t* page_out) {
  const size_t ns = L.seg_pages.size();
  if (ns == 0 || e.n < 0 || (e.n > 0 && (!e.src || !e.dst || !e.group || !e.first || !e.valid)))
    return false;
  const uint64_t page = L.seg_page_bytes[0];
  if (page == 0 || page >= (1ull << 32)) return false;
  uint64_t common_owners = ~0ull;
  for (size_t s = 0; s < ns; ++s) {
    if (L.seg_page_bytes[s] != page) return false;
    common_owners &= L.seg_owner_mask[s];
  }
  const int64_t ng = int64_t(L.group_ratio.size());
  out->entries.clear();
  out->entries.reserve(size_t(e.n));
  for (int64_t i = 0; i < e.n; ++i) {
    const int64_t g = e.group[i];
    if (g < 0 || g >= ng) return false;
    if (!((common_owners >> g) & 1)) return false;  // some segment skips this group
    uint64_t off = 0, len = 0;
    if (!byte_extent(page, L.group_ratio[g], e.first[i], e.valid[i], &off, &len).ok()) return false;
    if (len == 0) continue;
    GridEntry ge{e.src[i], e.dst[i], uint32_t(off), uint32_t(len), 0, 0};
    out->entries.push_back(ge);
  }
  *page_out = page;
  return true;
}

bool ids_in(const std::vector<GridEntry>& v, bool src, uint64_t limit) {
  for (const GridEntry& g : v) {
    const int64_t id = src ? g.src_id : g.dst_id;
    if (id < 0 || uint64_t(id) >= limit) return false;
  }
  return true;
}

uint64_t min_blocks(const Layout& L) {
  uint64_t m = ~0ull;
  for (uint64_t b : L.seg_num_blocks) m = std::min(m, b);
  return m;
}

std::vector<Range> page_ranges(const Layout& L) {
  std::vector<Range> r;
  for (size_t s = 0; s < L.seg_pages.size(); ++s)
    r.push_back(Range{L.seg_pages[s], L.seg_pages[s] + L.seg_page_bytes[s] * L.seg_num_blocks[s]});
  return r;
}

std::vector<int64_t> dst_ids(const std::vector<GridEntry>& v) {
  std::vector<int64_t> d;
  d.reserve(v.size());
  for (const GridEntry& g : v) d.push_back(g.dst_id);
  return d;
}

// True when no block id is both a source and a target of the entries.
bool sources_not_targets(const std::vector<GridEntry>& v) {
  std::vector<int64_t> src;
  src.reserve(v.size());
  for (const GridEntry& g : v) src.push_back(g.src_id);
  std::vector<int64_t> dst = dst_ids(v);
  std::sort(src.begin(), src.end());
  std::sort(dst.begin(), dst.end());
  size_t i = 0, j = 0;
  while (i < src.size() && j < dst.size()) {
    if (src[i] == dst[j]) return false;
    if (src[i] < dst[j]) ++i; else ++j;
  }
  return true;
}

}  // namespace

bool grid_swap_blocks(const Layout& L, const Entries& e, bool is_swap_in, uint64_t host_base,
                      GridPlan* out) {
  if (!L.host_pool || !host_base) return false;
  uint64_t page = 0;
  if (!grid_entries(L, e, out, &page)) return false;
  const uint64_t dev_limit = min_blocks(L);
  if (!ids_in(out->entries, !is_swap_in, dev_limit)) return false;
  if (!ids_in(out->entries, is_swap_in, L.host_num_rows)) return false;
  if (!unique_ids(dst_ids(out->entries))) return false;
  const std::vector<Range> dev = page_ranges(L);
  const std::vector<Range> host{Range{host_base, host_base + L.host_pool_bytes}};
  if (!disjoint_sets(dev, host)) return false;
  const size_t ns = L.seg_pages.size();
  out->segs.clear();
  const uint64_t row_base = host_base + L.host_row_offset;
  for (size_t s = 0; s < ns; ++s) {
    const uint64_t hb = row_base + L.seg_cpu_offset[s];
    if (is_swap_in)
      out->segs.push_back(GridSeg{hb, L.host_row_bytes, L.seg_pages[s], page});
    else
      out->segs.push_back(GridSeg{L.seg_pages[s], page, hb, L.host_row_bytes});
  }
  out->host_side = is_swap_in ? 1 : 2;
  out->row_base = row_base;
  out->row_stride = L.host_row_bytes;
  // Whole, gap-free spans: full pages and cpu offsets tiling [0, S*page).
  bool full = true;
  for (const GridEntry& g : out->entries)
    if (g.off != 0 || g.len != page) { full = false; break; }
  if (full) {
    std::vector<uint64_t> offs(L.seg_cpu_offset);
    std::sort(offs.begin(), offs.end());
    for (size_t s = 0; s < ns && full; ++s) full = offs[s] == s * page;
  }
  out->row_span = full ? ns * page : 0;
  out->extents = out->entries.size() * ns;
  out->copied = 0;
  for (const GridEntry& g : out->entries) out->copied += uint64_t(g.len) * ns;
  return true;
}

bool grid_migrate(const Layout& S, const Layout& T, const Entries& e, GridPlan* out) {
  const size_t ns = S.seg_pages.size();
  if (T.seg_pages.size() != ns || S.group_ratio != T.group_ratio) return false;
  for (size_t s = 0; s < ns; ++s)
    if (S.seg_page_bytes[s] != T.seg_page_bytes[s] || S.seg_owner_mask[s] != T.seg_owner_mask[s])
      return false;
  uint64_t page = 0;
  if (!grid_entries(S, e, out, &page)) return false;
  if (!ids_in(out->entries, true, min_blocks(S))) return false;
  if (!ids_in(out->entries, false, min_blocks(T))) return false;
  if (!unique_ids(dst_ids(out->entries))) return false;
  if (!disjoint_sets(page_ranges(S), page_ranges(T))) {
    // Both sides are the same cache (block copies inside one GPU's cache):
    // still one grid when its segments do not alias each other and no block
    // is both read and written, so that no copy reads bytes another writes
    // and any order of the copies gives the sequential result.
    if (S.seg_pages != T.seg_pages || S.seg_num_blocks != T.seg_num_blocks ||
        !pairwise_disjoint(page_ranges(S)) || !sources_not_targets(out->entries))
      return false;
  }
  out->segs.clear();
  for (size_t s = 0; s < ns; ++s)
    out->segs.push_back(GridSeg{S.seg_pages[s], page, T.seg_pages[s], page});
  out->host_side = 0;
  out->row_base = out->row_stride = out->row_span = 0;
  out->extents = out->entries.size() * ns;
  out->copied = 0;
  for (const GridEntry& g : out->entries) out->copied += uint64_t(g.len) * ns;
  return true;
}

bool grid_swap(const int64_t* src_ids, const int64_t* dst_ids_, int64_t n, bool is_swap_in,
               uint64_t cache, uint64_t cache_bytes, uint64_t block_bytes, uint64_t swap,
               uint64_t swap_bytes, GridPlan* out) {
  if (n < 0 || (n > 0 && (!src_ids || !dst_ids_)) || block_bytes == 0 ||
      block_bytes >= (1ull << 32) || !cache || !swap)
    return false;
  const uint64_t cache_blocks = cache_bytes / block_bytes;
  const uint64_t swap_blocks = swap_bytes / block_bytes;
  out->entries.clear();
  out->entries.reserve(size_t(n));
  for (int64_t i = 0; i < n; ++i) {
    const int64_t dev = is_swap_in ? dst_ids_[i] : src_ids[i];
    const int64_t slot = is_swap_in ? src_ids[i] : dst_ids_[i];
    if (dev < 0 || uint64_t(dev) >= cache_blocks) return false;
    if (slot < 0 || uint64_t(slot) >= swap_blocks) return false;
    out->entries.push_back(GridEntry{src_ids[i], dst_ids_[i], 0, uint32_t(block_bytes), 0, 0});
  }
  if (!unique_ids(dst_ids(out->entries))) return false;
  if (!disjoint_sets({Range{cache, cache + cache_blocks * block_bytes}},
                     {Range{swap, swap + swap_blocks * block_bytes}}))
    return false;
  out->segs.clear();
  if (is_swap_in)
    out->segs.push_back(GridSeg{swap, block_bytes, cache, block_bytes});
  else
    out->segs.push_back(GridSeg{cache, block_bytes, swap, block_bytes});
  out->host_side = is_swap_in ? 1 : 2;
  out->row_base = swap;
  out->row_stride = block_bytes;
  out->row_span = block_bytes;
  out->extents = out->entries.size();
  out->copied = out->entries.size() * block_bytes;
  return true;
}

uint64_t grid_finalize(GridPlan* p, uint32_t tile_shift) {
  const uint64_t ns = p->segs.size();
  uint64_t tiles = 0;
  for (GridEntry& g : p->entries) {
    const uint64_t per = (uint64_t(g.len) + (1ull << tile_shift) - 1) >> tile_shift;
    g.tile_begin = uint32_t(tiles);
    g.tiles_per_seg = uint32_t(per);
    tiles += per * ns;
    if (tiles > 0xffffffffull) return tiles;
  }
  return tiles;
}

void grid_expand(const GridPlan& p, uint32_t tile_shift, std::vector<Copy>* out) {
  out->clear();
  const uint32_t n = uint32_t(p.entries.size());
  if (n == 0) return;
  const GridEntry& last = p.entries.back();
  const uint64_t tiles = uint64_t(last.tile_begin) + uint64_t(last.tiles_per_seg) * p.segs.size();
  uint32_t cur = grid_find(p.entries.data(), n, 0);
  for (uint64_t t = 0; t < tiles; ++t) {
    while (cur + 1 < n && p.entries[cur + 1].tile_begin <= t) ++cur;
    uint64_t src, dst;
    uint32_t len;
    grid_resolve(p.entries[cur], p.segs.data(), uint32_t(t), tile_shift, &src, &dst, &len);
    if (!out->empty() && out->back().src + out->back().len == src &&
        out->back().dst + out->back().len == dst)
      out->back().len += len;
    else
      out->push_back(Copy{src, dst, len});
  }
}

}  // namespace kvx
