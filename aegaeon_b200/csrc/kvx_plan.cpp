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

}  // namespace kvx
