/*
 * kvx_oracle.c - CPU restatement of the reference's KV swap semantics.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load this library: it is the checker the
 * CUDA path is compared with, never part of the product path.
 *
 * Functions and the reference code they restate (paths in the Aegaeon repo):
 *   oracle_swap        ops/swap.cu:25-60  one block copy per id pair, in order,
 *                      block = block_bytes bytes at id*block_bytes
 *   oracle_byte_extent aegaeon/cache_transfer.py:113-165 (same checks)
 *   oracle_swap_blocks aegaeon/worker.py:2270-2329 segment-major loop over
 *                      entries, owner filter, byte extent, zero-length skip,
 *                      host row offset tp_rank*composite + cpu_offset + off
 *   oracle_gather_mt / oracle_scatter_mt
 *                      the CPU path named as the baseline (index_select /
 *                      index_copy_ over the block mapping): the same byte
 *                      movement between two host buffers, split over threads.
 *
 * Copies run strictly in the reference's order, so repeated destinations end
 * with the last writer's bytes, as the reference's in-order copies do.
 * Return value: 0 on success, otherwise the kvx status code of the first
 * failing check (no copy is made when a check fails: all checks run first).
 */
#include <pthread.h>
#include <stdint.h>
#include <string.h>

#define ORC_OK 0
#define ORC_INVALID 1
#define ORC_GROUP 3
#define ORC_EXTENT 4
#define ORC_BLOCK_ID 5

int oracle_version(void) { return 1; }

/* prefix_bytes_for_kernel_blocks, cache_transfer.py:113-135 */
static int prefix_bytes(uint64_t page, int64_t ratio, int64_t valid, uint64_t* out) {
  if (page == 0) return ORC_EXTENT;
  if (ratio <= 0) return ORC_EXTENT;
  if (valid < 0 || valid > ratio) return ORC_EXTENT;
  if (page % (uint64_t)ratio) return ORC_EXTENT;
  *out = page / (uint64_t)ratio * (uint64_t)valid;
  return ORC_OK;
}

/* byte_extent_for_kernel_blocks, cache_transfer.py:138-165 */
int oracle_byte_extent(uint64_t page, int64_t ratio, int64_t first, int64_t count,
                       uint64_t* off, uint64_t* len) {
  if (first < 0) return ORC_EXTENT;
  if (first > ((int64_t)1 << 48) || count > ((int64_t)1 << 48) ||
      count < -((int64_t)1 << 48))
    return ORC_EXTENT;
  if (first + count > ratio) return ORC_EXTENT;
  int rc = prefix_bytes(page, ratio, first, off);
  if (rc) return rc;
  return prefix_bytes(page, ratio, count, len);
}

/* ops/swap.cu:25-60 */
int oracle_swap(const int64_t* src, const int64_t* dst, int64_t n, int is_swap_in,
                uint8_t* cache, uint64_t cache_bytes, uint64_t block_bytes,
                uint8_t* swap, uint64_t swap_bytes) {
  if (n < 0) return ORC_INVALID;
  if (block_bytes == 0) return ORC_OK;
  const uint64_t cache_blocks = cache_bytes / block_bytes;
  const uint64_t swap_blocks = swap_bytes / block_bytes;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t dev = is_swap_in ? dst[i] : src[i];
    const int64_t slot = is_swap_in ? src[i] : dst[i];
    if (dev < 0 || (uint64_t)dev >= cache_blocks) return ORC_BLOCK_ID;
    if (slot < 0 || (uint64_t)slot >= swap_blocks) return ORC_BLOCK_ID;
  }
  for (int64_t i = 0; i < n; ++i) {
    if (is_swap_in)
      memcpy(cache + (uint64_t)dst[i] * block_bytes, swap + (uint64_t)src[i] * block_bytes,
             block_bytes);
    else
      memcpy(swap + (uint64_t)dst[i] * block_bytes, cache + (uint64_t)src[i] * block_bytes,
             block_bytes);
  }
  return ORC_OK;
}

/* worker.py:2270-2329.  seg_pages[s] is a host buffer holding the GPU pages
 * of segment s (num_blocks[s] pages of page_bytes[s]); host rows of row_bytes
 * at `pool`; this rank's bytes begin at row_offset. */
static int swap_blocks_pass(int do_copy, int64_t num_segments, uint8_t* const* seg_pages,
                            const uint64_t* page_bytes, const uint64_t* num_blocks,
                            const uint64_t* cpu_offsets, const uint64_t* owner_masks,
                            int64_t num_groups, const int64_t* ratios, uint8_t* pool,
                            uint64_t num_rows, uint64_t row_bytes, uint64_t row_offset,
                            int64_t n, const int64_t* src, const int64_t* dst,
                            const int64_t* group, const int64_t* first,
                            const int64_t* valid, int is_swap_in, uint64_t* copied) {
  uint64_t total = 0;
  for (int64_t s = 0; s < num_segments; ++s) {
    for (int64_t i = 0; i < n; ++i) {
      const int64_t g = group[i];
      if (!((owner_masks[s] >> g) & 1ull)) continue;
      uint64_t off = 0, len = 0;
      int rc = oracle_byte_extent(page_bytes[s], ratios[g], first[i], valid[i], &off, &len);
      if (rc) return rc;
      if (len == 0) continue;
      const int64_t dev = is_swap_in ? dst[i] : src[i];
      const int64_t row = is_swap_in ? src[i] : dst[i];
      if (dev < 0 || (uint64_t)dev >= num_blocks[s]) return ORC_BLOCK_ID;
      if (row < 0 || (uint64_t)row >= num_rows) return ORC_BLOCK_ID;
      const uint64_t host_off = row_offset + cpu_offsets[s] + off;
      if (host_off + len > row_bytes) return ORC_INVALID;
      total += len;
      if (!do_copy) continue;
      uint8_t* gpu = seg_pages[s] + (uint64_t)dev * page_bytes[s] + off;
      uint8_t* host = pool + (uint64_t)row * row_bytes + host_off;
      if (is_swap_in)
        memcpy(gpu, host, len);
      else
        memcpy(host, gpu, len);
    }
  }
  (void)num_groups;
  if (copied) *copied = total;
  return ORC_OK;
}

int oracle_swap_blocks(int64_t num_segments, uint8_t* const* seg_pages,
                       const uint64_t* page_bytes, const uint64_t* num_blocks,
                       const uint64_t* cpu_offsets, const uint64_t* owner_masks,
                       int64_t num_groups, const int64_t* ratios, uint8_t* pool,
                       uint64_t num_rows, uint64_t row_bytes, uint64_t row_offset, int64_t n,
                       const int64_t* src, const int64_t* dst, const int64_t* group,
                       const int64_t* first, const int64_t* valid, int is_swap_in,
                       uint64_t* copied) {
  if (n < 0 || num_segments < 0) return ORC_INVALID;
  for (int64_t i = 0; i < n; ++i) /* worker.py:2244-2246, before any copy */
    if (group[i] < 0 || group[i] >= num_groups) return ORC_GROUP;
  int rc = swap_blocks_pass(0, num_segments, seg_pages, page_bytes, num_blocks, cpu_offsets,
                            owner_masks, num_groups, ratios, pool, num_rows, row_bytes,
                            row_offset, n, src, dst, group, first, valid, is_swap_in, copied);
  if (rc) return rc;
  return swap_blocks_pass(1, num_segments, seg_pages, page_bytes, num_blocks, cpu_offsets,
                          owner_masks, num_groups, ratios, pool, num_rows, row_bytes, row_offset,
                          n, src, dst, group, first, valid, is_swap_in, copied);
}

/* ---- threaded CPU baseline: gather/scatter whole blocks between host buffers */
struct mt_job {
  const int64_t* src;
  const int64_t* dst;
  int64_t begin, end;
  const uint8_t* from;
  uint8_t* to;
  uint64_t block_bytes;
};

static void* mt_worker(void* arg) {
  struct mt_job* j = (struct mt_job*)arg;
  for (int64_t i = j->begin; i < j->end; ++i)
    memcpy(j->to + (uint64_t)j->dst[i] * j->block_bytes,
           j->from + (uint64_t)j->src[i] * j->block_bytes, j->block_bytes);
  return 0;
}

/* to[dst[i]] = from[src[i]] for all i, over `threads` threads (no checks: the
 * caller validated ids; destinations must be distinct). */
int oracle_copy_blocks_mt(const int64_t* src, const int64_t* dst, int64_t n,
                          const uint8_t* from, uint8_t* to, uint64_t block_bytes,
                          int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  struct mt_job jobs[256];
  for (int t = 0; t < threads; ++t) {
    jobs[t].src = src;
    jobs[t].dst = dst;
    jobs[t].begin = n * t / threads;
    jobs[t].end = n * (t + 1) / threads;
    jobs[t].from = from;
    jobs[t].to = to;
    jobs[t].block_bytes = block_bytes;
  }
  for (int t = 1; t < threads; ++t) pthread_create(&tid[t], 0, mt_worker, &jobs[t]);
  mt_worker(&jobs[0]);
  for (int t = 1; t < threads; ++t) pthread_join(tid[t], 0);
  return ORC_OK;
}
