/*
 * kvx.h - C ABI of the B200-native KV-cache movement library (libkvx.so).
 *
 * The library moves paged K/V blocks between GPU HBM and page-locked host
 * slots (swap-out / swap-in) and between two GPUs over NVLink (migration).
 * Every entry point takes plain pointers and sizes, returns an int status
 * (KVX_OK == 0) and is asynchronous on the CUDA stream it is given, exactly
 * like the reference operator it replaces: it returns once the work is queued.
 * The caller orders later work with an event on that stream.
 *
 * All validation happens on the host before anything is queued: an invalid
 * request copies nothing and returns a non-zero status; kvx_last_error()
 * then holds a one-line description for the calling thread.
 *
 * Reference interfaces replaced (paths inside the Aegaeon project):
 *   kvx_swap            <- swap()                  ops/swap.cu:25-60, ops/ops.h:4-10,
 *                                                   pybind "swap" ops/ops.cpp:4-6
 *   kvx_layout_create   <- host view set-up         aegaeon/worker.py:1396-1433 (segments,
 *                                                   owners, kv_swap_view) + vllm_cache.py:75-101
 *   kvx_swap_blocks     <- Worker.swap_blocks loop  aegaeon/worker.py:2230-2329
 *   kvx_migrate_blocks  <- Worker.migrate_blocks    aegaeon/worker.py:2420-2430 (stub in the
 *                                                   reference: raises NotImplementedError)
 *   kvx_ipc_export /
 *   kvx_ipc_import      <- register_kvcache_mem_handles aegaeon/worker.py:2439-2451 (stub)
 *   kvx_upload_chunked  <- weight upload during switch aegaeon/loader/quick_loader.py:398-444
 *   kvx_upload_weights  <- pipeline_storage_transfer
 *                          quick_model_loader/quick_model_loader/model_loader.py:348-369,
 *                          load_tensors_content aegaeon/loader/quick_loader.py:326-340
 *   kvx_byte_extent     <- byte_extent_for_kernel_blocks aegaeon/cache_transfer.py:138-165
 */
#ifndef KVX_H_
#define KVX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define KVX_OK 0
#define KVX_ERR_INVALID_ARGUMENT 1 /* null pointer, negative count, bad flag   */
#define KVX_ERR_LENGTH_MISMATCH 2  /* metadata lists of different lengths     */
#define KVX_ERR_GROUP 3            /* cache-group id outside the group table   */
#define KVX_ERR_EXTENT 4           /* kernel-block extent invalid for the page */
#define KVX_ERR_BLOCK_ID 5         /* block / slot id outside its buffer       */
#define KVX_ERR_HOST_MEMORY 6      /* host buffer not usable for this mode     */
#define KVX_ERR_CUDA 7             /* a CUDA runtime call failed               */
#define KVX_ERR_DEVICE_TIMEOUT 8   /* a bounded device-side wait gave up       */
#define KVX_ERR_LAYOUT 9           /* the two layouts of a migration differ    */
#define KVX_ERR_NO_MEMORY 10       /* a library work area could not be made    */
#define KVX_ERR_IO 11              /* a file could not be opened or read       */
#define KVX_ERR_FORMAT 12          /* a file is not valid in its format        */

/* ---- transfer modes (the `mode` argument of the copy entry points) ------- */
#define KVX_MODE_AUTO 0     /* per-call choice by size and fragmentation:      */
                            /* at most 2 coalesced copies -> CE_EXTENT; host   */
                            /* memory not mapped -> CE; payload >= 16 MiB with */
                            /* mean host run >= 4 MiB -> CE; otherwise SM       */
#define KVX_MODE_SM 1       /* SM kernel, 32-byte vector loads/stores; host    */
                            /* side through its device-mapped address          */
#define KVX_MODE_CE 2       /* copy engines over coalesced runs; HBM side      */
                            /* gathered into / scattered from a staging area   */
#define KVX_MODE_SM_BULK 3  /* device<->device only (local, or a peer's pages  */
                            /* mapped over NVLink): TMA bulk copies through    */
                            /* shared memory, no multicast                     */
#define KVX_MODE_CE_EXTENT 4 /* one copy-engine copy per coalesced extent, no */
                            /* staging (fast when extents are already large)   */

const char* kvx_status_string(int status);
/* Detail message of the last failing call made by this thread ("" if none). */
const char* kvx_last_error(void);
int kvx_version(void);

/* ---- a1: drop-in for the reference's swap op ------------------------------
 * For i in [0, num_ids): copy `block_bytes` bytes
 *   swap-in : kv_swap [source_block_ids[i]] -> kv_cache[target_block_ids[i]]
 *   swap-out: kv_cache[source_block_ids[i]] -> kv_swap [target_block_ids[i]]
 * where buffer[id] is the byte range [id*block_bytes, (id+1)*block_bytes).
 * kv_cache is device memory of the current device; kv_swap is host memory
 * (page-locked for the SM path; any host memory for the copy-engine path).
 * The reference derives block_bytes as kv_cache.numel()*2/kv_cache.size(0)
 * (ops/swap.cu:34); callers pass that value.  When a target id repeats, the
 * last occurrence wins, as with the reference's in-order copies.
 * Replaces: swap() ops/swap.cu:25-60.                                        */
int kvx_swap(const int64_t* source_block_ids, const int64_t* target_block_ids,
             int64_t num_ids, int is_swap_in, void* kv_cache,
             uint64_t kv_cache_bytes, uint64_t block_bytes, void* kv_swap,
             uint64_t kv_swap_bytes, int mode, void* stream);

/* ---- a2/a7/a8: segmented multi-layer layout -------------------------------
 * A layout describes, for one GPU, the backing tensors ("segments") of a
 * composite KV block and the host pool that holds swapped blocks:
 *   segment s: device pages at segment_pages[s] (block id b at
 *              b*segment_page_bytes[s]), segment_num_blocks[s] pages;
 *              cpu_offset = byte offset of this segment inside one host row;
 *              owner mask = bit g set when cache group g may copy it.
 *   group g  : group_blocks_per_kv_block[g] kernel blocks per physical block.
 *   host pool: host_pool bytes, row r at r*host_row_bytes; the bytes of this
 *              GPU start at host_row_offset inside each row (tp_rank times the
 *              composite page in the reference).
 * host_pool may be NULL for a layout used only as a migration endpoint.
 * The layout copies the tables, not the memory they point to.
 * Replaces: worker.py:1396-1433 (owners, kv_swap_view), vllm_cache.py:75-101. */
typedef struct kvx_layout kvx_layout;

int kvx_layout_create(int device, int64_t num_segments,
                      void* const* segment_pages,
                      const uint64_t* segment_page_bytes,
                      const uint64_t* segment_num_blocks,
                      const uint64_t* segment_cpu_offsets,
                      const uint64_t* segment_owner_masks, int64_t num_groups,
                      const int64_t* group_blocks_per_kv_block, void* host_pool,
                      uint64_t host_pool_bytes, uint64_t host_row_bytes,
                      uint64_t host_row_offset, kvx_layout** layout_out);
int kvx_layout_destroy(kvx_layout* layout);

/* Swap the live extents of entries between GPU pages and host rows.
 * Entry i: block source_block_ids[i] -> target_block_ids[i] (GPU page id and
 * host row id, by direction), owned by cache group group_ids[i], live extent =
 * kernel blocks [first_kernel_blocks[i], first+valid_kernel_blocks[i]) of the
 * page.  For every segment owned by the group the byte extent
 *   (page/ratio*first, page/ratio*valid)
 * is copied; zero-length extents are skipped.  copied_bytes / copy_extents
 * (optional, may be NULL) report the totals the reference logs.
 * Replaces: Worker.swap_blocks hot loop, worker.py:2230-2329.               */
int kvx_swap_blocks(kvx_layout* layout, int64_t num_entries,
                    const int64_t* source_block_ids,
                    const int64_t* target_block_ids, const int64_t* group_ids,
                    const int64_t* first_kernel_blocks,
                    const int64_t* valid_kernel_blocks, int is_swap_in, int mode,
                    void* stream, uint64_t* copied_bytes,
                    uint64_t* copy_extents);

/* ---- a10: GPU -> GPU migration over NVLink ---------------------------------
 * Same entry semantics as kvx_swap_blocks, with source pages in `source` and
 * target pages in `target`.  The copy runs on the SMs of the current device,
 * which must be able to address both layouts' pages: its own memory, and a
 * peer's memory mapped into this process with kvx_ipc_import.  Pull (run on
 * the target GPU, source pages imported) and push (run on the source GPU,
 * target pages imported) are both valid; each load or store that crosses
 * NVLink is a plain peer access (no multicast): 16/32-byte vector accesses
 * in KVX_MODE_SM (AUTO), bulk copies through shared memory in
 * KVX_MODE_SM_BULK.  The segment tables
 * of the two layouts must agree in count, page sizes and owners, and their
 * group tables must be equal.
 * Fills: Worker.migrate_blocks, worker.py:2420-2430 (NotImplementedError in
 * the reference; its prefill->decode route is swap-out then swap-in).       */
int kvx_migrate_blocks(kvx_layout* source, kvx_layout* target,
                       int64_t num_entries, const int64_t* source_block_ids,
                       const int64_t* target_block_ids,
                       const int64_t* group_ids,
                       const int64_t* first_kernel_blocks,
                       const int64_t* valid_kernel_blocks, int mode,
                       void* stream, uint64_t* copied_bytes,
                       uint64_t* copy_extents);

/* ---- IPC memory handles (peer mapping of a KV cache) -----------------------
 * export: 64-byte handle of the allocation holding dev_ptr, plus the offset
 * of dev_ptr inside that allocation.  import: maps the allocation (peer access
 * enabled lazily) and returns base+offset.  close: unmaps a pointer returned by
 * import.  Fills: register/unregister_kvcache_mem_handles, worker.py:2439-2451. */
int kvx_ipc_export(void* dev_ptr, uint8_t* handle_out64, uint64_t* offset_out);
int kvx_ipc_import(int device, const uint8_t* handle64, uint64_t offset,
                   void** dev_ptr_out);
int kvx_ipc_close(int device, void* dev_ptr);

/* ---- (f3) events ordering moves across workers -------------------------------
 * Pooled CUDA events, interprocess handles, and a cache of opened handles.
 * Replaces the per-call cudaIpcOpenEventHandle / cudaStreamWaitEvent /
 * cudaEventDestroy of Worker._wait_source_events (aegaeon/worker.py:2351-2394,
 * utils.py:263-288).  create: an event of the current device from the pool
 * (interprocess != 0: shareable).  query: *done = 1 once its last record has
 * completed.  ipc_handle: 64 bytes for another process.  open_ipc: the event
 * behind a handle, opened once and cached by the handle bytes (release drops
 * the reference, the cache keeps the event; forget_ipc closes it).
 * stream_wait_events: `stream` waits for every event of the list.  release:
 * back to the pool (an interprocess event whose handle was shared must not be
 * released while another process may still wait on that record). */
typedef struct kvx_event kvx_event;
int kvx_event_create(int interprocess, kvx_event** out);
int kvx_event_record(kvx_event* event, void* stream);
int kvx_event_query(kvx_event* event, int* done);
int kvx_event_synchronize(kvx_event* event);
int kvx_event_ipc_handle(kvx_event* event, uint8_t* handle_out64);
int kvx_event_open_ipc(const uint8_t* handle64, kvx_event** out);
int kvx_event_forget_ipc(const uint8_t* handle64);
int kvx_stream_wait_events(void* stream, kvx_event* const* events, int64_t n);
int kvx_event_release(kvx_event* event);

/* ---- (f1) chunked weight upload for a model switch --------------------------
 * Host -> device copy of `bytes` bytes in pieces of at most chunk_bytes on
 * `stream` (0: one piece): kvx_upload_weights below with one buffer and every
 * host thread, so a pageable source goes through the bounce buffers.
 * Replaces: the slice_storage.copy_(non_blocking=True) loop,
 * aegaeon/loader/quick_loader.py:398-444.                                    */
int kvx_upload_chunked(void* dst_device, const void* src_host, uint64_t bytes,
                       uint64_t chunk_bytes, void* stream);

/* ---- f1: weight upload of a model switch ----------------------------------
 * Copies num_buffers host buffers (weight storages) into device buffers of
 * the current device in pieces of chunk_bytes, in order, on `stream`.
 *  * Page-locked (or managed) sources: one cudaMemcpyAsync per piece; the
 *    call returns once they are queued.
 *  * Pageable sources: through two page-locked bounce buffers of
 *    min(chunk_bytes, 64 MiB) owned by the library (allocated on first use).  host_threads threads copy
 *    piece k+1 into one bounce buffer while the copy engine moves piece k out
 *    of the other, the two-stage pipeline of the reference's
 *    pipeline_storage_transfer (pageable -> pinned -> device, cut into
 *    pieces).  The call returns when the last piece is queued; it blocks only
 *    to reuse a bounce buffer.
 * Destinations must be device memory of the current device.  Errors:
 * KVX_ERR_INVALID_ARGUMENT (null pointers, chunk_bytes 0, a destination that
 * is not device memory of the current device), KVX_ERR_CUDA.
 * Replaces: pipeline_storage_transfer,
 * quick_model_loader/quick_model_loader/model_loader.py:348-369, and the
 * per-storage slice_storage.copy_(non_blocking=True) of load_tensors_content,
 * aegaeon/loader/quick_loader.py:326-340 (64 MiB cuts as in the disabled
 * variant at :398-444).                                                      */
int kvx_upload_weights(void* const* dst_device, const void* const* src_host,
                       const uint64_t* bytes, int64_t num_buffers, uint64_t chunk_bytes,
                       int host_threads, void* stream);

/* ---- a3: extent arithmetic (host only, no GPU needed) ---------------------
 * (first, count) kernel blocks of a page of page_bytes split into
 * kernel_blocks_per_page -> (byte_offset, byte_length).  Same checks and
 * results as byte_extent_for_kernel_blocks, cache_transfer.py:138-165.      */
int kvx_byte_extent(uint64_t page_bytes, int64_t kernel_blocks_per_page,
                    int64_t first_kernel_block, int64_t num_kernel_blocks,
                    uint64_t* byte_offset_out, uint64_t* byte_length_out);

/* ---- planning introspection (host only, no GPU needed) ---------------------
 * Run the validation and planning of kvx_swap_blocks / kvx_swap without
 * touching a GPU and return the copies the SM path would issue, as (source
 * address, destination address, bytes) triples: when the request has a grid
 * form (uniform pages, distinct targets, disjoint memory) these come from the
 * same tile resolver the kernel uses, entry by entry; otherwise from the item
 * planner in the reference's issue order (segment-major, then entries).  *num_copies_inout
 * holds the capacity of the three arrays on entry and the number of copies on
 * return (when the capacity is too small the arrays are left unfilled and
 * KVX_OK is returned with the required count).  Used by tests of the host
 * logic and by callers that want to inspect a plan.                          */
int kvx_plan_swap_blocks(const kvx_layout* layout, int64_t num_entries,
                         const int64_t* source_block_ids,
                         const int64_t* target_block_ids,
                         const int64_t* group_ids,
                         const int64_t* first_kernel_blocks,
                         const int64_t* valid_kernel_blocks, int is_swap_in,
                         uint64_t* src_addrs, uint64_t* dst_addrs,
                         uint64_t* lengths, int64_t* num_copies_inout);
int kvx_plan_swap(const int64_t* source_block_ids,
                  const int64_t* target_block_ids, int64_t num_ids,
                  int is_swap_in, uint64_t kv_cache, uint64_t kv_cache_bytes,
                  uint64_t block_bytes, uint64_t kv_swap,
                  uint64_t kv_swap_bytes, uint64_t* src_addrs,
                  uint64_t* dst_addrs, uint64_t* lengths,
                  int64_t* num_copies_inout);

/* ---- statistics and device status ------------------------------------------
 * kvx_last_mode: the transfer mode the last successful copy call of this
 * thread used (KVX_MODE_SM / _CE / _SM_BULK / _CE_EXTENT).
 * kvx_device_status: reads (and with reset != 0 clears) the device error word
 * written by kernels whose bounded waits gave up; synchronizes the device.  */
int kvx_last_mode(void);
/* Number of copy kernels this process has launched through the library. */
uint64_t kvx_kernel_launches(void);
/* Per-launch timing of the copy kernels: while enabled, every launch is
 * bracketed by two CUDA events on its stream.  _read synchronizes those
 * events and returns, since the previous read, the number of launches, their
 * summed durations, the busy time (union of the launch intervals per device:
 * launches on different streams that overlapped count once) and the HBM bytes
 * they move (read + write when both sides are local memory, one side when the
 * other is host or peer memory). */
int kvx_kernel_timing(int enable);
int kvx_kernel_timing_read(uint64_t* launches, double* total_ms, double* busy_ms,
                           uint64_t* hbm_bytes);
int kvx_device_status(int device, int reset, int* status_out);

/* Self-test of the device-side timeout path: launches, on `stream`, a kernel
 * that waits (with the same bounded mbarrier wait the TMA copy kernel uses) on
 * a barrier nothing arrives on.  After limit_ns the wait gives up and the
 * kernel sets the device status word to KVX_ERR_DEVICE_TIMEOUT, which
 * kvx_device_status then reports; the context stays usable.  No counterpart
 * in the reference (it has no device-side waits). */
int kvx_selftest_bounded_wait(uint64_t limit_ns, void* stream);

/* Tuning knobs of KVX_MODE_AUTO and of the kernels; 0 keeps the current value
 * (ce_pipeline: -1 keeps it).
 *   sm_ctas_host : CTAs of an SM kernel that touches host memory (default,
 *                  and 0 through kvx_set_option: 3/4 of the SM count when it
 *                  writes host memory, 5/4 when it reads it)
 *   sm_ctas_dev  : CTAs of an SM kernel that touches device memory only
 *   ce_min_run   : mean coalesced host-run bytes from which AUTO uses the CE
 *   staging_bytes: size of each staging area of the copy-engine mode
 *                  (one per direction and device, 1 GiB by default)
 * Environment: KVX_SM_CTAS_HOST, KVX_SM_CTAS_DEV, KVX_CE_MIN_RUN,
 * KVX_STAGING_BYTES, KVX_CE_PIPELINE=1 to double-buffer the staging area
 * (gather/scatter of one half on an internal stream while the copy engines
 * move the other; helps a single direction, hurts concurrent directions),
 * KVX_VEC_BYTES (32 default: 256-bit loads/stores where aligned; 16),
 * KVX_BULK_CTAS_PER_SM (2 default; 1), KVX_CE_MIN_BYTES (16 MiB: smallest
 * payload AUTO stages through the copy engines), KVX_DIRECT_MAX (2: most
 * coalesced copies AUTO sends to the copy engines directly; 0 never) and
 * KVX_INLINE (1: grid plans of at most 1020 records travel in the kernel's
 * parameters, in lists of 124, 508 or 1020 records, instead of through the
 * descriptor ring; 0 never). */
int kvx_configure(int64_t sm_ctas_host, int64_t sm_ctas_dev,
                  int64_t ce_min_run, int64_t staging_bytes,
                  int64_t ce_pipeline /* -1 keep, 0 off, 1 on */);

/* No counterpart in the reference (it has no tuning knobs on this path).
 * One tuning knob by name (0 on success, KVX_ERR_INVALID_ARGUMENT for an
 * unknown name or a value out of range).  Names: "ce_streams" (1..8: streams
 * that share the host-run copies of one copy-engine call; default 1, env
 * KVX_CE_STREAMS), "ce_streams_max_run" (those streams are used only when the
 * mean host run is at most this many bytes; env KVX_CE_STREAMS_MAX_RUN),
 * "ce_max_copy" (largest single copy-engine copy of the staged mode; longer
 * host runs go as pieces of this size; 0 = no limit, env KVX_CE_MAX_COPY),
 * "ce_min_run", "ce_min_bytes", "sm_ctas_host", "sm_ctas_host_out" and
 * "sm_ctas_host_in" (CTAs of the SM kernel that writes host memory, or reads
 * it; each overrides sm_ctas_host for its direction; 0: not set; env
 * KVX_SM_CTAS_HOST_OUT / KVX_SM_CTAS_HOST_IN), "sm_ctas_dev", "direct_max",
 * "staging_bulk" (1: TMA bulk kernel for the staging gather/scatter, 0: the
 * vector kernel), "bulk_ctas_per_sm" (1 or 2), "bulk_waves" (1..64: the TMA
 * kernel's grid as this many waves of resident CTAs, 16 by default; env
 * KVX_BULK_WAVES),
 * "vec_bytes" (16 or 32), "host_bulk" (1: SM-mode copies with a host side
 * go through the TMA bulk kernel, 16 KiB bulk copies to or from the mapped
 * host rows; 0 default: the vector kernel; env KVX_HOST_BULK), as above.
 * Settings are process-wide. */
int kvx_set_option(const char* name, int64_t value);

/* ---- (f4) safetensors header ------------------------------------------------
 * Reads the header of a .safetensors file and validates it as the
 * `safetensors` crate 0.4.3 does (SafeTensors::read_metadata): header length,
 * UTF-8 JSON, dtypes, offsets tiling the data without gaps, sizes equal to
 * shape x dtype, nothing after the last tensor.  Writes the JSON the reference
 * returns (file_path, size, offset = 8 + header length, tensor_info_map of
 * dtype / shape / data_offsets) into `out` (NUL-terminated) when `capacity`
 * exceeds its length; *length_out always receives the length.
 * Errors: KVX_ERR_IO (cannot open/read), KVX_ERR_FORMAT (invalid header).
 * Replaces: read_safetensors_meta_as_json, quick_model_loader/rsrc/lib.rs:19-51. */
int kvx_safetensors_meta_json(const char* file_path, char* out,
                              uint64_t capacity, uint64_t* length_out);

/* ---- allocation-free swap ---------------------------------------------------
 * No counterpart in the reference.  For callers that must not allocate GPU
 * memory while they swap: a runtime that owns all of HBM through its own
 * arena, a process swapping out near its memory limit during a model switch,
 * or code where an allocation would synchronise the device.  Same copy as
 * kvx_swap in its SM zero-copy mode (kv_swap must be page-locked and mapped
 * for the device, or managed memory), same checks, same last-writer rule for
 * repeated targets.  A stream that is capturing is refused with
 * KVX_ERR_INVALID_ARGUMENT before anything is queued: the ids go to the
 * device through static host storage that the next call rewrites.
 * Its scratch is a fixed device array of KVX_NOALLOC_MAX_IDS source and
 * target ids (1 MiB), compiled into the library and held by every GPU that
 * loads it until the process exits; more ids per call are rejected with
 * KVX_ERR_INVALID_ARGUMENT (message in kvx_last_error).  Nothing is
 * allocated: no cudaMalloc, cudaFree or allocating library call.
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  All calls share the array and each call
 * overwrites the ids it uses (nothing needs to start at zero): calls whose
 * GPU work overlaps, e.g. on two streams without an event between them, race
 * on it.  Calls on one stream are ordered and safe.                         */
#define KVX_NOALLOC_MAX_IDS 65536
int kvx_swap_noalloc(const int64_t* source_block_ids,
                     const int64_t* target_block_ids, int64_t num_ids,
                     int is_swap_in, void* kv_cache, uint64_t kv_cache_bytes,
                     uint64_t block_bytes, void* kv_swap,
                     uint64_t kv_swap_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KVX_H_ */
