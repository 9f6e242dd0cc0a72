// C ABI of libkvx.so: per-device runtime state, transfer-mode selection and
// the entry points declared in include/kvx.h.
//
// Execution model (all on the caller's stream, nothing synchronous unless a
// library work area must be recycled):
//   1. plan   : validate and turn the request into an ordered copy list
//               (kvx_plan.cpp), split into conflict-free waves, coalesce;
//   2. upload : write the kernel item table into a page-locked descriptor ring
//               and queue one host->device copy of it;
//   3. launch : one copy kernel per wave (SM mode), or per staging chunk a
//               gather/scatter kernel plus copy-engine copies (CE mode);
//   4. fence  : record a pooled event on the stream that frees the ring
//               region (and the staging area) for reuse.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/kvx.h"
#include "kvx_kernels.cuh"
#include "kvx_plan.h"

namespace kvx {
namespace {

thread_local std::string t_last_error;
thread_local int t_last_mode = 0;
std::atomic<uint64_t> g_kernel_launches{0};

// Optional per-launch timing: an event pair around every copy kernel, read
// back by kvx_kernel_timing_read.  Off unless a caller enables it.
struct TimedLaunch {
  int device;
  cudaEvent_t begin, end;
  uint64_t hbm_bytes;
};
std::atomic<bool> g_timing{false};
std::mutex g_timing_mu;
std::vector<TimedLaunch> g_timed;

int set_error(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int cuda_error(cudaError_t e, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                  cudaGetErrorString(e) + ")";
  return set_error(KVX_ERR_CUDA, m);
}

#define KVX_CUDA(call)                                  \
  do {                                                  \
    cudaError_t e_ = (call);                            \
    if (e_ != cudaSuccess) return cuda_error(e_, #call); \
  } while (0)

int from_plan(const Error& e) {
  if (e.ok()) return KVX_OK;
  return set_error(e.code, e.msg);
}

// ---- tunables ----------------------------------------------------------------
constexpr int kMaxCeStreams = 8;

struct Tunables {
  int64_t sm_ctas_host = 0;    // 0: by direction (3/4 of the SMs to host, 5/4 from host)
  int64_t sm_ctas_host_out = 0;  // writes to host memory only; 0: sm_ctas_host's rule
  int64_t sm_ctas_host_in = 0;   // reads from host memory only; 0: sm_ctas_host's rule
  int64_t sm_ctas_dev = 0;     // 0: by launch size, 4 to 16 x number of SMs
  // Mean coalesced host run from which AUTO stages through the copy engines.
  // Measured on B200 (896 KiB rows, scattered in groups): the copy engines
  // pay about 5 us per copy, so with ~1.2 MiB runs they reach 0.82 of the
  // link one way and 0.70 with both directions active, and 0.89 / 0.79 with
  // ~2.3 MiB runs, where the SM path holds 0.92 and 0.85 at any run length;
  // at ~4.7 MiB the two tie (0.93 / 0.85) and from ~9 MiB the copy engines
  // win (0.95 / 0.89).
  int64_t ce_min_run = 4ll << 20;
  // AUTO stages through the copy engines only from this payload up: below it
  // one zero-copy kernel beats gather + DMA (measured on B200: the SM path is
  // 3-17% faster from 0.5 to 8 MiB per call, the copy engines 3-6% faster at
  // 32 MiB).
  int64_t ce_min_bytes = 16ll << 20;
  int64_t staging_bytes = 1ll << 30;
  int64_t ce_pipeline = 0;  // double-buffered staging with a helper stream
  int64_t vec_bytes = 32;   // bytes per thread access of the vector kernel (16 or 32)
  int64_t bulk_ctas_per_sm = 2;  // CTAs per SM of the TMA kernel (1 or 2)
  // Most waves of resident CTAs in a TMA kernel grid (bulk_grid).  Each CTA
  // copies one contiguous span of the launch, so with a single wave the launch
  // waits for the slowest of 296 spans; 16 waves of short spans balance
  // themselves.  Measured on B200 (1 GiB staging chunk): isolated 0.93 ->
  // 1.00 of the copy peak, live beside the other direction's DMA 0.77 -> 0.85.
  int64_t bulk_waves = 16;
  int64_t staging_bulk = 1;      // staging gather/scatter: 1 TMA kernel, 0 vector kernel
  int64_t inline_lists = 1;      // small grid plans passed in kernel parameters
  int64_t direct_max = 2;        // AUTO: at most this many copies go straight to the copy engine
  // Copy-engine mode: the host-run copies of one call spread round-robin over
  // this many streams (each feeds its own copy-engine queue), so the setup
  // gap of one short copy overlaps the transfer of another.
  int64_t ce_streams = 1;
  int64_t ce_streams_max_run = 4ll << 20;  // ... only when the mean run is at most this
  // Largest single copy-engine copy of the staged mode (0: one copy per host
  // run, however long); longer runs are issued as pieces of this size.
  int64_t ce_max_copy = 0;
  // SM mode with a host side: the TMA bulk kernel (16 KiB bulk copies between
  // shared memory and the device-mapped host rows) instead of the vector
  // kernel's 32-byte accesses.  Off by default.
  int64_t host_bulk = 0;
};
std::mutex g_tun_mu;
Tunables g_tun;

int64_t env_i64(const char* name, int64_t dflt) {
  const char* v = std::getenv(name);
  if (!v || !*v) return dflt;
  return std::strtoll(v, nullptr, 0);
}

Tunables tunables() {
  static std::once_flag once;
  std::call_once(once, [] {
    std::lock_guard<std::mutex> g(g_tun_mu);
    g_tun.sm_ctas_host = env_i64("KVX_SM_CTAS_HOST", g_tun.sm_ctas_host);
    g_tun.sm_ctas_host_out = env_i64("KVX_SM_CTAS_HOST_OUT", g_tun.sm_ctas_host_out);
    g_tun.sm_ctas_host_in = env_i64("KVX_SM_CTAS_HOST_IN", g_tun.sm_ctas_host_in);
    g_tun.sm_ctas_dev = env_i64("KVX_SM_CTAS_DEV", g_tun.sm_ctas_dev);
    g_tun.ce_min_run = env_i64("KVX_CE_MIN_RUN", g_tun.ce_min_run);
    g_tun.ce_min_bytes = env_i64("KVX_CE_MIN_BYTES", g_tun.ce_min_bytes);
    g_tun.staging_bytes = env_i64("KVX_STAGING_BYTES", g_tun.staging_bytes);
    g_tun.ce_pipeline = env_i64("KVX_CE_PIPELINE", g_tun.ce_pipeline);
    g_tun.vec_bytes = env_i64("KVX_VEC_BYTES", g_tun.vec_bytes) == 16 ? 16 : 32;
    g_tun.bulk_ctas_per_sm = env_i64("KVX_BULK_CTAS_PER_SM", g_tun.bulk_ctas_per_sm) == 1 ? 1 : 2;
    g_tun.bulk_waves = std::max<int64_t>(1, env_i64("KVX_BULK_WAVES", g_tun.bulk_waves));
    g_tun.staging_bulk = env_i64("KVX_STAGING_BULK", g_tun.staging_bulk) ? 1 : 0;
    g_tun.inline_lists = env_i64("KVX_INLINE", g_tun.inline_lists) ? 1 : 0;
    g_tun.direct_max = env_i64("KVX_DIRECT_MAX", g_tun.direct_max);
    g_tun.ce_streams = std::max<int64_t>(1, std::min<int64_t>(
        kMaxCeStreams, env_i64("KVX_CE_STREAMS", g_tun.ce_streams)));
    g_tun.ce_streams_max_run = env_i64("KVX_CE_STREAMS_MAX_RUN", g_tun.ce_streams_max_run);
    g_tun.ce_max_copy = env_i64("KVX_CE_MAX_COPY", g_tun.ce_max_copy);
    g_tun.host_bulk = env_i64("KVX_HOST_BULK", g_tun.host_bulk) ? 1 : 0;
  });
  std::lock_guard<std::mutex> g(g_tun_mu);
  return g_tun;
}

// ---- per-device state ---------------------------------------------------------
struct Region {
  cudaEvent_t ev;
  size_t begin, end;
};

struct Staging {
  char* dev = nullptr;
  size_t cap = 0;
  cudaEvent_t last = nullptr;  // recorded after the latest use
  bool used = false;
  // Double-buffered pipeline: the gather/scatter kernels of one half run on
  // `helper` while the copy engines move the other half on the caller's stream.
  cudaStream_t helper = nullptr;
  cudaEvent_t ev_start = nullptr, ev_dev[2] = {}, ev_link[2] = {};
  // Streams that share the host-run copies of one call (run_streams > 1).
  cudaStream_t run_stream[kMaxCeStreams] = {};
  cudaEvent_t run_done[kMaxCeStreams] = {};
  cudaEvent_t run_fork = nullptr;
};

struct DeviceState {
  int device = 0;
  int sms = 148;
  std::mutex mu;
  // Descriptor ring: page-locked host + device copies of item tables.
  char* ring_host = nullptr;
  char* ring_dev = nullptr;
  size_t ring_cap = 0;
  size_t ring_head = 0;
  std::deque<Region> inflight;
  std::vector<cudaEvent_t> pool;
  Staging staging[2];  // [0] device->host, [1] host->device
  bool bulk_ready = false;
  // Weight upload from pageable memory: two page-locked bounce buffers, each
  // guarded by the event recorded after the copy that last read it.
  std::mutex upload_mu;
  char* bounce[2] = {nullptr, nullptr};
  size_t bounce_cap = 0;
  cudaEvent_t bounce_ev[2] = {nullptr, nullptr};
  bool bounce_used[2] = {false, false};
};

std::mutex g_dev_mu;
DeviceState* g_devs[64] = {};

class DeviceGuard {
 public:
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
    if (prev_ != dev) {
      ok_ = cudaSetDevice(dev) == cudaSuccess;
      switched_ = true;
    }
  }
  ~DeviceGuard() {
    if (switched_ && prev_ >= 0) cudaSetDevice(prev_);
  }
  bool ok() const { return ok_; }

 private:
  int prev_ = -1;
  bool switched_ = false;
  bool ok_ = true;
};

int get_state(int device, DeviceState** out) {
  if (device < 0 || device >= 64)
    return set_error(KVX_ERR_INVALID_ARGUMENT, "device index out of range");
  std::lock_guard<std::mutex> g(g_dev_mu);
  if (!g_devs[device]) {
    int sms = 0;
    cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return cuda_error(e, "cudaDeviceGetAttribute");
    auto* st = new DeviceState();
    st->device = device;
    st->sms = sms;
    g_devs[device] = st;
  }
  *out = g_devs[device];
  return KVX_OK;
}

int take_event(DeviceState* st, cudaEvent_t* ev) {
  if (!st->pool.empty()) {
    *ev = st->pool.back();
    st->pool.pop_back();
    return KVX_OK;
  }
  KVX_CUDA(cudaEventCreateWithFlags(ev, cudaEventDisableTiming));
  return KVX_OK;
}

int retire_front(DeviceState* st, bool block) {
  Region r = st->inflight.front();
  if (block) {
    KVX_CUDA(cudaEventSynchronize(r.ev));
  } else {
    cudaError_t q = cudaEventQuery(r.ev);
    if (q == cudaErrorNotReady) return 1;
    if (q != cudaSuccess) return cuda_error(q, "cudaEventQuery");
  }
  st->inflight.pop_front();
  st->pool.push_back(r.ev);
  return KVX_OK;
}

// Reserve `bytes` of the descriptor ring; returns the offset.
int ring_acquire(DeviceState* st, size_t bytes, size_t* off) {
  bytes = (bytes + 255) & ~size_t(255);
  if (bytes > st->ring_cap) {
    while (!st->inflight.empty()) {
      int rc = retire_front(st, true);
      if (rc) return rc;
    }
    if (st->ring_host) cudaFreeHost(st->ring_host);
    if (st->ring_dev) cudaFree(st->ring_dev);
    st->ring_host = st->ring_dev = nullptr;
    size_t cap = std::max<size_t>(bytes * 2, size_t(8) << 20);
    cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&st->ring_host), cap,
                                  cudaHostAllocDefault);
    if (e != cudaSuccess) return cuda_error(e, "cudaHostAlloc(descriptor ring)");
    e = cudaMalloc(reinterpret_cast<void**>(&st->ring_dev), cap);
    if (e != cudaSuccess) {
      cudaFreeHost(st->ring_host);
      st->ring_host = nullptr;
      return cuda_error(e, "cudaMalloc(descriptor ring)");
    }
    st->ring_cap = cap;
    st->ring_head = 0;
  }
  while (!st->inflight.empty()) {  // reclaim finished regions, non-blocking
    int rc = retire_front(st, false);
    if (rc == 1) break;
    if (rc) return rc;
  }
  size_t start = st->ring_head;
  if (start + bytes > st->ring_cap) start = 0;
  for (;;) {
    bool clash = false;
    for (const Region& r : st->inflight)
      if (r.begin < start + bytes && start < r.end) {
        clash = true;
        break;
      }
    if (!clash) break;
    int rc = retire_front(st, true);
    if (rc) return rc;
  }
  st->ring_head = start + bytes;
  *off = start;
  return KVX_OK;
}

int ring_release_on(DeviceState* st, size_t off, size_t bytes, cudaStream_t s) {
  cudaEvent_t ev;
  int rc = take_event(st, &ev);
  if (rc) return rc;
  KVX_CUDA(cudaEventRecord(ev, s));
  st->inflight.push_back(Region{ev, off, off + ((bytes + 255) & ~size_t(255))});
  return KVX_OK;
}

int pipeline_ready(Staging* sg) {
  if (sg->helper) return KVX_OK;
  KVX_CUDA(cudaStreamCreateWithFlags(&sg->helper, cudaStreamNonBlocking));
  KVX_CUDA(cudaEventCreateWithFlags(&sg->ev_start, cudaEventDisableTiming));
  for (int b = 0; b < 2; ++b) {
    KVX_CUDA(cudaEventCreateWithFlags(&sg->ev_dev[b], cudaEventDisableTiming));
    KVX_CUDA(cudaEventCreateWithFlags(&sg->ev_link[b], cudaEventDisableTiming));
  }
  return KVX_OK;
}

int run_streams_ready(Staging* sg, int k) {
  if (!sg->run_fork) KVX_CUDA(cudaEventCreateWithFlags(&sg->run_fork, cudaEventDisableTiming));
  for (int j = 0; j < k; ++j) {
    if (sg->run_stream[j]) continue;
    KVX_CUDA(cudaStreamCreateWithFlags(&sg->run_stream[j], cudaStreamNonBlocking));
    KVX_CUDA(cudaEventCreateWithFlags(&sg->run_done[j], cudaEventDisableTiming));
  }
  return KVX_OK;
}

int staging_get(DeviceState* st, int idx, size_t want, cudaStream_t s,
                Staging** out) {
  Staging& sg = st->staging[idx];
  if (!sg.dev || sg.cap < want) {
    if (sg.dev) {
      if (sg.used) KVX_CUDA(cudaEventSynchronize(sg.last));
      cudaFree(sg.dev);
      sg.dev = nullptr;
    }
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&sg.dev), want);
    if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(staging)");
    sg.cap = want;
    sg.used = false;
    if (!sg.last) KVX_CUDA(cudaEventCreateWithFlags(&sg.last, cudaEventDisableTiming));
  }
  if (sg.used) KVX_CUDA(cudaStreamWaitEvent(s, sg.last, 0));
  *out = &sg;
  return KVX_OK;
}

// ---- kernel launch ---------------------------------------------------------
enum class Path { kHostSrc, kHostDst, kDevice, kPeer };

// Both sides device memory: this GPU's own, or a peer's mapped over NVLink
// (the TMA bulk kernel may serve these; host memory goes through the SMs).
bool device_side(Path p) { return p == Path::kDevice || p == Path::kPeer; }

// Grid of the vector kernel for a launch of n_tiles 32 KiB tiles.  Each CTA
// copies one contiguous span of tiles.  With a host side: host_path_ctas (the
// two directions' kernels share the SMs).  Device-only: about 4 tiles per
// CTA, between 4 and 16 CTAs per SM (2 resident, so up to 8 waves): large
// launches get short spans that balance across the SMs, small ones keep a
// few tiles per CTA.  An explicit setting overrides either (for a host side:
// sm_ctas_host_out / sm_ctas_host_in before sm_ctas_host).
uint32_t vec_grid(const DeviceState* st, Path p, const Tunables& tn, uint32_t n_tiles) {
  uint64_t ctas;
  if (p == Path::kHostSrc || p == Path::kHostDst) {
    const bool to_host = p == Path::kHostDst;
    const int64_t one_way = to_host ? tn.sm_ctas_host_out : tn.sm_ctas_host_in;
    ctas = one_way > 0              ? uint64_t(one_way)
           : tn.sm_ctas_host > 0 ? uint64_t(tn.sm_ctas_host)
                                 : host_path_ctas(st->sms, to_host);
  } else if (tn.sm_ctas_dev > 0) {
    ctas = uint64_t(tn.sm_ctas_dev);
  } else {
    ctas = std::min<uint64_t>(std::max<uint64_t>(n_tiles / 4, 4ull * st->sms), 16ull * st->sms);
  }
  return uint32_t(std::min<uint64_t>(n_tiles, ctas));
}

// Grid of the TMA bulk kernel for n_tiles 16 KiB chunks: about 8 chunks per
// CTA (its 6-stage ring needs a few to pay for its set-up), at least one wave
// of resident CTAs, at most bulk_waves waves.
uint32_t bulk_grid(const DeviceState* st, const Tunables& tn, uint32_t n_tiles) {
  const uint64_t resident = uint64_t(tn.bulk_ctas_per_sm) * uint64_t(st->sms);
  const uint64_t cap = resident * uint64_t(std::max<int64_t>(tn.bulk_waves, 1));
  const uint64_t ctas = std::min<uint64_t>(std::max<uint64_t>(n_tiles / 8, resident), cap);
  return uint32_t(std::min<uint64_t>(n_tiles, ctas));
}

bool all_aligned16(const std::vector<Copy>& v) {
  for (const Copy& c : v)
    if ((c.src | c.dst | c.len) & 15) return false;
  return true;
}

// Tables of every launch of one call, uploaded with one copy.
struct Upload {
  std::vector<char> bytes;
  size_t add(const void* p, size_t n) {
    const size_t off = (bytes.size() + 255) & ~size_t(255);
    bytes.resize(off + n);
    if (n) std::memcpy(bytes.data() + off, p, n);
    return off;
  }
};

struct Launch {
  bool grid = false;     // grid list (entries x segments) or item list
  size_t table_off = 0;  // byte offset of the items / grid entries in the upload
  size_t segs_off = 0;   // grid: byte offset of the segment table
  uint32_t n = 0;        // items or entries
  uint32_t n_tiles = 0;
  bool bulk = false;
  Path path = Path::kDevice;
  uint64_t bytes = 0;    // payload bytes of this launch
};

// HBM bytes a launch moves on this GPU: read + write when both sides are
// local, one side when the other is host or peer memory.
uint64_t hbm_bytes_of(const Launch& l) {
  return l.path == Path::kDevice ? 2 * l.bytes : l.bytes;
}

uint64_t payload_of(const std::vector<Copy>& v) {
  uint64_t b = 0;
  for (const Copy& c : v) b += c.len;
  return b;
}

int upload(DeviceState* st, const Upload& up, cudaStream_t s, size_t* ring_off) {
  const size_t bytes = up.bytes.size();
  int rc = ring_acquire(st, bytes ? bytes : 256, ring_off);
  if (rc) return rc;
  if (bytes) {
    std::memcpy(st->ring_host + *ring_off, up.bytes.data(), bytes);
    KVX_CUDA(cudaMemcpyAsync(st->ring_dev + *ring_off, st->ring_host + *ring_off, bytes,
                             cudaMemcpyHostToDevice, s));
  }
  return KVX_OK;
}

int release(DeviceState* st, size_t ring_off, const Upload& up, cudaStream_t s) {
  return ring_release_on(st, ring_off, up.bytes.size() ? up.bytes.size() : 256, s);
}

int ensure_bulk(DeviceState* st) {
  if (st->bulk_ready) return KVX_OK;
  KVX_CUDA(cudaFuncSetAttribute(kvx_copy_bulk<ItemList>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, int(kBulkSmem)));
  KVX_CUDA(cudaFuncSetAttribute(kvx_copy_bulk<GridList>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, int(kBulkSmem)));
  st->bulk_ready = true;
  return KVX_OK;
}

constexpr uint32_t kVecShift = 15;
constexpr uint32_t kVecTile = 1u << kVecShift;  // 32 KiB

template <class List>
void launch_list(const List& list, const Launch& l, const DeviceState* st, cudaStream_t s,
                 const Tunables& tn) {
  if (l.bulk) {
    // Up to two 96 KiB CTAs fit on an SM.
    const uint32_t grid = bulk_grid(st, tn, l.n_tiles);
    kvx_copy_bulk<List><<<grid, 32, kBulkSmem, s>>>(list, l.n_tiles);
  } else {
    const uint32_t grid = vec_grid(st, l.path, tn, l.n_tiles);
    const bool host_src = l.path == Path::kHostSrc;
    if (tn.vec_bytes == 32) {
      if (host_src)
        kvx_copy_vec<kSrcHost, List, 32><<<grid, kVecThreads, 0, s>>>(list, l.n_tiles, kVecShift);
      else
        kvx_copy_vec<kSrcDevice, List, 32><<<grid, kVecThreads, 0, s>>>(list, l.n_tiles,
                                                                        kVecShift);
    } else if (host_src) {
      kvx_copy_vec<kSrcHost, List><<<grid, kVecThreads, 0, s>>>(list, l.n_tiles, kVecShift);
    } else {
      kvx_copy_vec<kSrcDevice, List><<<grid, kVecThreads, 0, s>>>(list, l.n_tiles, kVecShift);
    }
  }
}

int launch_kernel(DeviceState* st, size_t ring_off, const Launch& l, cudaStream_t s,
                  const Tunables& tn) {
  if (l.bulk) {
    int rc = ensure_bulk(st);
    if (rc) return rc;
  }
  const char* base = st->ring_dev + ring_off;
  if (l.grid)
    launch_list(GridList{reinterpret_cast<const GridEntry*>(base + l.table_off), l.n,
                         reinterpret_cast<const GridSeg*>(base + l.segs_off)},
                l, st, s, tn);
  else
    launch_list(ItemList{reinterpret_cast<const Item*>(base + l.table_off), l.n}, l, st, s, tn);
  KVX_CUDA(cudaGetLastError());
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return KVX_OK;
}

// Runs `launch` (one kernel launch), bracketed by timing events when timing
// is enabled.
template <class F>
int timed(const DeviceState* st, const Launch& l, cudaStream_t s, F&& launch) {
  if (!g_timing.load(std::memory_order_relaxed)) return launch();
  TimedLaunch t{st->device, nullptr, nullptr, hbm_bytes_of(l)};
  KVX_CUDA(cudaEventCreate(&t.begin));
  KVX_CUDA(cudaEventCreate(&t.end));
  KVX_CUDA(cudaEventRecord(t.begin, s));
  int rc = launch();
  KVX_CUDA(cudaEventRecord(t.end, s));
  std::lock_guard<std::mutex> g(g_timing_mu);
  g_timed.push_back(t);
  return rc;
}

int launch_one(DeviceState* st, size_t ring_off, const Launch& l, cudaStream_t s,
               const Tunables& tn) {
  if (l.n_tiles == 0) return KVX_OK;
  return timed(st, l, s, [&] { return launch_kernel(st, ring_off, l, s, tn); });
}

// Grid plans up to kInlineRecordsMax records (entries + segments) go to the
// kernel in its parameters: no descriptor upload, no ring fence.
bool fits_inline(const GridPlan& p) {
  return p.entries.size() + p.segs.size() <= kInlineRecordsMax;
}

template <class InlineList>
int launch_inline_as(const DeviceState* st, const GridPlan& p, const Launch& l, cudaStream_t s,
                     const Tunables& tn) {
  InlineList list;
  list.n = uint32_t(p.entries.size());
  list.n_segs = uint32_t(p.segs.size());
  std::memcpy(list.rec, p.entries.data(), p.entries.size() * sizeof(GridEntry));
  std::memcpy(list.rec + 2 * list.n, p.segs.data(), p.segs.size() * sizeof(GridSeg));
  const uint32_t grid = vec_grid(st, l.path, tn, l.n_tiles);
  const bool host_src = l.path == Path::kHostSrc;
  if (tn.vec_bytes == 32) {
    if (host_src)
      kvx_copy_vec_inline<kSrcHost, 32, InlineList><<<grid, kVecThreads, 0, s>>>(list, l.n_tiles,
                                                                                 kVecShift);
    else
      kvx_copy_vec_inline<kSrcDevice, 32, InlineList><<<grid, kVecThreads, 0, s>>>(
          list, l.n_tiles, kVecShift);
  } else if (host_src) {
    kvx_copy_vec_inline<kSrcHost, 16, InlineList><<<grid, kVecThreads, 0, s>>>(list, l.n_tiles,
                                                                               kVecShift);
  } else {
    kvx_copy_vec_inline<kSrcDevice, 16, InlineList><<<grid, kVecThreads, 0, s>>>(list, l.n_tiles,
                                                                                 kVecShift);
  }
  KVX_CUDA(cudaGetLastError());
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return KVX_OK;
}

// One vector-kernel launch of a finalized grid plan passed by value, in the
// smallest parameter-space list that holds it.
int launch_inline(DeviceState* st, const GridPlan& p, const Launch& l, cudaStream_t s,
                  const Tunables& tn) {
  if (l.n_tiles == 0) return KVX_OK;
  const size_t records = p.entries.size() + p.segs.size();
  return timed(st, l, s, [&] {
    if (records <= kInlineRecords) return launch_inline_as<InlineGridList>(st, p, l, s, tn);
    if (records <= kInlineRecordsMid) return launch_inline_as<InlineGridListMid>(st, p, l, s, tn);
    return launch_inline_as<InlineGridListMax>(st, p, l, s, tn);
  });
}

// Append an item-list launch for `copies` (one wave, coalesced by the caller).
int add_items(Upload* up, std::vector<Launch>* launches, const std::vector<Copy>& copies,
              Path path, bool bulk) {
  std::vector<Item> items;
  const uint64_t tiles = build_items(copies, bulk ? kBulkChunk : kVecTile, &items);
  if (tiles > 0xffffffffull)
    return set_error(KVX_ERR_INVALID_ARGUMENT, "request too large for one launch");
  Launch l;
  l.table_off = up->add(items.data(), items.size() * sizeof(Item));
  l.n = uint32_t(items.size());
  l.n_tiles = uint32_t(tiles);
  l.bulk = bulk;
  l.path = path;
  l.bytes = payload_of(copies);
  launches->push_back(l);
  return KVX_OK;
}

bool grid_aligned16(const GridPlan& p) {
  for (const GridSeg& g : p.segs)
    if ((g.src_base | g.src_stride | g.dst_base | g.dst_stride) & 15) return false;
  for (const GridEntry& e : p.entries)
    if ((e.off | e.len) & 15) return false;
  return true;
}

// Append a grid launch (finalizes `p` for the chosen tile size).
int add_grid(Upload* up, std::vector<Launch>* launches, GridPlan* p, Path path, bool bulk) {
  const uint64_t tiles = grid_finalize(p, bulk ? kBulkShift : kVecShift);
  if (tiles > 0xffffffffull)
    return set_error(KVX_ERR_INVALID_ARGUMENT, "request too large for one launch");
  Launch l;
  l.grid = true;
  l.table_off = up->add(p->entries.data(), p->entries.size() * sizeof(GridEntry));
  l.segs_off = up->add(p->segs.data(), p->segs.size() * sizeof(GridSeg));
  l.n = uint32_t(p->entries.size());
  l.n_tiles = uint32_t(tiles);
  l.bulk = bulk;
  l.path = path;
  l.bytes = p->copied;
  launches->push_back(l);
  return KVX_OK;
}

int run_launches(DeviceState* st, const Upload& up, const std::vector<Launch>& launches,
                 cudaStream_t s, const Tunables& tn) {
  size_t off = 0;
  int rc = upload(st, up, s, &off);
  if (rc) return rc;
  for (const Launch& l : launches) {
    rc = launch_one(st, off, l, s, tn);
    if (rc) return rc;
  }
  return release(st, off, up, s);
}

// Run waves of device-visible copies through the SM kernels (one launch per
// wave, one descriptor upload for all of them).
int run_sm(DeviceState* st, const std::vector<Copy>& copies,
           const std::vector<size_t>& waves, Path path, bool allow_bulk,
           cudaStream_t s, const Tunables& tn) {
  Upload up;
  std::vector<Launch> launches;
  size_t begin = 0;
  for (size_t end : waves) {
    std::vector<Copy> w(copies.begin() + begin, copies.begin() + end);
    begin = end;
    coalesce(&w);
    const bool bulk = allow_bulk && (device_side(path) || tn.host_bulk) && all_aligned16(w);
    int rc = add_items(&up, &launches, w, path, bulk);
    if (rc) return rc;
  }
  return run_launches(st, up, launches, s, tn);
}

// One grid launch through the SM kernels.
int run_sm_grid(DeviceState* st, GridPlan* p, Path path, bool allow_bulk, cudaStream_t s,
                const Tunables& tn) {
  Upload up;
  std::vector<Launch> launches;
  const bool bulk = allow_bulk && (device_side(path) || tn.host_bulk) && grid_aligned16(*p);
  int rc = add_grid(&up, &launches, p, path, bulk);
  if (rc) return rc;
  if (!bulk && tn.inline_lists && fits_inline(*p))
    return launch_inline(st, *p, launches.front(), s, tn);
  return run_launches(st, up, launches, s, tn);
}

size_t staging_cap(const Tunables& tn) {
  return size_t(std::max<int64_t>(tn.staging_bytes, 1 << 20)) & ~size_t(4095);
}

// Copy-engine path through a staging area.  `copies` use the caller's host
// addresses; host_is_src selects the direction.
int run_ce_staged(DeviceState* st, const std::vector<Copy>& copies,
                  const std::vector<size_t>& waves, bool host_is_src,
                  bool allow_bulk, cudaStream_t s, const Tunables& tn) {
  if (payload_of(copies) == 0) return KVX_OK;
  Staging* sg = nullptr;
  int rc = staging_get(st, host_is_src ? 1 : 0, staging_cap(tn), s, &sg);
  if (rc) return rc;
  const uint64_t sbase = reinterpret_cast<uint64_t>(sg->dev);
  // Build every chunk's item table first (one upload).
  std::vector<StagedChunk> all_chunks;
  Upload up;
  std::vector<Launch> launches;
  size_t begin = 0;
  for (size_t end : waves) {
    std::vector<Copy> w(copies.begin() + begin, copies.begin() + end);
    begin = end;
    std::vector<StagedChunk> chunks;
    plan_staged(w, host_is_src, std::min<uint64_t>(sg->cap, staging_cap(tn)), &chunks);
    for (StagedChunk& ch : chunks) {
      for (Copy& m : ch.device_moves) (host_is_src ? m.src : m.dst) += sbase;
      rc = add_items(&up, &launches, ch.device_moves, Path::kDevice,
                     allow_bulk && all_aligned16(ch.device_moves));
      if (rc) return rc;
      all_chunks.push_back(std::move(ch));
    }
  }
  size_t off = 0;
  rc = upload(st, up, s, &off);
  if (rc) return rc;
  for (size_t i = 0; i < all_chunks.size(); ++i) {
    const StagedChunk& ch = all_chunks[i];
    if (host_is_src) {
      for (const Copy& r : ch.host_runs)
        KVX_CUDA(cudaMemcpyAsync(sg->dev + r.dst, reinterpret_cast<const void*>(r.src), r.len,
                                 cudaMemcpyHostToDevice, s));
      rc = launch_one(st, off, launches[i], s, tn);
      if (rc) return rc;
    } else {
      rc = launch_one(st, off, launches[i], s, tn);
      if (rc) return rc;
      for (const Copy& r : ch.host_runs)
        KVX_CUDA(cudaMemcpyAsync(reinterpret_cast<void*>(r.dst), sg->dev + r.src, r.len,
                                 cudaMemcpyDeviceToHost, s));
    }
  }
  KVX_CUDA(cudaEventRecord(sg->last, s));
  sg->used = true;
  return release(st, off, up, s);
}

// Host ids of a swap grid plan, sorted, with the order of the entries.
std::vector<std::pair<int64_t, uint32_t>> host_order(const GridPlan& p) {
  std::vector<std::pair<int64_t, uint32_t>> v;
  v.reserve(p.entries.size());
  for (uint32_t i = 0; i < p.entries.size(); ++i)
    v.emplace_back(p.host_side == 1 ? p.entries[i].src_id : p.entries[i].dst_id, i);
  std::sort(v.begin(), v.end());
  return v;
}

// Mean bytes of the host-contiguous runs of a swap grid plan.
uint64_t grid_mean_run(const GridPlan& p) {
  if (p.entries.empty() || !p.row_span) return 0;
  const auto v = host_order(p);
  uint64_t runs = 1;
  for (size_t i = 1; i < v.size(); ++i)
    if (!(p.row_stride == p.row_span && v[i].first == v[i - 1].first + 1)) ++runs;
  return p.copied / runs;
}

// Copy-engine path for a swap grid plan whose entries write whole composite
// spans.  The staging area is split in two halves laid out as consecutive
// spans in host-row order.  Swap-out: the gather kernel fills half k%2 on an
// internal helper stream while the copy engines drain the other half on the
// caller's stream (one cudaMemcpyAsync per run of consecutive host rows).
// Swap-in: the copy engines fill half k%2 on the caller's stream while the
// scatter kernel empties the other half on the helper stream.  Events order
// every reuse of a half; the caller's stream ends after all of it.
int run_ce_grid(DeviceState* st, const GridPlan& p, cudaStream_t s, const Tunables& tn) {
  const bool host_is_src = p.host_side == 1;
  const uint64_t span = p.row_span;
  Staging* sg = nullptr;
  int rc = staging_get(st, host_is_src ? 1 : 0, staging_cap(tn), s, &sg);
  if (rc) return rc;
  rc = pipeline_ready(sg);
  if (rc) return rc;
  // The area may be larger than the current setting (it is kept, not
  // shrunk); chunks follow the setting.
  const uint64_t cap_eff = std::min<uint64_t>(sg->cap, staging_cap(tn));
  const uint64_t half = cap_eff / 2;
  // Pipeline (opt-in) only when the call needs more than one half-area chunk.
  // Measured on B200: +1-3% for one direction alone, but with swap-out and
  // swap-in running at once the two extra helper streams couple the
  // directions through the device's hardware queues (72-92 GB/s instead of
  // a steady 91), so it is off by default.
  const bool pipelined = tn.ce_pipeline > 0 && half >= span && p.entries.size() > half / span;
  const uint64_t rows = (pipelined ? half : cap_eff) / span;
  const uint64_t sbase = reinterpret_cast<uint64_t>(sg->dev);
  const auto order = host_order(p);
  struct Run {
    uint64_t host, staging, len;
  };
  std::vector<std::vector<Run>> runs;
  std::vector<int> buf_of;
  Upload up;
  std::vector<Launch> launches;
  size_t chunk_index = 0;
  for (size_t c0 = 0; c0 < order.size(); c0 += rows, ++chunk_index) {
    const size_t c1 = std::min<size_t>(order.size(), c0 + rows);
    const int b = pipelined ? int(chunk_index & 1) : 0;
    const uint64_t base = sbase + uint64_t(b) * half;
    GridPlan chunk;
    chunk.segs = p.segs;  // staging side: segment s at its cpu offset in a span
    for (GridSeg& g : chunk.segs) {
      if (host_is_src) {
        g.src_base = base + (g.src_base - p.row_base);
        g.src_stride = span;
      } else {
        g.dst_base = base + (g.dst_base - p.row_base);
        g.dst_stride = span;
      }
    }
    chunk.entries.reserve(c1 - c0);
    std::vector<Run> rr;
    for (size_t k = c0; k < c1; ++k) {
      GridEntry e = p.entries[order[k].second];
      const int64_t pos = int64_t(k - c0);
      if (host_is_src) e.src_id = pos; else e.dst_id = pos;
      chunk.entries.push_back(e);
      chunk.copied += uint64_t(e.len) * chunk.segs.size();
      const uint64_t h = p.row_base + uint64_t(order[k].first) * p.row_stride;
      const uint64_t st_off = uint64_t(b) * half + uint64_t(pos) * span;
      if (!rr.empty() && rr.back().host + rr.back().len == h &&
          rr.back().staging + rr.back().len == st_off)
        rr.back().len += span;
      else
        rr.push_back(Run{h, st_off, span});
    }
    rc = add_grid(&up, &launches, &chunk, Path::kDevice,
                  tn.staging_bulk && grid_aligned16(chunk));
    if (rc) return rc;
    runs.push_back(std::move(rr));
    buf_of.push_back(b);
  }
  size_t off = 0;
  rc = upload(st, up, s, &off);  // the table copy is ordered on s, before ev_start
  if (rc) return rc;
  // Short host runs: the copies of each chunk go round-robin over k streams
  // forked from s (and joined back into s), so copy engines overlap their
  // per-copy gaps.
  size_t n_runs = 0;
  for (const auto& rr : runs) n_runs += rr.size();
  int k_streams = 1;
  if (!pipelined && tn.ce_streams > 1 && n_runs > 1 &&
      p.copied / std::max<size_t>(n_runs, 1) <= uint64_t(tn.ce_streams_max_run)) {
    k_streams = int(std::min<int64_t>(tn.ce_streams, int64_t(n_runs)));
    rc = run_streams_ready(sg, k_streams);
    if (rc) return rc;
  }
  const uint64_t piece = tn.ce_max_copy > 0 ? uint64_t(tn.ce_max_copy) : ~uint64_t(0);
  auto copy_runs = [&](const std::vector<Run>& rr) -> int {
    if (k_streams == 1) {
      for (const Run& r : rr) {
        for (uint64_t o = 0; o < r.len; o += piece) {
          const uint64_t len = std::min(piece, r.len - o);
          if (host_is_src)
            KVX_CUDA(cudaMemcpyAsync(sg->dev + r.staging + o,
                                     reinterpret_cast<const void*>(r.host + o), len,
                                     cudaMemcpyHostToDevice, s));
          else
            KVX_CUDA(cudaMemcpyAsync(reinterpret_cast<void*>(r.host + o),
                                     sg->dev + r.staging + o, len, cudaMemcpyDeviceToHost, s));
        }
      }
      return KVX_OK;
    }
    KVX_CUDA(cudaEventRecord(sg->run_fork, s));
    for (int j = 0; j < k_streams; ++j)
      KVX_CUDA(cudaStreamWaitEvent(sg->run_stream[j], sg->run_fork, 0));
    for (size_t i = 0; i < rr.size(); ++i) {
      const Run& r = rr[i];
      cudaStream_t q = sg->run_stream[i % size_t(k_streams)];
      if (host_is_src)
        KVX_CUDA(cudaMemcpyAsync(sg->dev + r.staging, reinterpret_cast<const void*>(r.host),
                                 r.len, cudaMemcpyHostToDevice, q));
      else
        KVX_CUDA(cudaMemcpyAsync(reinterpret_cast<void*>(r.host), sg->dev + r.staging, r.len,
                                 cudaMemcpyDeviceToHost, q));
    }
    for (int j = 0; j < k_streams; ++j) {
      KVX_CUDA(cudaEventRecord(sg->run_done[j], sg->run_stream[j]));
      KVX_CUDA(cudaStreamWaitEvent(s, sg->run_done[j], 0));
    }
    return KVX_OK;
  };
  cudaStream_t h = pipelined ? sg->helper : s;
  if (pipelined) {
    KVX_CUDA(cudaEventRecord(sg->ev_start, s));
    KVX_CUDA(cudaStreamWaitEvent(h, sg->ev_start, 0));
  }
  for (size_t i = 0; i < launches.size(); ++i) {
    const int b = buf_of[i];
    if (host_is_src) {
      if (pipelined && i >= 2) KVX_CUDA(cudaStreamWaitEvent(s, sg->ev_dev[b], 0));
      rc = copy_runs(runs[i]);
      if (rc) return rc;
      if (pipelined) {
        KVX_CUDA(cudaEventRecord(sg->ev_link[b], s));
        KVX_CUDA(cudaStreamWaitEvent(h, sg->ev_link[b], 0));
      }
      rc = launch_one(st, off, launches[i], h, tn);
      if (rc) return rc;
      if (pipelined) KVX_CUDA(cudaEventRecord(sg->ev_dev[b], h));
    } else {
      if (pipelined && i >= 2) KVX_CUDA(cudaStreamWaitEvent(h, sg->ev_link[b], 0));
      rc = launch_one(st, off, launches[i], h, tn);
      if (rc) return rc;
      if (pipelined) {
        KVX_CUDA(cudaEventRecord(sg->ev_dev[b], h));
        KVX_CUDA(cudaStreamWaitEvent(s, sg->ev_dev[b], 0));
      }
      rc = copy_runs(runs[i]);
      if (rc) return rc;
      if (pipelined) KVX_CUDA(cudaEventRecord(sg->ev_link[b], s));
    }
  }
  // Swap-in: the caller's stream ends after the last scatter (the helper
  // stream runs its kernels in order).
  if (pipelined && host_is_src && !launches.empty())
    KVX_CUDA(cudaStreamWaitEvent(s, sg->ev_dev[buf_of.back()], 0));
  KVX_CUDA(cudaEventRecord(sg->last, s));
  sg->used = true;
  return release(st, off, up, s);
}

// One copy-engine copy per coalesced extent (no staging, no kernel).
// `merge` coalesces neighbours that are contiguous on both sides; callers
// whose copies may span several tensors (segments) and are not merged per
// segment already pass false, since one copy-engine copy must stay inside one
// allocation.
int run_ce_extent(const std::vector<Copy>& copies, const std::vector<size_t>& waves,
                  cudaStream_t s, bool merge = true) {
  size_t begin = 0;
  for (size_t end : waves) {
    std::vector<Copy> w(copies.begin() + begin, copies.begin() + end);
    begin = end;
    if (merge) coalesce(&w);
    for (const Copy& c : w)
      KVX_CUDA(cudaMemcpyAsync(reinterpret_cast<void*>(c.dst),
                               reinterpret_cast<const void*>(c.src), c.len,
                               cudaMemcpyDefault, s));
  }
  return KVX_OK;
}

// The (entry x segment) copies of a grid plan, for the paths that need a copy
// list (one copy per entry and segment).
std::vector<Copy> grid_copies(GridPlan p) {
  grid_finalize(&p, 31);
  std::vector<Copy> v;
  grid_expand(p, 31, &v);
  return v;
}

// The same copies for one copy-engine copy per extent: segment by segment,
// entries in source order, neighbours coalesced only inside a segment.  A
// grid plan's copies never conflict (distinct targets, no overlap between the
// sides), so their order is free, and consecutive blocks of one segment merge
// into one copy.  Copies are never merged across segments: two segment
// tensors may sit next to each other in the virtual address space while
// belonging to different allocations (or, on a peer, to different IPC
// mappings), and one copy-engine copy must stay inside one allocation.
std::vector<Copy> grid_extents(const GridPlan& p) {
  std::vector<uint32_t> order(p.entries.size());
  for (uint32_t i = 0; i < order.size(); ++i) order[i] = i;
  std::sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
    const GridEntry& x = p.entries[a];
    const GridEntry& y = p.entries[b];
    return x.src_id != y.src_id ? x.src_id < y.src_id : x.off < y.off;
  });
  std::vector<Copy> v;
  v.reserve(p.entries.size() * p.segs.size());
  for (const GridSeg& g : p.segs) {
    const size_t first = v.size();
    for (uint32_t i : order) {
      const GridEntry& e = p.entries[i];
      if (e.len == 0) continue;
      const Copy c{g.src_base + uint64_t(e.src_id) * g.src_stride + e.off,
                   g.dst_base + uint64_t(e.dst_id) * g.dst_stride + e.off, e.len};
      if (v.size() > first && v.back().src + v.back().len == c.src &&
          v.back().dst + v.back().len == c.dst)
        v.back().len += c.len;
      else
        v.push_back(c);
    }
  }
  return v;
}

// Host memory facts for the SM path.
struct HostInfo {
  bool mapped = false;     // device can address it
  uint64_t dev_base = 0;   // device-visible address of `ptr`
};

HostInfo host_info(const void* ptr, int device) {
  HostInfo h;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
    cudaGetLastError();
    return h;
  }
  if (a.type == cudaMemoryTypeHost && a.devicePointer) {
    h.mapped = true;
    h.dev_base = reinterpret_cast<uint64_t>(a.devicePointer);
  } else if (a.type == cudaMemoryTypeManaged) {
    h.mapped = true;
    h.dev_base = reinterpret_cast<uint64_t>(ptr);
  }
  (void)device;
  return h;
}

int check_device_memory(const void* ptr, int device, const char* what) {
  cudaPointerAttributes a;
  cudaError_t e = cudaPointerGetAttributes(&a, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(KVX_ERR_INVALID_ARGUMENT, std::string(what) + " is not CUDA memory");
  }
  if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged)
    return set_error(KVX_ERR_INVALID_ARGUMENT, std::string(what) + " is not device memory");
  if (a.type == cudaMemoryTypeDevice && a.device != device)
    return set_error(KVX_ERR_INVALID_ARGUMENT,
                     std::string(what) + " lives on device " + std::to_string(a.device) +
                         ", not on the current device " + std::to_string(device));
  return KVX_OK;
}

// Execute host<->device copies (caller host addresses) in the chosen mode.
int execute_host_copies(DeviceState* st, std::vector<Copy>& copies, bool is_swap_in,
                        const HostInfo& hi, uint64_t host_caller_base, int mode,
                        cudaStream_t s) {
  const Tunables tn = tunables();
  if (copies.empty()) {
    t_last_mode = mode == KVX_MODE_AUTO ? KVX_MODE_SM : mode;
    return KVX_OK;
  }
  if (mode == KVX_MODE_AUTO) {
    if (!hi.mapped) {
      mode = KVX_MODE_CE;
    } else if (tn.direct_max > 0 && copies.size() <= uint64_t(tn.direct_max)) {
      mode = KVX_MODE_CE_EXTENT;
    } else if (payload_of(copies) < uint64_t(std::max<int64_t>(tn.ce_min_bytes, 0))) {
      mode = KVX_MODE_SM;
    } else {
      const uint64_t run = mean_host_run(copies, is_swap_in);
      mode = (tn.ce_min_run > 0 && run >= uint64_t(tn.ce_min_run)) ? KVX_MODE_CE : KVX_MODE_SM;
    }
  }
  if (mode == KVX_MODE_SM_BULK) mode = KVX_MODE_SM;  // bulk is device-only
  const std::vector<size_t> waves = split_waves(copies);
  int rc;
  if (mode == KVX_MODE_SM) {
    if (!hi.mapped)
      return set_error(KVX_ERR_HOST_MEMORY,
                       "host buffer is not page-locked/device-mapped; the SM mode "
                       "needs cudaHostAlloc or cudaHostRegister memory");
    const uint64_t delta = hi.dev_base - host_caller_base;  // modular
    for (Copy& c : copies) (is_swap_in ? c.src : c.dst) += delta;
    rc = run_sm(st, copies, waves, is_swap_in ? Path::kHostSrc : Path::kHostDst,
                tn.host_bulk != 0, s, tn);
  } else if (mode == KVX_MODE_CE) {
    rc = run_ce_staged(st, copies, waves, is_swap_in, tn.staging_bulk != 0, s, tn);
  } else if (mode == KVX_MODE_CE_EXTENT) {
    rc = run_ce_extent(copies, waves, s);
  } else {
    return set_error(KVX_ERR_INVALID_ARGUMENT, "unknown transfer mode " + std::to_string(mode));
  }
  if (rc == KVX_OK) t_last_mode = mode;
  return rc;
}

// Small plans that end up as at most `direct_max` coalesced copies: those
// copies (one copy-engine copy each beats a kernel launch).  Only plans of at
// most 16 copies are expanded to check.
bool direct_copies(const GridPlan& p, const Tunables& tn, std::vector<Copy>* out) {
  if (tn.direct_max <= 0 || p.entries.size() * p.segs.size() > 16) return false;
  std::vector<Copy> v = grid_extents(p);
  if (v.size() > uint64_t(tn.direct_max)) return false;
  *out = std::move(v);
  return true;
}

// Execute a swap grid plan (built with the caller's host addresses).
int execute_grid_host(DeviceState* st, GridPlan* p, const HostInfo& hi,
                      uint64_t host_caller_base, int mode, cudaStream_t s) {
  const Tunables tn = tunables();
  const bool is_swap_in = p->host_side == 1;
  if (p->entries.empty()) {
    t_last_mode = mode == KVX_MODE_AUTO ? KVX_MODE_SM : mode;
    return KVX_OK;
  }
  // Partial extents leave gaps in the host rows: their host runs come from the
  // expanded copy list (computed once, reused by the copy-engine path).
  std::vector<Copy> expanded;
  const bool partial = p->row_span == 0;
  if (mode == KVX_MODE_AUTO) {
    if (!hi.mapped) {
      mode = KVX_MODE_CE;
    } else if (direct_copies(*p, tn, &expanded)) {
      mode = KVX_MODE_CE_EXTENT;
    } else if (tn.ce_min_run <= 0 || p->copied < uint64_t(std::max<int64_t>(tn.ce_min_bytes, 0))) {
      mode = KVX_MODE_SM;
    } else if (!partial) {
      mode = grid_mean_run(*p) >= uint64_t(tn.ce_min_run) ? KVX_MODE_CE : KVX_MODE_SM;
    } else {
      expanded = grid_copies(*p);
      mode = mean_host_run(expanded, is_swap_in) >= uint64_t(tn.ce_min_run) ? KVX_MODE_CE
                                                                           : KVX_MODE_SM;
    }
  }
  if (mode == KVX_MODE_SM_BULK) mode = KVX_MODE_SM;  // bulk is device-only
  int rc;
  if (mode == KVX_MODE_SM) {
    if (!hi.mapped)
      return set_error(KVX_ERR_HOST_MEMORY,
                       "host buffer is not page-locked/device-mapped; the SM mode "
                       "needs cudaHostAlloc or cudaHostRegister memory");
    const uint64_t delta = hi.dev_base - host_caller_base;  // modular
    for (GridSeg& g : p->segs) (is_swap_in ? g.src_base : g.dst_base) += delta;
    rc = run_sm_grid(st, p, is_swap_in ? Path::kHostSrc : Path::kHostDst, tn.host_bulk != 0,
                     s, tn);
  } else if (mode == KVX_MODE_CE) {
    if (p->row_span && p->row_span <= staging_cap(tn)) {
      rc = run_ce_grid(st, *p, s, tn);
    } else {
      if (expanded.empty()) expanded = grid_copies(*p);
      rc = run_ce_staged(st, expanded, {expanded.size()}, is_swap_in, tn.staging_bulk != 0, s,
                         tn);
    }
  } else if (mode == KVX_MODE_CE_EXTENT) {
    // (already set, ordered and coalesced, when AUTO chose direct copies)
    if (expanded.empty()) expanded = grid_extents(*p);
    rc = run_ce_extent(expanded, {expanded.size()}, s, /*merge=*/false);
  } else {
    return set_error(KVX_ERR_INVALID_ARGUMENT, "unknown transfer mode " + std::to_string(mode));
  }
  if (rc == KVX_OK) t_last_mode = mode;
  return rc;
}

// ---- weight upload (model switch) ------------------------------------------

// Persistent host threads for the pageable-upload copies: each call splits
// one memcpy into shares of at least 4 MiB that the pool's threads and the
// calling thread take in turn; the call returns when every share is copied.
// One job at a time (uploads of a device already serialize on its bounce
// buffers).  The pool is created on first use and lives until the process
// exits.
class CopyPool {
 public:
  static CopyPool& get() {
    static CopyPool* pool = new CopyPool();  // never destroyed: its threads outlive callers
    return *pool;
  }

  void copy(char* dst, const char* src, size_t n, int threads) {
    constexpr size_t kMinShare = size_t(4) << 20;
    const size_t parts = std::max<size_t>(
        1, std::min<size_t>(size_t(std::max(threads, 1)), n / kMinShare));
    if (parts == 1) {
      std::memcpy(dst, src, n);
      return;
    }
    std::lock_guard<std::mutex> one_job(call_mu_);
    grow(int(parts) - 1);
    auto job = std::make_shared<Job>();
    job->dst = dst;
    job->src = src;
    job->n = n;
    job->parts = parts;
    job->share = (n / parts + 4095) & ~size_t(4095);
    job->left.store(parts);
    {
      std::lock_guard<std::mutex> g(mu_);
      current_ = job;
      ++generation_;
    }
    cv_.notify_all();
    work(*job);
    std::unique_lock<std::mutex> g(job->mu);
    job->done_cv.wait(g, [&] { return job->left.load() == 0; });
  }

 private:
  struct Job {
    char* dst = nullptr;
    const char* src = nullptr;
    size_t n = 0, parts = 0, share = 0;
    std::atomic<size_t> next{0};
    std::atomic<size_t> left{0};
    std::mutex mu;
    std::condition_variable done_cv;
  };

  static void work(Job& job) {
    for (;;) {
      const size_t k = job.next.fetch_add(1);
      if (k >= job.parts) return;
      const size_t a = std::min(job.n, k * job.share);
      const size_t b = k + 1 == job.parts ? job.n : std::min(job.n, (k + 1) * job.share);
      if (a < b) std::memcpy(job.dst + a, job.src + a, b - a);
      if (job.left.fetch_sub(1) == 1) {
        std::lock_guard<std::mutex> g(job.mu);
        job.done_cv.notify_all();
      }
    }
  }

  void grow(int want) {
    while (int(workers_.size()) < want) {
      workers_.emplace_back([this] {
        uint64_t seen = 0;
        for (;;) {
          std::shared_ptr<Job> job;
          {
            std::unique_lock<std::mutex> g(mu_);
            cv_.wait(g, [&] { return generation_ != seen; });
            seen = generation_;
            job = current_;
          }
          if (job) work(*job);
        }
      });
    }
  }

  std::mutex call_mu_, mu_;
  std::condition_variable cv_;
  std::vector<std::thread> workers_;
  std::shared_ptr<Job> current_;
  uint64_t generation_ = 0;
};

void parallel_memcpy(char* dst, const char* src, size_t n, int threads) {
  CopyPool::get().copy(dst, src, n, threads);
}

int bounce_ready(DeviceState* st, size_t want) {
  if (st->bounce_cap >= want) return KVX_OK;
  for (int b = 0; b < 2; ++b) {
    if (st->bounce_used[b]) KVX_CUDA(cudaEventSynchronize(st->bounce_ev[b]));
    if (st->bounce[b]) cudaFreeHost(st->bounce[b]);
    st->bounce[b] = nullptr;
    st->bounce_used[b] = false;
  }
  st->bounce_cap = 0;
  for (int b = 0; b < 2; ++b) {
    cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&st->bounce[b]), want,
                                  cudaHostAllocDefault);
    if (e != cudaSuccess) return cuda_error(e, "cudaHostAlloc(upload bounce buffer)");
    if (!st->bounce_ev[b])
      KVX_CUDA(cudaEventCreateWithFlags(&st->bounce_ev[b], cudaEventDisableTiming));
  }
  st->bounce_cap = want;
  return KVX_OK;
}

// Page-locked or device-addressable host source: the copy engine reads it
// directly.
bool host_is_pinned(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost || a.type == cudaMemoryTypeManaged;
}

}  // namespace

// Sets the message kvx_last_error() returns to this thread (used by the
// entry points defined in other files of the library).
void record_error(const std::string& msg) { t_last_error = msg; }

}  // namespace kvx

struct kvx_layout {
  kvx::Layout L;
  kvx::HostInfo host;
  // Device that holds every segment page (-1: pages on several devices), found
  // by the first migration and kept: the page table never changes.
  int pages_device = -2;  // -2: not looked up yet
  std::mutex mu;
};

using namespace kvx;

namespace {
// Fills lay->pages_device on first use; every segment page must be device memory.
int pages_device(kvx_layout* lay) {
  std::lock_guard<std::mutex> g(lay->mu);
  if (lay->pages_device != -2) return KVX_OK;
  int dev = -2;
  for (uint64_t p : lay->L.seg_pages) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, reinterpret_cast<void*>(p)) != cudaSuccess) {
      cudaGetLastError();
      return set_error(KVX_ERR_INVALID_ARGUMENT, "segment pages are not CUDA memory");
    }
    if (a.type != cudaMemoryTypeDevice)
      return set_error(KVX_ERR_INVALID_ARGUMENT, "segment pages are not device memory");
    dev = (dev == -2 || dev == a.device) ? a.device : -1;
  }
  lay->pages_device = dev == -2 ? -1 : dev;
  return KVX_OK;
}
}  // namespace

extern "C" {

const char* kvx_status_string(int status) {
  switch (status) {
    case KVX_OK: return "ok";
    case KVX_ERR_INVALID_ARGUMENT: return "invalid argument";
    case KVX_ERR_LENGTH_MISMATCH: return "metadata length mismatch";
    case KVX_ERR_GROUP: return "invalid cache-group id";
    case KVX_ERR_EXTENT: return "invalid kernel-block extent";
    case KVX_ERR_BLOCK_ID: return "block id out of range";
    case KVX_ERR_HOST_MEMORY: return "host memory not usable";
    case KVX_ERR_CUDA: return "CUDA error";
    case KVX_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case KVX_ERR_LAYOUT: return "layouts differ";
    case KVX_ERR_NO_MEMORY: return "out of memory";
    case KVX_ERR_IO: return "file cannot be read";
    case KVX_ERR_FORMAT: return "invalid file format";
    default: return "unknown status";
  }
}

const char* kvx_last_error(void) { return t_last_error.c_str(); }
int kvx_version(void) { return 10000; }
int kvx_last_mode(void) { return t_last_mode; }
uint64_t kvx_kernel_launches(void) { return g_kernel_launches.load(); }

int kvx_kernel_timing(int enable) {
  g_timing.store(enable != 0);
  return KVX_OK;
}

int kvx_kernel_timing_read(uint64_t* launches, double* total_ms, double* busy_ms,
                           uint64_t* hbm_bytes) {
  t_last_error.clear();
  std::vector<TimedLaunch> v;
  {
    std::lock_guard<std::mutex> g(g_timing_mu);
    v.swap(g_timed);
  }
  uint64_t n = 0, bytes = 0;
  double ms = 0;
  int rc = KVX_OK;
  // Intervals relative to the first launch of each device, to merge the
  // launches that overlapped (several streams) into busy time.
  std::map<int, std::vector<std::pair<double, double>>> spans;
  std::map<int, cudaEvent_t> ref;
  for (TimedLaunch& t : v) {
    float e = 0, b0 = 0, e0 = 0;
    cudaError_t err = cudaEventSynchronize(t.end);
    if (err == cudaSuccess) err = cudaEventElapsedTime(&e, t.begin, t.end);
    if (!ref.count(t.device)) ref[t.device] = t.begin;
    if (err == cudaSuccess) err = cudaEventElapsedTime(&b0, ref[t.device], t.begin);
    if (err == cudaSuccess) err = cudaEventElapsedTime(&e0, ref[t.device], t.end);
    if (err != cudaSuccess && rc == KVX_OK) rc = cuda_error(err, "cudaEventElapsedTime");
    ++n;
    ms += e;
    bytes += t.hbm_bytes;
    spans[t.device].emplace_back(b0, e0);
  }
  double busy = 0;
  for (auto& kv : spans) {
    auto& iv = kv.second;
    std::sort(iv.begin(), iv.end());
    double cb = 0, ce = 0;
    bool open = false;
    for (const auto& x : iv) {
      if (!open || x.first > ce) {
        if (open) busy += ce - cb;
        cb = x.first;
        ce = x.second;
        open = true;
      } else if (x.second > ce) {
        ce = x.second;
      }
    }
    if (open) busy += ce - cb;
  }
  for (TimedLaunch& t : v) {
    cudaEventDestroy(t.begin);
    cudaEventDestroy(t.end);
  }
  if (launches) *launches = n;
  if (total_ms) *total_ms = ms;
  if (busy_ms) *busy_ms = busy;
  if (hbm_bytes) *hbm_bytes = bytes;
  return rc;
}

int kvx_configure(int64_t sm_ctas_host, int64_t sm_ctas_dev, int64_t ce_min_run,
                  int64_t staging_bytes, int64_t ce_pipeline) {
  tunables();
  std::lock_guard<std::mutex> g(g_tun_mu);
  if (sm_ctas_host > 0) g_tun.sm_ctas_host = sm_ctas_host;
  if (sm_ctas_dev > 0) g_tun.sm_ctas_dev = sm_ctas_dev;
  if (ce_min_run != 0) g_tun.ce_min_run = ce_min_run < 0 ? 0 : ce_min_run;
  if (staging_bytes > 0) g_tun.staging_bytes = staging_bytes;
  if (ce_pipeline >= 0) g_tun.ce_pipeline = ce_pipeline;
  return KVX_OK;
}

int kvx_set_option(const char* name, int64_t value) {
  t_last_error.clear();
  if (!name) return set_error(KVX_ERR_INVALID_ARGUMENT, "null option name");
  tunables();
  std::lock_guard<std::mutex> g(g_tun_mu);
  const std::string n(name);
  if (n == "ce_streams") {
    if (value < 1 || value > kMaxCeStreams)
      return set_error(KVX_ERR_INVALID_ARGUMENT, "ce_streams must be in [1, 8]");
    g_tun.ce_streams = value;
  } else if (n == "host_bulk") {
    g_tun.host_bulk = value ? 1 : 0;
  } else if (n == "staging_bulk") {
    g_tun.staging_bulk = value ? 1 : 0;
  } else if (n == "bulk_ctas_per_sm") {
    if (value != 1 && value != 2)
      return set_error(KVX_ERR_INVALID_ARGUMENT, "bulk_ctas_per_sm must be 1 or 2");
    g_tun.bulk_ctas_per_sm = value;
  } else if (n == "bulk_waves") {
    if (value < 1 || value > 64)
      return set_error(KVX_ERR_INVALID_ARGUMENT, "bulk_waves must be in [1, 64]");
    g_tun.bulk_waves = value;
  } else if (n == "vec_bytes") {
    if (value != 16 && value != 32)
      return set_error(KVX_ERR_INVALID_ARGUMENT, "vec_bytes must be 16 or 32");
    g_tun.vec_bytes = value;
  } else if (n == "ce_max_copy") {
    if (value < 0) return set_error(KVX_ERR_INVALID_ARGUMENT, "ce_max_copy must be >= 0");
    g_tun.ce_max_copy = value;
  } else if (n == "ce_streams_max_run") {
    g_tun.ce_streams_max_run = value;
  } else if (n == "ce_min_run") {
    g_tun.ce_min_run = value < 0 ? 0 : value;
  } else if (n == "ce_min_bytes") {
    g_tun.ce_min_bytes = value;
  } else if (n == "sm_ctas_host") {
    g_tun.sm_ctas_host = value;
  } else if (n == "sm_ctas_host_out") {
    g_tun.sm_ctas_host_out = value;
  } else if (n == "sm_ctas_host_in") {
    g_tun.sm_ctas_host_in = value;
  } else if (n == "sm_ctas_dev") {
    g_tun.sm_ctas_dev = value;
  } else if (n == "direct_max") {
    g_tun.direct_max = value;
  } else {
    return set_error(KVX_ERR_INVALID_ARGUMENT, "unknown option " + n);
  }
  return KVX_OK;
}

int kvx_byte_extent(uint64_t page_bytes, int64_t kernel_blocks_per_page,
                    int64_t first_kernel_block, int64_t num_kernel_blocks,
                    uint64_t* byte_offset_out, uint64_t* byte_length_out) {
  t_last_error.clear();
  if (!byte_offset_out || !byte_length_out)
    return set_error(KVX_ERR_INVALID_ARGUMENT, "null output pointer");
  return from_plan(byte_extent(page_bytes, kernel_blocks_per_page, first_kernel_block,
                               num_kernel_blocks, byte_offset_out, byte_length_out));
}

int kvx_plan_swap(const int64_t* source_block_ids, const int64_t* target_block_ids,
                  int64_t num_ids, int is_swap_in, uint64_t kv_cache,
                  uint64_t kv_cache_bytes, uint64_t block_bytes, uint64_t kv_swap,
                  uint64_t kv_swap_bytes, uint64_t* src_addrs, uint64_t* dst_addrs,
                  uint64_t* lengths, int64_t* num_copies_inout) {
  t_last_error.clear();
  if (!num_copies_inout) return set_error(KVX_ERR_INVALID_ARGUMENT, "null count");
  std::vector<Copy> copies;
  GridPlan gp;
  if (grid_swap(source_block_ids, target_block_ids, num_ids, is_swap_in != 0, kv_cache,
                kv_cache_bytes, block_bytes, kv_swap, kv_swap_bytes, &gp)) {
    grid_finalize(&gp, kVecShift);
    grid_expand(gp, kVecShift, &copies);
  } else {
    int rc = from_plan(plan_swap(source_block_ids, target_block_ids, num_ids, is_swap_in != 0,
                                 kv_cache, kv_cache_bytes, block_bytes, kv_swap,
                                 kv_swap_bytes, &copies));
    if (rc) return rc;
  }
  const int64_t cap = *num_copies_inout;
  *num_copies_inout = int64_t(copies.size());
  if (cap < int64_t(copies.size()) || !src_addrs || !dst_addrs || !lengths) return KVX_OK;
  for (size_t i = 0; i < copies.size(); ++i) {
    src_addrs[i] = copies[i].src;
    dst_addrs[i] = copies[i].dst;
    lengths[i] = copies[i].len;
  }
  return KVX_OK;
}

int kvx_swap(const int64_t* source_block_ids, const int64_t* target_block_ids,
             int64_t num_ids, int is_swap_in, void* kv_cache, uint64_t kv_cache_bytes,
             uint64_t block_bytes, void* kv_swap, uint64_t kv_swap_bytes, int mode,
             void* stream) {
  t_last_error.clear();
  std::vector<Copy> copies;
  int rc = from_plan(plan_swap(source_block_ids, target_block_ids, num_ids, is_swap_in != 0,
                               reinterpret_cast<uint64_t>(kv_cache), kv_cache_bytes,
                               block_bytes, reinterpret_cast<uint64_t>(kv_swap),
                               kv_swap_bytes, &copies));
  if (rc) return rc;
  if (copies.empty()) {
    t_last_mode = mode == KVX_MODE_AUTO ? KVX_MODE_SM : mode;
    return KVX_OK;
  }
  int device = 0;
  KVX_CUDA(cudaGetDevice(&device));
  rc = check_device_memory(kv_cache, device, "kv_cache");
  if (rc) return rc;
  DeviceState* st = nullptr;
  rc = get_state(device, &st);
  if (rc) return rc;
  const HostInfo hi = host_info(kv_swap, device);
  GridPlan gp;
  const bool grid = grid_swap(source_block_ids, target_block_ids, num_ids, is_swap_in != 0,
                              reinterpret_cast<uint64_t>(kv_cache), kv_cache_bytes, block_bytes,
                              reinterpret_cast<uint64_t>(kv_swap), kv_swap_bytes, &gp);
  std::lock_guard<std::mutex> g(st->mu);
  if (grid)
    return execute_grid_host(st, &gp, hi, reinterpret_cast<uint64_t>(kv_swap), mode,
                             reinterpret_cast<cudaStream_t>(stream));
  return execute_host_copies(st, copies, is_swap_in != 0, hi,
                             reinterpret_cast<uint64_t>(kv_swap), mode,
                             reinterpret_cast<cudaStream_t>(stream));
}

int kvx_layout_create(int device, int64_t num_segments, void* const* segment_pages,
                      const uint64_t* segment_page_bytes, const uint64_t* segment_num_blocks,
                      const uint64_t* segment_cpu_offsets,
                      const uint64_t* segment_owner_masks, int64_t num_groups,
                      const int64_t* group_blocks_per_kv_block, void* host_pool,
                      uint64_t host_pool_bytes, uint64_t host_row_bytes,
                      uint64_t host_row_offset, kvx_layout** layout_out) {
  t_last_error.clear();
  if (!layout_out) return set_error(KVX_ERR_INVALID_ARGUMENT, "null layout_out");
  *layout_out = nullptr;
  if (num_segments < 0 || num_groups < 0)
    return set_error(KVX_ERR_INVALID_ARGUMENT, "negative table size");
  if (num_segments > 0 && (!segment_pages || !segment_page_bytes || !segment_num_blocks ||
                           !segment_cpu_offsets || !segment_owner_masks))
    return set_error(KVX_ERR_INVALID_ARGUMENT, "null segment table");
  if (num_groups > 0 && !group_blocks_per_kv_block)
    return set_error(KVX_ERR_INVALID_ARGUMENT, "null group table");
  auto lay = std::make_unique<kvx_layout>();
  Layout& L = lay->L;
  L.device = device;
  for (int64_t s = 0; s < num_segments; ++s) {
    L.seg_pages.push_back(reinterpret_cast<uint64_t>(segment_pages[s]));
    L.seg_page_bytes.push_back(segment_page_bytes[s]);
    L.seg_num_blocks.push_back(segment_num_blocks[s]);
    L.seg_cpu_offset.push_back(segment_cpu_offsets[s]);
    L.seg_owner_mask.push_back(segment_owner_masks[s]);
  }
  L.group_ratio.assign(group_blocks_per_kv_block, group_blocks_per_kv_block + num_groups);
  L.host_pool = reinterpret_cast<uint64_t>(host_pool);
  L.host_pool_bytes = host_pool ? host_pool_bytes : 0;
  L.host_row_bytes = host_pool ? host_row_bytes : 0;
  L.host_row_offset = host_pool ? host_row_offset : 0;
  L.host_num_rows = (host_pool && host_row_bytes) ? host_pool_bytes / host_row_bytes : 0;
  int rc = from_plan(validate_layout(L));
  if (rc) return rc;
  if (host_pool) {
    // Best effort: a CPU-only process (no driver) still gets a layout usable
    // for planning; the copy entry points re-check the mapping.
    lay->host = host_info(host_pool, device);
    L.host_pool_dev = lay->host.mapped ? lay->host.dev_base : 0;
  }
  *layout_out = lay.release();
  return KVX_OK;
}

int kvx_layout_destroy(kvx_layout* layout) {
  delete layout;
  return KVX_OK;
}

int kvx_plan_swap_blocks(const kvx_layout* layout, int64_t num_entries,
                         const int64_t* source_block_ids, const int64_t* target_block_ids,
                         const int64_t* group_ids, const int64_t* first_kernel_blocks,
                         const int64_t* valid_kernel_blocks, int is_swap_in,
                         uint64_t* src_addrs, uint64_t* dst_addrs, uint64_t* lengths,
                         int64_t* num_copies_inout) {
  t_last_error.clear();
  if (!layout || !num_copies_inout)
    return set_error(KVX_ERR_INVALID_ARGUMENT, "null layout or count");
  Entries e{num_entries, source_block_ids, target_block_ids, group_ids,
            first_kernel_blocks, valid_kernel_blocks};
  std::vector<Copy> copies;
  GridPlan gp;
  if (grid_swap_blocks(layout->L, e, is_swap_in != 0, layout->L.host_pool, &gp)) {
    grid_finalize(&gp, kVecShift);
    grid_expand(gp, kVecShift, &copies);
  } else {
    int rc = from_plan(plan_swap_blocks(layout->L, e, is_swap_in != 0, layout->L.host_pool,
                                        &copies, nullptr));
    if (rc) return rc;
  }
  const int64_t cap = *num_copies_inout;
  *num_copies_inout = int64_t(copies.size());
  if (cap < int64_t(copies.size()) || !src_addrs || !dst_addrs || !lengths) return KVX_OK;
  for (size_t i = 0; i < copies.size(); ++i) {
    src_addrs[i] = copies[i].src;
    dst_addrs[i] = copies[i].dst;
    lengths[i] = copies[i].len;
  }
  return KVX_OK;
}

int kvx_swap_blocks(kvx_layout* layout, int64_t num_entries,
                    const int64_t* source_block_ids, const int64_t* target_block_ids,
                    const int64_t* group_ids, const int64_t* first_kernel_blocks,
                    const int64_t* valid_kernel_blocks, int is_swap_in, int mode,
                    void* stream, uint64_t* copied_bytes, uint64_t* copy_extents) {
  t_last_error.clear();
  if (!layout) return set_error(KVX_ERR_INVALID_ARGUMENT, "null layout");
  Entries e{num_entries, source_block_ids, target_block_ids, group_ids,
            first_kernel_blocks, valid_kernel_blocks};
  // Grid form first (O(entries) host work); the item planner otherwise, which
  // is also the one that reports invalid requests.
  GridPlan gp;
  const bool grid = grid_swap_blocks(layout->L, e, is_swap_in != 0, layout->L.host_pool, &gp);
  std::vector<Copy> copies;
  uint64_t copied = 0, extents = 0;
  int rc = KVX_OK;
  if (grid) {
    copied = gp.copied;
    extents = gp.extents;
  } else {
    rc = from_plan(plan_swap_blocks(layout->L, e, is_swap_in != 0, layout->L.host_pool,
                                    &copies, &copied));
    if (rc) return rc;
    extents = copies.size();
  }
  if (copied_bytes) *copied_bytes = copied;
  if (copy_extents) *copy_extents = extents;
  if (extents == 0) {
    t_last_mode = mode == KVX_MODE_AUTO ? KVX_MODE_SM : mode;
    return KVX_OK;
  }
  DeviceGuard dg(layout->L.device);
  if (!dg.ok()) return set_error(KVX_ERR_CUDA, "cannot select the layout's device");
  DeviceState* st = nullptr;
  rc = get_state(layout->L.device, &st);
  if (rc) return rc;
  if (!layout->host.mapped) {  // re-query: the pool may have been registered since
    layout->host = host_info(reinterpret_cast<void*>(layout->L.host_pool), layout->L.device);
    layout->L.host_pool_dev = layout->host.mapped ? layout->host.dev_base : 0;
  }
  std::lock_guard<std::mutex> g(st->mu);
  if (grid)
    return execute_grid_host(st, &gp, layout->host, layout->L.host_pool, mode,
                             reinterpret_cast<cudaStream_t>(stream));
  return execute_host_copies(st, copies, is_swap_in != 0, layout->host, layout->L.host_pool,
                             mode, reinterpret_cast<cudaStream_t>(stream));
}

int kvx_migrate_blocks(kvx_layout* source, kvx_layout* target, int64_t num_entries,
                       const int64_t* source_block_ids, const int64_t* target_block_ids,
                       const int64_t* group_ids, const int64_t* first_kernel_blocks,
                       const int64_t* valid_kernel_blocks, int mode, void* stream,
                       uint64_t* copied_bytes, uint64_t* copy_extents) {
  t_last_error.clear();
  if (!source || !target) return set_error(KVX_ERR_INVALID_ARGUMENT, "null layout");
  Entries e{num_entries, source_block_ids, target_block_ids, group_ids,
            first_kernel_blocks, valid_kernel_blocks};
  GridPlan gp;
  const bool grid = grid_migrate(source->L, target->L, e, &gp);
  std::vector<Copy> copies;
  uint64_t copied = 0, extents = 0;
  int rc = KVX_OK;
  if (grid) {
    copied = gp.copied;
    extents = gp.extents;
  } else {
    rc = from_plan(plan_migrate(source->L, target->L, e, &copies, &copied));
    if (rc) return rc;
    extents = copies.size();
  }
  if (copied_bytes) *copied_bytes = copied;
  if (copy_extents) *copy_extents = extents;
  if (extents == 0) {
    t_last_mode = mode == KVX_MODE_AUTO ? KVX_MODE_SM : mode;
    return KVX_OK;
  }
  int device = 0;
  KVX_CUDA(cudaGetDevice(&device));
  DeviceState* st = nullptr;
  rc = get_state(device, &st);
  if (rc) return rc;
  // Local when every page table base of both layouts is memory of this GPU;
  // otherwise some side is a peer mapping and only the vector kernel is used.
  bool local = true;
  for (kvx_layout* lay : {source, target}) {
    rc = pages_device(lay);
    if (rc) return rc;
    if (lay->pages_device != device) local = false;
  }
  const Tunables tn = tunables();
  std::lock_guard<std::mutex> g(st->mu);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (mode == KVX_MODE_AUTO) mode = KVX_MODE_SM;
  const Path path = local ? Path::kDevice : Path::kPeer;
  if (mode == KVX_MODE_CE || mode == KVX_MODE_CE_EXTENT) {
    if (grid) copies = grid_extents(gp);
    rc = run_ce_extent(copies, grid ? std::vector<size_t>{copies.size()} : split_waves(copies), s,
                       /*merge=*/false);
    mode = KVX_MODE_CE_EXTENT;
  } else if (mode == KVX_MODE_SM || mode == KVX_MODE_SM_BULK) {
    // TMA bulk copies also cross NVLink: plain (non-multicast) bulk loads
    // from a peer's pages (pull) or bulk stores into them (push).
    const bool bulk = mode == KVX_MODE_SM_BULK;
    if (grid)
      rc = run_sm_grid(st, &gp, path, bulk, s, tn);
    else
      rc = run_sm(st, copies, split_waves(copies), path, bulk, s, tn);
    mode = bulk ? KVX_MODE_SM_BULK : KVX_MODE_SM;
  } else {
    return set_error(KVX_ERR_INVALID_ARGUMENT, "unknown transfer mode");
  }
  if (rc == KVX_OK) t_last_mode = mode;
  return rc;
}

// ---- IPC -----------------------------------------------------------------------
namespace {
std::mutex g_ipc_mu;
std::map<uint64_t, uint64_t> g_ipc_bases;  // returned pointer -> mapped base

using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
GetRangeFn get_range_fn() {
  static GetRangeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<GetRangeFn>(nullptr);
    return reinterpret_cast<GetRangeFn>(p);
  }();
  return fn;
}
}  // namespace

int kvx_ipc_export(void* dev_ptr, uint8_t* handle_out64, uint64_t* offset_out) {
  t_last_error.clear();
  if (!dev_ptr || !handle_out64 || !offset_out)
    return set_error(KVX_ERR_INVALID_ARGUMENT, "null argument");
  GetRangeFn fn = get_range_fn();
  if (!fn) return set_error(KVX_ERR_CUDA, "cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return set_error(KVX_ERR_INVALID_ARGUMENT, "pointer is not in a device allocation");
  cudaIpcMemHandle_t h;
  KVX_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  std::memcpy(handle_out64, &h, 64);
  *offset_out = reinterpret_cast<uint64_t>(dev_ptr) - uint64_t(base);
  return KVX_OK;
}

int kvx_ipc_import(int device, const uint8_t* handle64, uint64_t offset, void** dev_ptr_out) {
  t_last_error.clear();
  if (!handle64 || !dev_ptr_out) return set_error(KVX_ERR_INVALID_ARGUMENT, "null argument");
  DeviceGuard dg(device);
  if (!dg.ok()) return set_error(KVX_ERR_CUDA, "cannot select device");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, 64);
  void* base = nullptr;
  KVX_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  const uint64_t p = reinterpret_cast<uint64_t>(base) + offset;
  {
    std::lock_guard<std::mutex> g(g_ipc_mu);
    g_ipc_bases[p] = reinterpret_cast<uint64_t>(base);
  }
  *dev_ptr_out = reinterpret_cast<void*>(p);
  return KVX_OK;
}

int kvx_ipc_close(int device, void* dev_ptr) {
  t_last_error.clear();
  uint64_t base = 0;
  {
    std::lock_guard<std::mutex> g(g_ipc_mu);
    auto it = g_ipc_bases.find(reinterpret_cast<uint64_t>(dev_ptr));
    if (it == g_ipc_bases.end())
      return set_error(KVX_ERR_INVALID_ARGUMENT, "pointer was not returned by kvx_ipc_import");
    base = it->second;
    g_ipc_bases.erase(it);
  }
  DeviceGuard dg(device);
  KVX_CUDA(cudaIpcCloseMemHandle(reinterpret_cast<void*>(base)));
  return KVX_OK;
}

int kvx_upload_weights(void* const* dst_device, const void* const* src_host,
                       const uint64_t* bytes, int64_t num_buffers, uint64_t chunk_bytes,
                       int host_threads, void* stream) {
  t_last_error.clear();
  if (num_buffers < 0) return set_error(KVX_ERR_INVALID_ARGUMENT, "negative buffer count");
  if (num_buffers == 0) return KVX_OK;
  if (!dst_device || !src_host || !bytes)
    return set_error(KVX_ERR_INVALID_ARGUMENT, "null array argument");
  if (chunk_bytes == 0) return set_error(KVX_ERR_INVALID_ARGUMENT, "chunk_bytes must be > 0");
  int device = 0;
  KVX_CUDA(cudaGetDevice(&device));
  std::vector<bool> pinned(static_cast<size_t>(num_buffers), false);
  bool any_pageable = false;
  for (int64_t i = 0; i < num_buffers; ++i) {
    if (bytes[i] == 0) continue;
    if (!dst_device[i] || !src_host[i])
      return set_error(KVX_ERR_INVALID_ARGUMENT, "null buffer " + std::to_string(i));
    int rc = check_device_memory(dst_device[i], device, "destination buffer");
    if (rc) return rc;
    pinned[size_t(i)] = host_is_pinned(src_host[i]);
    any_pageable |= !pinned[size_t(i)];
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  DeviceState* st = nullptr;
  if (any_pageable) {
    int rc = get_state(device, &st);
    if (rc) return rc;
  }
  // Pageable pieces go through page-locked bounce buffers of at most 64 MiB
  // each (the reference's cut size), whatever chunk_bytes asks for.
  const uint64_t bounce_piece = std::min<uint64_t>(chunk_bytes, uint64_t(64) << 20);
  std::unique_lock<std::mutex> lock;
  if (st) {
    lock = std::unique_lock<std::mutex>(st->upload_mu);
    int rc = bounce_ready(st, size_t(bounce_piece));
    if (rc) return rc;
  }
  int next = 0;  // bounce buffer of the next pageable chunk
  for (int64_t i = 0; i < num_buffers; ++i) {
    char* dst = static_cast<char*>(dst_device[i]);
    const char* src = static_cast<const char*>(src_host[i]);
    const uint64_t step = pinned[size_t(i)] ? chunk_bytes : bounce_piece;
    for (uint64_t o = 0; o < bytes[i]; o += step) {
      const uint64_t n = std::min(step, bytes[i] - o);
      if (pinned[size_t(i)]) {
        KVX_CUDA(cudaMemcpyAsync(dst + o, src + o, n, cudaMemcpyHostToDevice, s));
        continue;
      }
      // The host fills one bounce buffer while the copy engine drains the
      // other; a buffer is refilled once the copy that read it has finished.
      const int b = next;
      next ^= 1;
      if (st->bounce_used[b]) KVX_CUDA(cudaEventSynchronize(st->bounce_ev[b]));
      parallel_memcpy(st->bounce[b], src + o, size_t(n), host_threads);
      KVX_CUDA(cudaMemcpyAsync(dst + o, st->bounce[b], n, cudaMemcpyHostToDevice, s));
      KVX_CUDA(cudaEventRecord(st->bounce_ev[b], s));
      st->bounce_used[b] = true;
    }
  }
  return KVX_OK;
}

int kvx_upload_chunked(void* dst_device, const void* src_host, uint64_t bytes,
                       uint64_t chunk_bytes, void* stream) {
  t_last_error.clear();
  if (bytes && (!dst_device || !src_host))
    return set_error(KVX_ERR_INVALID_ARGUMENT, "null pointer");
  if (bytes == 0) return KVX_OK;
  if (chunk_bytes == 0) chunk_bytes = bytes;
  const int threads = int(std::max(1u, std::thread::hardware_concurrency()));
  return kvx_upload_weights(&dst_device, &src_host, &bytes, 1, chunk_bytes, threads, stream);
}

int kvx_selftest_bounded_wait(uint64_t limit_ns, void* stream) {
  t_last_error.clear();
  if (limit_ns == 0 || limit_ns > 10ull * 1000 * 1000 * 1000)
    return set_error(KVX_ERR_INVALID_ARGUMENT, "limit_ns must be in (0, 10 s]");
  kvx_wait_selftest<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(limit_ns);
  KVX_CUDA(cudaGetLastError());
  return KVX_OK;
}

int kvx_device_status(int device, int reset, int* status_out) {
  t_last_error.clear();
  if (!status_out) return set_error(KVX_ERR_INVALID_ARGUMENT, "null status_out");
  DeviceGuard dg(device);
  if (!dg.ok()) return set_error(KVX_ERR_CUDA, "cannot select device");
  KVX_CUDA(cudaDeviceSynchronize());
  int v = 0;
  KVX_CUDA(cudaMemcpyFromSymbol(&v, g_kvx_device_status, sizeof(int)));
  if (reset) {
    const int zero = 0;
    KVX_CUDA(cudaMemcpyToSymbol(g_kvx_device_status, &zero, sizeof(int)));
  }
  *status_out = v;
  return KVX_OK;
}

}  // extern "C"
