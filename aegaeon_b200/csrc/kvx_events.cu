// Event pool and interprocess event cache for ordering KV moves across
// workers.
//
// The reference orders a move after earlier moves of the same request with
// CUDA IPC event handles shipped through Ray (aegaeon/worker.py:2248-2257,
// 2331, 2349, 2351-2394; aegaeon/utils.py:263-288): every swap_blocks call
// creates a new interprocess event and every waiter opens the handle again
// (cudaIpcOpenEventHandle), waits, and destroys it, per request and call.
// Here:
//   * events come from a per-device pool (created once, reused after their
//     last record completed and the holder released them);
//   * an opened IPC handle is cached by its 64 bytes, so repeated waits on
//     the same producer event do not reopen it;
//   * a stream waits on a whole list of events in one call.
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/kvx.h"

namespace kvx {
void record_error(const std::string& msg);  // kvx_runtime.cu
}

struct kvx_event {
  cudaEvent_t ev = nullptr;
  int device = 0;
  bool interprocess = false;
  bool imported = false;  // opened from another process's handle
  std::string key;        // handle bytes, for imported events
  int refs = 1;
};

namespace {

std::mutex g_mu;
std::vector<kvx_event*> g_free[64][2];          // [device][interprocess]
std::map<std::string, kvx_event*> g_imported;   // handle bytes -> event

int cuda_fail(cudaError_t e, const char* what) {
  kvx::record_error(std::string(what) + ": " + cudaGetErrorString(e));
  return KVX_ERR_CUDA;
}

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= 64) {
    kvx::record_error("device index out of range");
    return KVX_ERR_INVALID_ARGUMENT;
  }
  return KVX_OK;
}

}  // namespace

extern "C" {

int kvx_event_create(int interprocess, kvx_event** out) {
  kvx::record_error("");
  if (!out) return KVX_ERR_INVALID_ARGUMENT;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc) return rc;
  const int ip = interprocess ? 1 : 0;
  {
    std::lock_guard<std::mutex> g(g_mu);
    if (!g_free[dev][ip].empty()) {
      *out = g_free[dev][ip].back();
      g_free[dev][ip].pop_back();
      (*out)->refs = 1;
      return KVX_OK;
    }
  }
  auto* e = new kvx_event();
  e->device = dev;
  e->interprocess = ip != 0;
  const unsigned flags = cudaEventDisableTiming | (ip ? cudaEventInterprocess : 0);
  cudaError_t err = cudaEventCreateWithFlags(&e->ev, flags);
  if (err != cudaSuccess) {
    delete e;
    return cuda_fail(err, "cudaEventCreateWithFlags");
  }
  *out = e;
  return KVX_OK;
}

int kvx_event_record(kvx_event* ev, void* stream) {
  if (!ev || ev->imported) {
    kvx::record_error("cannot record an imported event");
    return KVX_ERR_INVALID_ARGUMENT;
  }
  cudaError_t e = cudaEventRecord(ev->ev, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KVX_OK : cuda_fail(e, "cudaEventRecord");
}

int kvx_event_query(kvx_event* ev, int* done) {
  if (!ev || !done) return KVX_ERR_INVALID_ARGUMENT;
  cudaError_t e = cudaEventQuery(ev->ev);
  if (e == cudaSuccess) {
    *done = 1;
    return KVX_OK;
  }
  if (e == cudaErrorNotReady) {
    cudaGetLastError();
    *done = 0;
    return KVX_OK;
  }
  return cuda_fail(e, "cudaEventQuery");
}

int kvx_event_synchronize(kvx_event* ev) {
  if (!ev) return KVX_ERR_INVALID_ARGUMENT;
  cudaError_t e = cudaEventSynchronize(ev->ev);
  return e == cudaSuccess ? KVX_OK : cuda_fail(e, "cudaEventSynchronize");
}

int kvx_event_ipc_handle(kvx_event* ev, uint8_t* handle_out64) {
  if (!ev || !handle_out64 || !ev->interprocess || ev->imported) {
    kvx::record_error("only interprocess events created here have a handle");
    return KVX_ERR_INVALID_ARGUMENT;
  }
  cudaIpcEventHandle_t h;
  static_assert(sizeof(h) == 64, "IPC event handle size");
  cudaError_t e = cudaIpcGetEventHandle(&h, ev->ev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetEventHandle");
  std::memcpy(handle_out64, &h, 64);
  return KVX_OK;
}

int kvx_event_open_ipc(const uint8_t* handle64, kvx_event** out) {
  kvx::record_error("");
  if (!handle64 || !out) return KVX_ERR_INVALID_ARGUMENT;
  std::string key(reinterpret_cast<const char*>(handle64), 64);
  std::lock_guard<std::mutex> g(g_mu);
  auto it = g_imported.find(key);
  if (it != g_imported.end()) {
    ++it->second->refs;
    *out = it->second;
    return KVX_OK;
  }
  cudaIpcEventHandle_t h;
  std::memcpy(&h, handle64, 64);
  auto* e = new kvx_event();
  cudaError_t err = cudaIpcOpenEventHandle(&e->ev, h);
  if (err != cudaSuccess) {
    delete e;
    return cuda_fail(err, "cudaIpcOpenEventHandle");
  }
  cudaGetDevice(&e->device);
  e->interprocess = true;
  e->imported = true;
  e->key = key;
  g_imported[key] = e;
  *out = e;
  return KVX_OK;
}

int kvx_stream_wait_events(void* stream, kvx_event* const* events, int64_t n) {
  if (n < 0 || (n > 0 && !events)) return KVX_ERR_INVALID_ARGUMENT;
  for (int64_t i = 0; i < n; ++i) {
    if (!events[i]) continue;
    cudaError_t e = cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), events[i]->ev, 0);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent");
  }
  return KVX_OK;
}

int kvx_event_release(kvx_event* ev) {
  if (!ev) return KVX_OK;
  std::lock_guard<std::mutex> g(g_mu);
  if (--ev->refs > 0) return KVX_OK;
  if (ev->imported) {
    // Imported handles stay cached: the producer may be waited on again.
    ev->refs = 0;
    return KVX_OK;
  }
  if (ev->device >= 0 && ev->device < 64) {
    g_free[ev->device][ev->interprocess ? 1 : 0].push_back(ev);
    return KVX_OK;
  }
  cudaEventDestroy(ev->ev);
  delete ev;
  return KVX_OK;
}

int kvx_event_forget_ipc(const uint8_t* handle64) {
  if (!handle64) return KVX_ERR_INVALID_ARGUMENT;
  std::string key(reinterpret_cast<const char*>(handle64), 64);
  std::lock_guard<std::mutex> g(g_mu);
  auto it = g_imported.find(key);
  if (it == g_imported.end()) return KVX_OK;
  kvx_event* e = it->second;
  g_imported.erase(it);
  cudaEventDestroy(e->ev);
  delete e;
  return KVX_OK;
}

}  // extern "C"
