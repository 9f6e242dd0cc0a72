/* Python call shim for the per-request entry points of libkvx.so (kvx_swap,
 * kvx_swap_blocks, kvx_migrate_blocks).
 *
 * A swap issued for one decode turn moves a handful of blocks, and then the
 * cost of getting from Python to the C ABI is most of the call: ctypes
 * marshals every argument and the id lists are converted one by one.  This
 * module does both in C (METH_FASTCALL, ids read straight from a list, tuple
 * or int64 buffer) and calls libkvx.so through function pointers that the
 * Python side takes from the ctypes-loaded library (bind()), so both routes
 * reach the same library instance and its thread-local error message.
 *
 * Every function returns the kvx status code; the caller maps it to an
 * exception (aegaeon_b200._lib.check).  Conversion errors raise here:
 * TypeError for a non-integer id, OverflowError for one outside int64 and
 * ValueError when the id lists differ in length.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>
#include <string.h>

#include "../../include/kvx.h"

typedef int (*swap_fn)(const int64_t*, const int64_t*, int64_t, int, void*, uint64_t, uint64_t,
                       void*, uint64_t, int, void*);
typedef int (*swap_blocks_fn)(kvx_layout*, int64_t, const int64_t*, const int64_t*,
                              const int64_t*, const int64_t*, const int64_t*, int, int, void*,
                              uint64_t*, uint64_t*);
typedef int (*migrate_blocks_fn)(kvx_layout*, kvx_layout*, int64_t, const int64_t*,
                                 const int64_t*, const int64_t*, const int64_t*, const int64_t*,
                                 int, void*, uint64_t*, uint64_t*);

static swap_fn g_swap = NULL;
static swap_blocks_fn g_swap_blocks = NULL;
static migrate_blocks_fn g_migrate_blocks = NULL;

/* Ids of one argument as an int64 array: borrowed from an int64 buffer, or
 * converted into `local` (when it fits) or a heap array. */
typedef struct {
  const int64_t* data;
  Py_ssize_t n;
  int64_t* heap;
  Py_buffer view;
  int has_view;
} Ids;

#define KVX_LOCAL_IDS 64

static void ids_release(Ids* ids) {
  if (ids->heap) PyMem_Free(ids->heap);
  if (ids->has_view) PyBuffer_Release(&ids->view);
  ids->heap = NULL;
  ids->has_view = 0;
}

static int ids_from(PyObject* obj, int64_t* local, Ids* out) {
  memset(out, 0, sizeof(*out));
  if (!PyList_Check(obj) && !PyTuple_Check(obj) && PyObject_CheckBuffer(obj)) {
    if (PyObject_GetBuffer(obj, &out->view, PyBUF_C_CONTIGUOUS | PyBUF_FORMAT) == 0) {
      const char* f = out->view.format ? out->view.format : "B";
      if (*f == '<' || *f == '=' || *f == '@') ++f;
      if (out->view.itemsize == 8 && (strcmp(f, "q") == 0 || strcmp(f, "l") == 0)) {
        out->has_view = 1;
        out->data = (const int64_t*)out->view.buf;
        out->n = out->view.len / 8;
        return 0;
      }
      PyBuffer_Release(&out->view);
    } else {
      PyErr_Clear();
    }
  }
  PyObject* seq = PySequence_Fast(obj, "block ids must be a sequence of integers");
  if (!seq) return -1;
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(seq);
  int64_t* dst = local;
  if (n > KVX_LOCAL_IDS) {
    dst = (int64_t*)PyMem_Malloc((size_t)n * sizeof(int64_t));
    if (!dst) {
      Py_DECREF(seq);
      PyErr_NoMemory();
      return -1;
    }
    out->heap = dst;
  }
  PyObject** items = PySequence_Fast_ITEMS(seq);
  for (Py_ssize_t i = 0; i < n; ++i) {
    PyObject* it = items[i];
    long long v;
    if (PyLong_CheckExact(it)) {
      v = PyLong_AsLongLong(it);
    } else {
      PyObject* idx = PyNumber_Index(it); /* TypeError for floats, strings, None */
      if (!idx) {
        Py_DECREF(seq);
        ids_release(out);
        return -1;
      }
      v = PyLong_AsLongLong(idx);
      Py_DECREF(idx);
    }
    if (v == -1 && PyErr_Occurred()) { /* OverflowError outside int64 */
      Py_DECREF(seq);
      ids_release(out);
      return -1;
    }
    dst[i] = (int64_t)v;
  }
  Py_DECREF(seq);
  out->data = dst;
  out->n = n;
  return 0;
}

static int as_u64(PyObject* o, uint64_t* v) {
  if (o == Py_None) {
    *v = 0;
    return 0;
  }
  *v = (uint64_t)PyLong_AsUnsignedLongLongMask(o);
  return (*v == (uint64_t)-1 && PyErr_Occurred()) ? -1 : 0;
}

static int as_int(PyObject* o, int* v) {
  long x = PyLong_AsLong(o);
  if (x == -1 && PyErr_Occurred()) return -1;
  *v = (int)x;
  return 0;
}

/* bind(kvx_swap_address, kvx_swap_blocks_address, kvx_migrate_blocks_address) */
static PyObject* py_bind(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  if (nargs != 3) {
    PyErr_SetString(PyExc_TypeError, "bind() takes 3 function addresses");
    return NULL;
  }
  uint64_t a, b, c;
  if (as_u64(args[0], &a) || as_u64(args[1], &b) || as_u64(args[2], &c)) return NULL;
  if (!a || !b || !c) {
    PyErr_SetString(PyExc_ValueError, "null function address");
    return NULL;
  }
  g_swap = (swap_fn)(uintptr_t)a;
  g_swap_blocks = (swap_blocks_fn)(uintptr_t)b;
  g_migrate_blocks = (migrate_blocks_fn)(uintptr_t)c;
  Py_RETURN_NONE;
}

static int bound(void) {
  if (g_swap && g_swap_blocks && g_migrate_blocks) return 1;
  PyErr_SetString(PyExc_RuntimeError, "kvx call shim used before bind()");
  return 0;
}

/* swap(source_ids, target_ids, is_swap_in, kv_cache, kv_cache_bytes,
 *      block_bytes, kv_swap, kv_swap_bytes, mode, stream) -> status */
static PyObject* py_swap(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  if (nargs != 10) {
    PyErr_SetString(PyExc_TypeError, "swap() takes 10 arguments");
    return NULL;
  }
  if (!bound()) return NULL;
  int is_in = PyObject_IsTrue(args[2]);
  if (is_in < 0) return NULL;
  uint64_t cache, cache_bytes, block_bytes, swap, swap_bytes, stream;
  int mode;
  if (as_u64(args[3], &cache) || as_u64(args[4], &cache_bytes) || as_u64(args[5], &block_bytes) ||
      as_u64(args[6], &swap) || as_u64(args[7], &swap_bytes) || as_int(args[8], &mode) ||
      as_u64(args[9], &stream))
    return NULL;
  int64_t ls[KVX_LOCAL_IDS], ld[KVX_LOCAL_IDS];
  Ids src, dst;
  if (ids_from(args[0], ls, &src)) return NULL;
  if (ids_from(args[1], ld, &dst)) {
    ids_release(&src);
    return NULL;
  }
  if (src.n != dst.n) {
    PyErr_Format(PyExc_ValueError,
                 "source_block_ids has %zd ids but target_block_ids has %zd", src.n, dst.n);
    ids_release(&src);
    ids_release(&dst);
    return NULL;
  }
  int rc;
  Py_BEGIN_ALLOW_THREADS
  rc = g_swap(src.data, dst.data, (int64_t)src.n, is_in, (void*)(uintptr_t)cache, cache_bytes,
              block_bytes, (void*)(uintptr_t)swap, swap_bytes, mode, (void*)(uintptr_t)stream);
  Py_END_ALLOW_THREADS
  ids_release(&src);
  ids_release(&dst);
  return PyLong_FromLong(rc);
}

/* The five entry lists of a segmented call (source, target, group, first,
 * valid) from args[first_arg..first_arg+4], then one library call:
 * `target` == 0 calls kvx_swap_blocks(source, ...), otherwise
 * kvx_migrate_blocks(source, target, ...).  Returns (status, copied, extents). */
static PyObject* entries_call(PyObject* const* args, int first_arg, uint64_t source,
                              uint64_t target, int is_in, int mode, uint64_t stream) {
  int64_t local[5][KVX_LOCAL_IDS];
  Ids ids[5];
  int got = 0;
  for (; got < 5; ++got)
    if (ids_from(args[first_arg + got], local[got], &ids[got])) break;
  PyObject* result = NULL;
  if (got == 5) {
    if (ids[0].n != ids[1].n || ids[0].n != ids[2].n || ids[0].n != ids[3].n ||
        ids[0].n != ids[4].n) {
      PyErr_Format(PyExc_ValueError,
                   "Swap block ids and metadata must have equal lengths: source=%zd, "
                   "target=%zd, groups=%zd, first=%zd, valid=%zd",
                   ids[0].n, ids[1].n, ids[2].n, ids[3].n, ids[4].n);
    } else {
      uint64_t copied = 0, extents = 0;
      int rc;
      Py_BEGIN_ALLOW_THREADS
      if (target)
        rc = g_migrate_blocks((kvx_layout*)(uintptr_t)source, (kvx_layout*)(uintptr_t)target,
                              (int64_t)ids[0].n, ids[0].data, ids[1].data, ids[2].data,
                              ids[3].data, ids[4].data, mode, (void*)(uintptr_t)stream,
                              &copied, &extents);
      else
        rc = g_swap_blocks((kvx_layout*)(uintptr_t)source, (int64_t)ids[0].n, ids[0].data,
                           ids[1].data, ids[2].data, ids[3].data, ids[4].data, is_in, mode,
                           (void*)(uintptr_t)stream, &copied, &extents);
      Py_END_ALLOW_THREADS
      result = Py_BuildValue("(iKK)", rc, (unsigned long long)copied,
                             (unsigned long long)extents);
    }
  }
  for (int i = 0; i < got; ++i) ids_release(&ids[i]);
  return result;
}

/* swap_blocks(layout, source_ids, target_ids, group_ids, first_kernel_blocks,
 *             valid_kernel_blocks, is_swap_in, mode, stream)
 *   -> (status, copied_bytes, copy_extents) */
static PyObject* py_swap_blocks(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  if (nargs != 9) {
    PyErr_SetString(PyExc_TypeError, "swap_blocks() takes 9 arguments");
    return NULL;
  }
  if (!bound()) return NULL;
  uint64_t layout, stream;
  int mode;
  int is_in = PyObject_IsTrue(args[6]);
  if (is_in < 0) return NULL;
  if (as_u64(args[0], &layout) || as_int(args[7], &mode) || as_u64(args[8], &stream))
    return NULL;
  if (!layout) {
    PyErr_SetString(PyExc_ValueError, "null layout");
    return NULL;
  }
  return entries_call(args, 1, layout, 0, is_in, mode, stream);
}

/* migrate_blocks(source_layout, target_layout, source_ids, target_ids,
 *                group_ids, first_kernel_blocks, valid_kernel_blocks, mode,
 *                stream) -> (status, copied_bytes, copy_extents) */
static PyObject* py_migrate_blocks(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  if (nargs != 9) {
    PyErr_SetString(PyExc_TypeError, "migrate_blocks() takes 9 arguments");
    return NULL;
  }
  if (!bound()) return NULL;
  uint64_t source, target, stream;
  int mode;
  if (as_u64(args[0], &source) || as_u64(args[1], &target) || as_int(args[7], &mode) ||
      as_u64(args[8], &stream))
    return NULL;
  if (!source || !target) {
    PyErr_SetString(PyExc_ValueError, "null layout");
    return NULL;
  }
  return entries_call(args, 2, source, target, 0, mode, stream);
}

static PyMethodDef kMethods[] = {
    {"bind", (PyCFunction)(void (*)(void))py_bind, METH_FASTCALL,
     "bind(kvx_swap_address, kvx_swap_blocks_address)"},
    {"swap", (PyCFunction)(void (*)(void))py_swap, METH_FASTCALL,
     "kvx_swap with ids from Python sequences; returns the status"},
    {"swap_blocks", (PyCFunction)(void (*)(void))py_swap_blocks, METH_FASTCALL,
     "kvx_swap_blocks with ids from Python sequences; returns (status, copied, extents)"},
    {"migrate_blocks", (PyCFunction)(void (*)(void))py_migrate_blocks, METH_FASTCALL,
     "kvx_migrate_blocks with ids from Python sequences; returns (status, copied, extents)"},
    {NULL, NULL, 0, NULL},
};

static struct PyModuleDef kModule = {
    PyModuleDef_HEAD_INIT, "_kvxcall", "Python call shim of libkvx.so", -1, kMethods,
    NULL, NULL, NULL, NULL};

PyMODINIT_FUNC PyInit__kvxcall(void) { return PyModule_Create(&kModule); }
