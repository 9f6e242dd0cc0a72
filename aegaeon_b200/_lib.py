"""ctypes binding of libkvx.so (the C ABI declared in include/kvx.h).

The shared library is built in-tree (``aegaeon_b200/libkvx.so``, see
``aegaeon_b200/build.py``).  There is no fallback: if it is missing, every
entry point raises ``RuntimeError`` naming the build command.
"""

from __future__ import annotations

import array
import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libkvx.so")

KVX_OK = 0
KVX_ERR_INVALID_ARGUMENT = 1
KVX_ERR_LENGTH_MISMATCH = 2
KVX_ERR_GROUP = 3
KVX_ERR_EXTENT = 4
KVX_ERR_BLOCK_ID = 5
KVX_ERR_HOST_MEMORY = 6
KVX_ERR_CUDA = 7
KVX_ERR_DEVICE_TIMEOUT = 8
KVX_ERR_LAYOUT = 9
KVX_ERR_NO_MEMORY = 10
KVX_ERR_IO = 11
KVX_ERR_FORMAT = 12

MODE_AUTO = 0
MODE_SM = 1
MODE_CE = 2
MODE_SM_BULK = 3
MODE_CE_EXTENT = 4
MODE_NAMES = {
    "auto": MODE_AUTO,
    "sm": MODE_SM,
    "ce": MODE_CE,
    "sm_bulk": MODE_SM_BULK,
    "ce_extent": MODE_CE_EXTENT,
}

_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_int = ctypes.c_int
_vp = ctypes.c_void_p
_p_i64 = ctypes.POINTER(_i64)
_p_u64 = ctypes.POINTER(_u64)

# name -> (restype, argtypes); kept in the order of include/kvx.h.
SIGNATURES = {
    "kvx_status_string": (ctypes.c_char_p, [_int]),
    "kvx_last_error": (ctypes.c_char_p, []),
    "kvx_version": (_int, []),
    "kvx_swap": (_int, [_p_i64, _p_i64, _i64, _int, _vp, _u64, _u64, _vp, _u64, _int, _vp]),
    "kvx_layout_create": (
        _int,
        [_int, _i64, ctypes.POINTER(_vp), _p_u64, _p_u64, _p_u64, _p_u64, _i64, _p_i64,
         _vp, _u64, _u64, _u64, ctypes.POINTER(_vp)],
    ),
    "kvx_layout_destroy": (_int, [_vp]),
    "kvx_swap_blocks": (
        _int,
        [_vp, _i64, _p_i64, _p_i64, _p_i64, _p_i64, _p_i64, _int, _int, _vp, _p_u64, _p_u64],
    ),
    "kvx_migrate_blocks": (
        _int,
        [_vp, _vp, _i64, _p_i64, _p_i64, _p_i64, _p_i64, _p_i64, _int, _vp, _p_u64, _p_u64],
    ),
    "kvx_ipc_export": (_int, [_vp, ctypes.POINTER(ctypes.c_uint8), _p_u64]),
    "kvx_ipc_import": (_int, [_int, ctypes.POINTER(ctypes.c_uint8), _u64, ctypes.POINTER(_vp)]),
    "kvx_ipc_close": (_int, [_int, _vp]),
    "kvx_event_create": (_int, [_int, ctypes.POINTER(_vp)]),
    "kvx_event_record": (_int, [_vp, _vp]),
    "kvx_event_query": (_int, [_vp, ctypes.POINTER(_int)]),
    "kvx_event_synchronize": (_int, [_vp]),
    "kvx_event_ipc_handle": (_int, [_vp, ctypes.POINTER(ctypes.c_uint8)]),
    "kvx_event_open_ipc": (_int, [ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(_vp)]),
    "kvx_event_forget_ipc": (_int, [ctypes.POINTER(ctypes.c_uint8)]),
    "kvx_stream_wait_events": (_int, [_vp, ctypes.POINTER(_vp), _i64]),
    "kvx_event_release": (_int, [_vp]),
    "kvx_upload_chunked": (_int, [_vp, _vp, _u64, _u64, _vp]),
    "kvx_upload_weights": (_int, [ctypes.POINTER(_vp), ctypes.POINTER(_vp), _p_u64, _i64, _u64,
                                  _int, _vp]),
    "kvx_byte_extent": (_int, [_u64, _i64, _i64, _i64, _p_u64, _p_u64]),
    "kvx_plan_swap_blocks": (
        _int,
        [_vp, _i64, _p_i64, _p_i64, _p_i64, _p_i64, _p_i64, _int, _p_u64, _p_u64, _p_u64, _p_i64],
    ),
    "kvx_plan_swap": (
        _int,
        [_p_i64, _p_i64, _i64, _int, _u64, _u64, _u64, _u64, _u64, _p_u64, _p_u64, _p_u64, _p_i64],
    ),
    "kvx_last_mode": (_int, []),
    "kvx_kernel_launches": (_u64, []),
    "kvx_kernel_timing": (_int, [_int]),
    "kvx_kernel_timing_read": (_int, [_p_u64, ctypes.POINTER(ctypes.c_double),
                                       ctypes.POINTER(ctypes.c_double), _p_u64]),
    "kvx_device_status": (_int, [_int, _int, ctypes.POINTER(_int)]),
    "kvx_selftest_bounded_wait": (_int, [_u64, _vp]),
    "kvx_configure": (_int, [_i64, _i64, _i64, _i64, _i64]),
    "kvx_set_option": (_int, [ctypes.c_char_p, _i64]),
    "kvx_swap_noalloc": (_int, [_p_i64, _p_i64, _i64, _int, _vp, _u64, _u64, _vp, _u64, _vp]),
    "kvx_safetensors_meta_json": (_int, [ctypes.c_char_p, ctypes.c_char_p, _u64, _p_u64]),
}

_lock = threading.Lock()
_lib = None


class KvxError(RuntimeError):
    """A libkvx call failed with a CUDA or device-side error."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def lib() -> ctypes.CDLL:
    """Load libkvx.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing; build it with "
                    "`python -c 'import __graft_entry__ as g; g.build()'` "
                    "or `python -m aegaeon_b200.build`"
                )
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


_shim = None


def shim():
    """The compiled call shim (``aegaeon_b200/_kvxcall*.so``, built with the
    library) bound to the functions of ``lib()``; raises if it is missing."""
    global _shim
    if _shim is not None:
        return _shim
    handle = lib()
    with _lock:
        if _shim is None:
            try:
                from . import _kvxcall
            except ImportError as e:
                raise RuntimeError(
                    f"the kvx call shim is missing ({e}); build it with "
                    "`python -c 'import __graft_entry__ as g; g.build()'` "
                    "or `python -m aegaeon_b200.build`"
                ) from e
            _kvxcall.bind(ctypes.cast(handle.kvx_swap, ctypes.c_void_p).value,
                          ctypes.cast(handle.kvx_swap_blocks, ctypes.c_void_p).value,
                          ctypes.cast(handle.kvx_migrate_blocks, ctypes.c_void_p).value)
            _shim = _kvxcall
    return _shim


def ids_arg(values):
    """Block ids as the call shim takes them: lists and tuples as they are,
    anything else (numpy arrays, tensors, ranges) as an int64 C array."""
    return values if isinstance(values, (list, tuple)) else i64_array(values)


def check(status: int) -> None:
    """Map a kvx status to the exception type the reference raises."""
    if status == KVX_OK:
        return
    msg = lib().kvx_last_error().decode(errors="replace") or lib().kvx_status_string(
        status
    ).decode()
    if status in (KVX_ERR_LENGTH_MISMATCH, KVX_ERR_GROUP, KVX_ERR_EXTENT, KVX_ERR_LAYOUT):
        raise ValueError(msg)
    if status == KVX_ERR_BLOCK_ID:
        raise IndexError(msg)
    if status in (KVX_ERR_INVALID_ARGUMENT, KVX_ERR_HOST_MEMORY):
        raise ValueError(msg)
    raise KvxError(status, msg)


def i64_array(values) -> ctypes.Array:
    """Block ids (list, tuple, range, array, numpy array or CPU/CUDA tensor)
    -> contiguous int64 C array.  Non-integer ids raise TypeError, ids outside
    int64 OverflowError."""
    if isinstance(values, (list, tuple, range)):
        # One C-level pass that rejects ids outside int64; the ctypes view
        # keeps the array alive.
        a = array.array("q", values)
        return (ctypes.c_int64 * len(a)).from_buffer(a) if len(a) else (ctypes.c_int64 * 0)()
    import numpy as np

    if hasattr(values, "detach") and hasattr(values, "cpu"):  # torch tensor
        values = values.detach().cpu().numpy()
    # One conversion into a fresh int64 array, then a zero-copy ctypes view
    # (the view keeps the array alive); much faster than building the ctypes
    # array element by element for long id lists.
    a = np.array(values, dtype=np.int64).reshape(-1)
    if a.size == 0:
        return (ctypes.c_int64 * 0)()
    return (ctypes.c_int64 * a.size).from_buffer(a)


def current_stream_handle(device_index: int) -> int:
    """cudaStream_t of the current torch stream of a device (torch's own raw
    accessor where it exists: several microseconds cheaper per call)."""
    import torch

    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return raw(device_index)
    return torch.cuda.current_stream(device_index).cuda_stream


def mode_of(mode) -> int:
    if isinstance(mode, str):
        try:
            return MODE_NAMES[mode]
        except KeyError:
            raise ValueError(f"unknown transfer mode {mode!r}; one of {sorted(MODE_NAMES)}")
    return int(mode)


def last_mode_name() -> str:
    m = lib().kvx_last_mode()
    for k, v in MODE_NAMES.items():
        if v == m:
            return k
    return str(m)


def configure(sm_ctas_host: int = 0, sm_ctas_dev: int = 0, ce_min_run: int = 0,
              staging_bytes: int = 0, ce_pipeline: int = -1) -> None:
    """Set the tuning knobs of the transfer-mode policy (0 keeps a value;
    ce_min_run < 0 disables the copy-engine choice of the AUTO mode;
    ce_pipeline: -1 keeps, 0 off, 1 double-buffered staging)."""
    check(lib().kvx_configure(sm_ctas_host, sm_ctas_dev, ce_min_run, staging_bytes,
                              ce_pipeline))


def set_option(name: str, value: int) -> None:
    """Set one tuning knob of the library by name (kvx_set_option)."""
    check(lib().kvx_set_option(name.encode(), int(value)))


def device_status(device: int, reset: bool = False) -> int:
    """Device error word written by kernels whose bounded waits gave up."""
    out = ctypes.c_int(0)
    check(lib().kvx_device_status(device, 1 if reset else 0, ctypes.byref(out)))
    return out.value


def kernel_timing(enable: bool) -> None:
    """Bracket every copy-kernel launch with CUDA events (see kvx.h)."""
    check(lib().kvx_kernel_timing(1 if enable else 0))


def kernel_timing_read() -> tuple[int, float, float, int]:
    """(launches, summed kernel ms, busy ms with overlaps counted once, HBM
    bytes) since the last read."""
    n = ctypes.c_uint64()
    ms = ctypes.c_double()
    busy = ctypes.c_double()
    b = ctypes.c_uint64()
    check(lib().kvx_kernel_timing_read(ctypes.byref(n), ctypes.byref(ms), ctypes.byref(busy),
                                       ctypes.byref(b)))
    return n.value, ms.value, busy.value, b.value
