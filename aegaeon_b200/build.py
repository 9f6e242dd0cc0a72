"""Build libkvx.so in-tree for sm_100a with nvcc.

``python -m aegaeon_b200.build`` (or ``__graft_entry__.build()``).  The
library links the CUDA runtime statically so that it does not depend on which
libcudart another extension in the process loaded first.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SOURCES = [
    os.path.join(HERE, "csrc", "kvx_plan.cpp"),
    os.path.join(HERE, "csrc", "kvx_runtime.cu"),
    os.path.join(HERE, "csrc", "kvx_noalloc.cu"),
    os.path.join(HERE, "csrc", "kvx_safetensors.cpp"),
    os.path.join(HERE, "csrc", "kvx_events.cu"),
]
HEADERS = [
    os.path.join(HERE, "csrc", "kvx_plan.h"),
    os.path.join(HERE, "csrc", "kvx_worklist.h"),
    os.path.join(HERE, "csrc", "kvx_kernels.cuh"),
    os.path.join(ROOT, "include", "kvx.h"),
]
OUT = os.path.join(HERE, "libkvx.so")
SHIM_SOURCE = os.path.join(HERE, "csrc", "kvx_pycall.c")
SHIM_OUT = os.path.join(HERE, "_kvxcall" + sysconfig.get_config_var("EXT_SUFFIX"))
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(p) <= t for p in SOURCES + HEADERS)


def build_shim(force: bool = False) -> str:
    """The Python call shim (plain C against the CPython headers; it reaches
    libkvx.so through function pointers handed over at import)."""
    deps = [SHIM_SOURCE, os.path.join(ROOT, "include", "kvx.h")]
    if (not force and os.path.exists(SHIM_OUT)
            and all(os.path.getmtime(p) <= os.path.getmtime(SHIM_OUT) for p in deps)):
        return SHIM_OUT
    cc = os.environ.get("CC") or shutil.which("gcc") or "cc"
    cmd = [cc, "-O2", "-Wall", "-shared", "-fPIC", "-I" + sysconfig.get_paths()["include"],
           SHIM_SOURCE, "-o", SHIM_OUT + ".tmp"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"{cc} failed ({res.returncode}):\n{res.stderr}\n{res.stdout}")
    os.replace(SHIM_OUT + ".tmp", SHIM_OUT)
    return SHIM_OUT


def build(force: bool = False, verbose: bool = False) -> str:
    build_shim(force)
    if not force and up_to_date():
        return OUT
    cmd = [
        nvcc(), "-O3", "-std=c++17", *ARCH_FLAGS, "-lineinfo",
        "-Xcompiler", "-fPIC,-Wall", "-shared", "-cudart", "static",
        *SOURCES, "-o", OUT + ".tmp",
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr}\n{res.stdout}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
