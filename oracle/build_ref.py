"""Compile the reference's own swap op (ops/ops.cpp + ops/swap.cu, read in
place from the reference checkout) into oracle/_ref/.

TEST INFRASTRUCTURE ONLY: the resulting module is the reference
implementation that tests/ and bench.py's reference arm compare against.

The recipe is torch.utils.cpp_extension with the two source files where they
lie; it does not run the reference's setup.py.  The module is named
``aegaeon_ref_ops`` and exports ``swap(source_block_ids, target_block_ids,
is_swap_in, kv_cache, kv_swap)`` exactly as the reference's pybind module
(ops/ops.cpp:4-6).  Output: oracle/_ref/aegaeon_ref_ops*.so (git-ignored;
travels to the GPU box with the working tree).
"""

from __future__ import annotations

import glob
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
# The Aegaeon checkout: AEGAEON_REFERENCE, else a directory named "reference"
# beside this repository's root.
DEFAULT_REFERENCE = os.environ.get(
    "AEGAEON_REFERENCE", os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))


def built_module_path() -> str | None:
    hits = sorted(glob.glob(os.path.join(REF_DIR, "aegaeon_ref_ops*.so")))
    return hits[0] if hits else None


def build(reference_root: str = DEFAULT_REFERENCE, verbose: bool = False) -> str | None:
    """Build if the reference checkout is present; return the .so path."""
    ops = os.path.join(reference_root, "ops")
    sources = [os.path.join(ops, "ops.cpp"), os.path.join(ops, "swap.cu")]
    if not all(os.path.exists(p) for p in sources):
        return built_module_path()
    existing = built_module_path()
    if existing and all(os.path.getmtime(existing) >= os.path.getmtime(p) for p in sources):
        return existing
    from torch.utils.cpp_extension import load

    build_dir = os.path.join(REF_DIR, "build")
    os.makedirs(build_dir, exist_ok=True)
    load(
        name="aegaeon_ref_ops",
        sources=sources,
        build_directory=build_dir,
        extra_cuda_cflags=["-gencode", "arch=compute_100a,code=sm_100a"],
        verbose=verbose,
        is_python_module=True,
    )
    so = sorted(glob.glob(os.path.join(build_dir, "aegaeon_ref_ops*.so")))
    if not so:
        raise RuntimeError("reference op build produced no module")
    target = os.path.join(REF_DIR, os.path.basename(so[0]))
    os.replace(so[0], target)
    return target


def load_module():
    """Import the built reference op module (requires torch imported)."""
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401  (the module links against torch)

    path = built_module_path()
    if not path:
        raise FileNotFoundError("oracle/_ref has no built reference op; run oracle/build_ref.py")
    loader = importlib.machinery.ExtensionFileLoader("aegaeon_ref_ops", path)
    spec = importlib.util.spec_from_file_location("aegaeon_ref_ops", path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else DEFAULT_REFERENCE, verbose=True))
