"""aegaeon_b200 - B200-native KV-cache movement (swap-out / swap-in between
HBM and page-locked host slots, GPU->GPU migration over NVLink) behind the
reference Aegaeon's own operator interfaces.

Modules:
  ops             drop-in for ``aegaeon.ops.swap`` (ops/swap.cu)
  swapper         ``Worker.swap_blocks`` / migration executor (worker.py)
  cache_transfer  extent arithmetic (aegaeon/cache_transfer.py)
  block_table     transfer planning (aegaeon/block_manager.py)
  switch          chunked weight upload overlapped with KV swap-in
  _lib            ctypes binding of libkvx.so (include/kvx.h)
"""

__version__ = "0.1.0"
