"""flock_b200 -- B200-native replacement for flock's per-token Qwen3 hot path.

The compute path is hand-written sm_100a CUDA behind a C-ABI shared library
(``libflock_cuda.so``, declared in ``include/flock_cuda.h``).  The Python
modules mirror the reference's ``kernels/`` module surface so a caller of
``kernels/lib.ts``, ``layer.ts``, ``model.ts`` and ``shard.ts`` finds the same
names here: ``lib``, ``layer`` (``Layer``, ``QWEN3_06B``), ``model``
(``Model``) and ``shard`` (``ShardedMatvec``, ``ShardedHead``).
"""
