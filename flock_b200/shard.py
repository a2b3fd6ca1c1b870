"""Tensor parallelism -- the kernels/shard.ts and shard_ref.ts planning surface.

Host-side planning (pure logic, mirrors kernels/shard_ref.ts):
    shard_ranges (:97), slice_rows (:137), slice_cols (:166),
    reduce_shard_argmax (:437), mem_shard_plan (:509)
GPU objects (C ABI):
    ShardedMatvec (shard.ts:138) -- N shards of one Q8_0 matrix, row-wise
        (output-split, concatenated, bit-identical to unsharded) or col-wise
        (input-split, partials summed serially in shard order);
    ShardedHead (shard.ts:459) -- row-sharded LM head with a per-shard argmax
        and the lowest-index cross-shard reduce.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np

from . import _abi
from .lib import Device, Q8_BLOCK


@dataclass(frozen=True)
class ShardRange:
    index: int
    start: int
    end: int
    count: int


def shard_ranges(total: int, n: int, align: int = 1) -> list[ShardRange]:
    """shard_ref.ts:97 -- remainder spread over the first shards."""
    if not isinstance(n, int) or n < 1:
        raise ValueError(f"n shards must be >= 1, got {n}")
    if not isinstance(total, int) or total < 0:
        raise ValueError(f"total must be >= 0, got {total}")
    if not isinstance(align, int) or align < 1:
        raise ValueError(f"align must be >= 1, got {align}")
    if total % align != 0:
        raise ValueError(f"total {total} is not a multiple of align {align}")
    units = total // align
    if units < n:
        raise ValueError(f"cannot cut {total} into {n} shards aligned to {align}: only {units} units")
    base, extra = divmod(units, n)
    out, at = [], 0
    for i in range(n):
        count = (base + (1 if i < extra else 0)) * align
        out.append(ShardRange(i, at, at + count, count))
        at += count
    return out


def slice_rows(qs: np.ndarray, scales: np.ndarray, rows: int, cols: int, start: int, end: int):
    """shard_ref.ts:137 -- rows [start, end) of a split tensor (views)."""
    if start < 0 or end > rows or start > end:
        raise ValueError(f"row range {start}..{end} is not inside 0..{rows}")
    nb = cols // Q8_BLOCK
    return qs[start * cols:end * cols], scales[start * nb * 2:end * nb * 2]


def slice_cols(qs: np.ndarray, scales: np.ndarray, rows: int, cols: int, start: int, end: int):
    """shard_ref.ts:166 -- columns [start, end) of every row (a gather)."""
    if start % Q8_BLOCK or end % Q8_BLOCK:
        raise ValueError(f"column range {start}..{end} must be multiples of {Q8_BLOCK}: "
                         "a Q8_0 block's scale cannot be split")
    if start < 0 or end > cols or start > end:
        raise ValueError(f"column range {start}..{end} is not inside 0..{cols}")
    nb = cols // 32
    q = qs.reshape(rows, cols)[:, start:end].reshape(-1).copy()
    s = scales.reshape(rows, nb * 2)[:, start // 32 * 2:end // 32 * 2].reshape(-1).copy()
    return q, s


def reduce_shard_argmax(parts: list[tuple[float, int, int]]) -> int:
    """shard_ref.ts:437 -- parts are (value, index within shard, row offset)."""
    if not parts:
        raise ValueError("nothing to reduce")
    bi, bv = -1, -math.inf
    for value, index, row_offset in parts:
        gi = row_offset + index
        if value > bv or (value == bv and gi < bi):
            bv, bi = value, gi
    return bi


def mem_shard_plan(rows: int, cols: int, n: int, direction: str = "row",
                   limit_bytes: int = 128 * 1024 * 1024, bytes_per_weight: float = 1.0,
                   scale_bytes_per_block: float = 2.0) -> dict:
    """shard_ref.ts:509 -- per-shard largest binding and the minimum shard count."""
    def per(r, c):
        qs = r * c * bytes_per_weight
        sc = r * math.ceil(c / Q8_BLOCK) * scale_bytes_per_block
        return max(qs, sc), qs + sc

    def rng(k):
        return shard_ranges(rows, k, 1) if direction == "row" else shard_ranges(cols, k, Q8_BLOCK)

    shards = [per(rg.count, cols) if direction == "row" else per(rows, rg.count) for rg in rng(n)]
    max_binding = max(b for b, _ in shards)
    min_n = None
    max_n = rows if direction == "row" else cols // Q8_BLOCK
    for k in range(1, max_n + 1):
        first = rng(k)[0].count  # the first shard carries the remainder: the largest
        m = per(first, cols)[0] if direction == "row" else per(rows, first)[0]
        if m <= limit_bytes:
            min_n = k
            break
    return {"max_binding_bytes": max_binding, "unsharded_max_binding_bytes": per(rows, cols)[0],
            "min_shards_for_limit": min_n, "limit_bytes": limit_bytes,
            "fits": max_binding <= limit_bytes,
            "shards": [{"max_binding_bytes": b, "total_bytes": t} for b, t in shards]}


class ShardedMatvec:
    """shard.ts:138 -- y = W x with W held as N shards on one device."""

    def __init__(self, dev: Device, handle, rows: int, cols: int, n: int, direction: str):
        self.dev, self.handle, self.rows, self.cols, self.n, self.direction = (
            dev, handle, rows, cols, n, direction)
        self.ranges = (shard_ranges(rows, n, 1) if direction == "row"
                       else shard_ranges(cols, n, Q8_BLOCK))

    @staticmethod
    def create(dev: Device, qs: np.ndarray, scales: np.ndarray, rows: int, cols: int, n: int,
               direction: str = "row", binding_limit: int | None = None) -> "ShardedMatvec":
        qs = np.ascontiguousarray(qs, np.uint8)
        scales = np.ascontiguousarray(scales, np.uint8)
        h = ctypes.c_void_p()
        _abi.call("flock_shard_matvec_create", dev.handle, _abi.ptr(qs, _abi._u8p),
                  _abi.ptr(scales, _abi._u8p), rows, cols, n, 0 if direction == "row" else 1,
                  binding_limit or 0, ctypes.byref(h))
        return ShardedMatvec(dev, h, rows, cols, n, direction)

    def run(self, x: np.ndarray) -> np.ndarray:
        """setInput + encode + output (shard.ts:320, :340, :400)."""
        x = np.ascontiguousarray(x, np.float32)
        if x.size != self.cols:
            raise ValueError(f"x is {x.size} floats, want {self.cols}")
        y = np.empty(self.rows, np.float32)
        _abi.call("flock_shard_matvec_run", self.handle, _abi.ptr(x, _abi._fp), _abi.ptr(y, _abi._fp))
        return y

    def partials(self) -> np.ndarray:
        """shard.ts:405 -- [n][rows] (column-wise only)."""
        p = np.empty(self.n * self.rows, np.float32)
        _abi.call("flock_shard_matvec_partials", self.handle, _abi.ptr(p, _abi._fp))
        return p.reshape(self.n, self.rows)

    def wire_bytes_per_call(self) -> int:
        n = ctypes.c_int64()
        _abi.call("flock_shard_matvec_wire_bytes", self.handle, ctypes.byref(n))
        return n.value

    def destroy(self) -> None:
        if self.handle:
            _abi.lib().flock_shard_matvec_free(self.handle)
            self.handle = None

    __del__ = destroy


class ShardedHead:
    """shard.ts:459 -- row-sharded LM head, argmax per shard, lowest index wins."""

    def __init__(self, dev: Device, handle, vocab: int, hidden: int, n: int):
        self.dev, self.handle, self.vocab, self.hidden, self.n = dev, handle, vocab, hidden, n
        self.ranges = shard_ranges(vocab, n, 1)

    @staticmethod
    def create(dev: Device, qs: np.ndarray, scales: np.ndarray, vocab: int, hidden: int,
               shards: int) -> "ShardedHead":
        qs = np.ascontiguousarray(qs, np.uint8)
        scales = np.ascontiguousarray(scales, np.uint8)
        h = ctypes.c_void_p()
        _abi.call("flock_sharded_head_create", dev.handle, _abi.ptr(qs, _abi._u8p),
                  _abi.ptr(scales, _abi._u8p), vocab, hidden, shards, ctypes.byref(h))
        return ShardedHead(dev, h, vocab, hidden, shards)

    def run(self, x: np.ndarray, want_logits: bool = True):
        x = np.ascontiguousarray(x, np.float32)
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        tok = ctypes.c_int32()
        _abi.call("flock_sharded_head_run", self.handle, _abi.ptr(x, _abi._fp),
                  _abi.ptr(logits, _abi._fp) if want_logits else None, ctypes.byref(tok))
        return tok.value, logits

    def argmax_buffers(self) -> list[tuple[float, int, int]]:
        """shard.ts:632 -- per-shard (value, index within shard, row offset)."""
        v = np.empty(self.n, np.float32)
        i = np.empty(self.n, np.int64)
        o = np.empty(self.n, np.int64)
        _abi.call("flock_sharded_head_shard_argmax", self.handle, _abi.ptr(v, _abi._fp),
                  _abi.ptr(i, _abi._i64p), _abi.ptr(o, _abi._i64p))
        return [(float(v[k]), int(i[k]), int(o[k])) for k in range(self.n)]

    def destroy(self) -> None:
        if self.handle:
            _abi.lib().flock_sharded_head_free(self.handle)
            self.handle = None

    __del__ = destroy
