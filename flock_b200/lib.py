"""Host-side plumbing mirroring kernels/lib.ts: quantizers, repack, device,
GPU tensors and comparison helpers.

Names follow the reference (kernels/lib.ts) in Python spelling:

    quantRowQ8 -> quant_row_q8        splitQ8 -> split_q8 (C ABI, bit-exact)
    quantMatrixQ8 -> quant_matrix_q8  getDevice -> get_device
    halfToF32 -> half_to_f32          maxRelErr -> max_rel_err

The reference's strict-f32 CPU references (cpuMatmulQ8F32, coop, SERIAL,
fma32) are the parity oracle and live in the repository's ``oracle/``
package, which only tests import; they are not part of the product.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _abi
from ._abi import FLOCK_F32, FLOCK_Q4_0, FLOCK_Q8_0, FlockError

Q8_BLOCK = 32
Q8_BYTES = 34  # f16 scale + 32 int8
Q4_BLOCK = 32
Q4_BYTES = 18  # f16 scale + 16 packed nibble pairs


def half_to_f32(h: int) -> float:
    """kernels/lib.ts:30 -- f16 bits to a number; inf/nan clamp to max finite."""
    s = -1.0 if (h & 0x8000) else 1.0
    e = (h >> 10) & 0x1F
    m = h & 0x3FF
    if e == 0:
        return s * m * 2.0 ** -24
    if e == 31:
        return s * 3.4028235e38
    return s * (1 + m / 1024) * 2.0 ** (e - 15)


def _f32to16(d: np.ndarray) -> np.ndarray:
    """web/js/wire.mjs:309 f32to16 on an array: round to f32, then RNE to f16."""
    with np.errstate(over="ignore"):
        return d.astype(np.float32).astype(np.float16).view(np.uint16)


def _js_round(x: np.ndarray) -> np.ndarray:
    """Math.round: halves go toward +infinity."""
    r = np.floor(x)
    return np.where(x - r >= 0.5, r + 1.0, r)


def quant_matrix_q8(w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """kernels/lib.ts:94 quantMatrixQ8 (each row as lib.ts:40 quantRowQ8)."""
    if cols % Q8_BLOCK:
        raise ValueError(f"cols {cols} must be a multiple of {Q8_BLOCK}")
    v = np.asarray(w, np.float32).reshape(rows * (cols // 32), 32).astype(np.float64)
    amax = np.abs(v).max(axis=1)
    d = amax / 127.0
    out = np.empty((v.shape[0], Q8_BYTES), np.uint8)
    out[:, 0:2] = _f32to16(d).view(np.uint8).reshape(-1, 2)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(d[:, None] == 0, 0.0, _js_round(v / d[:, None]))
    out[:, 2:] = (np.clip(q, -128, 127).astype(np.int64) & 0xFF).astype(np.uint8)
    return out.reshape(-1)


def quant_row_q8(vals: np.ndarray) -> np.ndarray:
    """kernels/lib.ts:40 quantRowQ8."""
    return quant_matrix_q8(vals, 1, len(vals))


def quant_matrix_q4(w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """kernels/lib.ts:103 quantMatrixQ4 (each row as lib.ts:64 quantRowQ4)."""
    if cols % Q4_BLOCK:
        raise ValueError(f"cols {cols} must be a multiple of {Q4_BLOCK}")
    v = np.asarray(w, np.float32).reshape(rows * (cols // 32), 32).astype(np.float64)
    # the first value of largest magnitude keeps its sign (strict > scan)
    idx = np.argmax(np.abs(v), axis=1)
    mx = v[np.arange(v.shape[0]), idx]
    d = mx / -8.0
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, 0.0, 1.0 / np.where(d == 0, 1.0, d))
    out = np.empty((v.shape[0], Q4_BYTES), np.uint8)
    out[:, 0:2] = _f32to16(d).view(np.uint8).reshape(-1, 2)
    x0 = v[:, :16] * inv[:, None] + 8.5
    x1 = v[:, 16:] * inv[:, None] + 8.5
    q0 = np.clip(np.floor(x0), 0, 15).astype(np.uint8)
    q1 = np.clip(np.floor(x1), 0, 15).astype(np.uint8)
    out[:, 2:] = q0 | (q1 << 4)
    return out.reshape(-1)


def quant_row_q4(vals: np.ndarray) -> np.ndarray:
    """kernels/lib.ts:64 quantRowQ4."""
    return quant_matrix_q4(vals, 1, len(vals))


def split_q8(packed: np.ndarray, rows: int, cols: int) -> tuple[np.ndarray, np.ndarray]:
    """kernels/lib.ts:126 splitQ8, done by the C ABI (flock_repack_q8)."""
    packed = np.ascontiguousarray(packed, np.uint8)
    qs = np.empty(rows * cols, np.uint8)
    sc = np.empty(rows * (cols // 32) * 2, np.uint8)
    _abi.call("flock_repack_q8", _abi.ptr(packed, _abi._u8p), rows, cols, _abi.ptr(qs, _abi._u8p),
              _abi.ptr(sc, _abi._u8p))
    return qs, sc


def split_q4(packed: np.ndarray, rows: int, cols: int) -> tuple[np.ndarray, np.ndarray]:
    """kernels/lib.ts:142 splitQ4, done by the C ABI (flock_repack_q4)."""
    packed = np.ascontiguousarray(packed, np.uint8)
    qs = np.empty(rows * (cols // 32) * 16, np.uint8)
    sc = np.empty(rows * (cols // 32) * 2, np.uint8)
    _abi.call("flock_repack_q4", _abi.ptr(packed, _abi._u8p), rows, cols, _abi.ptr(qs, _abi._u8p),
              _abi.ptr(sc, _abi._u8p))
    return qs, sc


class Device:
    """kernels/lib.ts:385 getDevice(): one GPU with its own CUDA stream."""

    def __init__(self, ordinal: int = 0):
        h = ctypes.c_void_p()
        _abi.call("flock_dev_open", ordinal, ctypes.byref(h))
        self.handle = h
        self.ordinal = ordinal

    def close(self) -> None:
        if self.handle:
            _abi.lib().flock_dev_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def sync(self) -> None:
        _abi.call("flock_dev_sync", self.handle)

    @property
    def sm_count(self) -> int:
        n = ctypes.c_int()
        _abi.call("flock_dev_sm_count", self.handle, ctypes.byref(n))
        return n.value

    def timer_start(self) -> None:
        _abi.call("flock_dev_timer_start", self.handle)

    def timer_stop(self) -> float:
        ms = ctypes.c_float()
        _abi.call("flock_dev_timer_stop", self.handle, ctypes.byref(ms))
        return ms.value


def get_device(ordinal: int = 0) -> Device:
    return Device(ordinal)


class GpuTensor:
    """kernels/layer.ts:73 GpuTensor: a Q8_0/Q4_0 tensor in split planes or f32 data."""

    def __init__(self, dev: Device, handle: ctypes.c_void_p, rows: int, cols: int, dtype: int):
        self.dev, self.handle, self.rows, self.cols, self.dtype = dev, handle, rows, cols, dtype

    @staticmethod
    def from_packed(dev: Device, packed: np.ndarray, rows: int, cols: int,
                    dtype: int = FLOCK_Q8_0) -> "GpuTensor":
        packed = np.ascontiguousarray(packed, np.uint8)
        h = ctypes.c_void_p()
        _abi.call("flock_tensor_from_packed", dev.handle, dtype, _abi.ptr(packed, _abi._u8p), rows,
                  cols, ctypes.byref(h))
        return GpuTensor(dev, h, rows, cols, dtype)

    @staticmethod
    def from_split(dev: Device, qs: np.ndarray, scales: np.ndarray, rows: int, cols: int,
                   dtype: int = FLOCK_Q8_0) -> "GpuTensor":
        qs = np.ascontiguousarray(qs, np.uint8)
        scales = np.ascontiguousarray(scales, np.uint8)
        h = ctypes.c_void_p()
        _abi.call("flock_tensor_from_split", dev.handle, dtype, _abi.ptr(qs, _abi._u8p),
                  _abi.ptr(scales, _abi._u8p), rows, cols, ctypes.byref(h))
        return GpuTensor(dev, h, rows, cols, dtype)

    @staticmethod
    def from_f32(dev: Device, data: np.ndarray) -> "GpuTensor":
        data = np.ascontiguousarray(data, np.float32)
        h = ctypes.c_void_p()
        _abi.call("flock_tensor_from_f32", dev.handle, _abi.ptr(data, _abi._fp), data.size,
                  ctypes.byref(h))
        return GpuTensor(dev, h, 1, data.size, FLOCK_F32)

    @property
    def nbytes(self) -> int:
        n = ctypes.c_int64()
        _abi.call("flock_tensor_bytes", self.handle, ctypes.byref(n))
        return n.value

    def free(self) -> None:
        if self.handle:
            _abi.lib().flock_tensor_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def max_rel_err(a: np.ndarray, b: np.ndarray) -> float:
    """kernels/lib.ts:322 maxRelErr (1e-6 floor on the denominator)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b) / np.maximum(1e-6, np.abs(b)))) if a.size else 0.0


def rand_vec(n: int, scale: float = 1.0, seed: int | None = None) -> np.ndarray:
    """kernels/lib.ts:595 randVec: uniform in [-scale, scale) (seedable here)."""
    rng = np.random.default_rng(seed)
    return ((rng.random(n) - 0.5) * 2 * scale).astype(np.float32)


__all__ = ["Q8_BLOCK", "Q8_BYTES", "Q4_BLOCK", "Q4_BYTES", "half_to_f32", "quant_row_q8",
           "quant_row_q4", "quant_matrix_q8", "quant_matrix_q4", "split_q8", "split_q4",
           "Device", "get_device", "GpuTensor", "max_rel_err", "rand_vec", "FlockError",
           "FLOCK_Q8_0", "FLOCK_Q4_0", "FLOCK_F32"]
