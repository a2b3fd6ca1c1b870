"""Op-level entry points: each individually validated kernel with host
inputs and outputs, the way the reference's kernel tests drive the WGSL
kernels one at a time (kernels/test_coop.ts, test_ops.ts, test_head.ts).

    matvec          kernels/q8_coop.wgsl:76 / q4_coop.wgsl:48
    rmsnorm         kernels/rmsnorm.wgsl:41
    rope            kernels/rope.wgsl:50
    swiglu, add     kernels/elementwise.wgsl:23, :31
    attention       kernels/attention.wgsl:58 (exact or split-K)
    attention_prefill  kernels/attention_prefill.wgsl:75
    embed           kernels/embed.wgsl:52
    argmax          kernels/argmax.wgsl:83, :112
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _abi
from .lib import Device, GpuTensor

_f = _abi._fp


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, np.float32)


def matvec(dev: Device, w: GpuTensor, x: np.ndarray, n_tokens: int = 1) -> np.ndarray:
    x = _f32(x)
    if x.size != n_tokens * w.cols:
        raise ValueError(f"x is {x.size} floats, want {n_tokens * w.cols}")
    out = np.empty(n_tokens * w.rows, np.float32)
    _abi.call("flock_op_matvec", dev.handle, w.handle, _abi.ptr(x, _f), n_tokens,
              _abi.ptr(out, _f))
    return out


def matvec_timed(dev: Device, w: GpuTensor, n_tokens: int = 1, iters: int = 50) -> float:
    """Mean ms per device-resident matvec launch (CUDA events)."""
    ms = ctypes.c_float()
    _abi.call("flock_op_matvec_timed", dev.handle, w.handle, n_tokens, iters, ctypes.byref(ms))
    return ms.value


def matvec_fast(dev: Device, w: GpuTensor, x: np.ndarray) -> np.ndarray:
    """One token's W x on the int8 tensor cores (FLOCK_MATVEC_FAST: x in three
    int8 digits per 32-block, reassociated; max relative error 1e-3)."""
    x = _f32(x)
    if x.size != w.cols:
        raise ValueError(f"x is {x.size} floats, want {w.cols}")
    out = np.empty(w.rows, np.float32)
    _abi.call("flock_op_matvec_fast", dev.handle, w.handle, _abi.ptr(x, _f), _abi.ptr(out, _f))
    return out


def matvec_fast_timed(dev: Device, w: GpuTensor, iters: int = 50, cold: bool = False) -> float:
    """Mean ms per device-resident FLOCK_MATVEC_FAST launch (CUDA events); cold:
    L2 evicted before each launch."""
    ms = ctypes.c_float()
    _abi.call("flock_op_matvec_fast_timed", dev.handle, w.handle, iters, int(cold),
              ctypes.byref(ms))
    return ms.value


def gemm(dev: Device, w: GpuTensor, x: np.ndarray, m: int) -> np.ndarray:
    """[m][cols] x W^T on the tensor cores (f16 operands, f32 accumulation)."""
    x = _f32(x)
    if x.size != m * w.cols:
        raise ValueError(f"x is {x.size} floats, want {m * w.cols}")
    out = np.empty(m * w.rows, np.float32)
    _abi.call("flock_op_gemm", dev.handle, w.handle, _abi.ptr(x, _f), m, _abi.ptr(out, _f))
    return out


def gemm_timed(dev: Device, w: GpuTensor, m: int, iters: int = 20) -> tuple:
    """(GEMM kernel ms, activation-conversion ms), means over device-resident
    calls timed with CUDA events around each kernel."""
    ms, img = ctypes.c_float(), ctypes.c_float()
    _abi.call("flock_op_gemm_timed", dev.handle, w.handle, m, iters, ctypes.byref(ms),
              ctypes.byref(img))
    return ms.value, img.value


def rmsnorm(dev: Device, x, g, n: int, n_vecs: int, eps: float) -> np.ndarray:
    x, g = _f32(x), _f32(g)
    out = np.empty(n * n_vecs, np.float32)
    _abi.call("flock_op_rmsnorm", dev.handle, _abi.ptr(x, _f), _abi.ptr(g, _f), n, n_vecs,
              ctypes.c_float(eps), _abi.ptr(out, _f))
    return out


def rope(dev: Device, x, n_tokens: int, n_heads: int, head_dim: int, pos0: int, inv_freq,
         pairing: str = "neox") -> np.ndarray:
    x, inv_freq = _f32(x), _f32(inv_freq)
    out = np.empty_like(x)
    _abi.call("flock_op_rope", dev.handle, _abi.ptr(x, _f), n_tokens, n_heads, head_dim, pos0,
              _abi.ptr(inv_freq, _f),
              _abi.FLOCK_ROPE_NEOX if pairing == "neox" else _abi.FLOCK_ROPE_NORM,
              _abi.ptr(out, _f))
    return out


def swiglu(dev: Device, gate, up) -> np.ndarray:
    gate, up = _f32(gate), _f32(up)
    out = np.empty_like(gate)
    _abi.call("flock_op_swiglu", dev.handle, _abi.ptr(gate, _f), _abi.ptr(up, _f), gate.size,
              _abi.ptr(out, _f))
    return out


def add(dev: Device, a, b) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    _abi.call("flock_op_add", dev.handle, _abi.ptr(a, _f), _abi.ptr(b, _f), a.size,
              _abi.ptr(out, _f))
    return out


def attention(dev: Device, q, k, v, n_heads: int, n_kv_heads: int, head_dim: int, n_keys: int,
              mode: str = "exact") -> np.ndarray:
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty(n_heads * head_dim, np.float32)
    _abi.call("flock_op_attention", dev.handle, _abi.ptr(q, _f), _abi.ptr(k, _f), _abi.ptr(v, _f),
              n_heads, n_kv_heads, head_dim, n_keys,
              _abi.FLOCK_ATTN_EXACT if mode == "exact" else _abi.FLOCK_ATTN_FAST,
              _abi.ptr(out, _f))
    return out


def attention_prefill(dev: Device, q, k, v, n_heads: int, n_kv_heads: int, head_dim: int,
                      n_queries: int, pos0: int) -> np.ndarray:
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty(n_queries * n_heads * head_dim, np.float32)
    _abi.call("flock_op_attention_prefill", dev.handle, _abi.ptr(q, _f), _abi.ptr(k, _f),
              _abi.ptr(v, _f), n_heads, n_kv_heads, head_dim, n_queries, pos0, _abi.ptr(out, _f))
    return out


def embed(dev: Device, table: GpuTensor, ids) -> np.ndarray:
    ids = np.ascontiguousarray(ids, np.int32)
    out = np.empty(ids.size * table.cols, np.float32)
    _abi.call("flock_op_embed", dev.handle, table.handle, _abi.ptr(ids, _abi._i32p), ids.size,
              _abi.ptr(out, _f))
    return out


def argmax(dev: Device, x) -> tuple[int, float]:
    x = _f32(x)
    idx = ctypes.c_int64()
    val = ctypes.c_float()
    _abi.call("flock_op_argmax", dev.handle, _abi.ptr(x, _f), x.size, ctypes.byref(idx),
              ctypes.byref(val))
    return idx.value, val.value
