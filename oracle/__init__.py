"""CPU parity oracle for the flock hot path -- TEST INFRASTRUCTURE ONLY.

This package is the checker the CUDA product path is compared against.  Only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import it; nothing under ``flock_b200/`` does, and the
product path fails loudly instead of falling back to it.

Two restatements of the reference's strict-f32 CPU references live here:

* ``liboracle.so`` (``flock_oracle.c``): the fast C restatement, OpenMP over
  rows, used at every size and as the timed CPU baseline.
* ``jsref``: a literal line-by-line transliteration in JS number semantics
  (Python floats are IEEE f64 like JS numbers; ``fround`` = cast to f32), used
  on small cases to cross-check the C restatement.

Parity pin: the reference (TypeScript + WGSL) cannot execute here -- there is
no JS engine or WebGPU stack on this machine or the GPU box -- and its tests
draw inputs from unseeded ``Math.random``, so it ships no numeric golden
vectors.  The oracle is pinned on the reference tests' constructed
known-answer cases (tests/test_oracle_kat.py) and on agreement between the two
independent restatements above; numeric outputs of the reference itself are
unpinned.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_dp = ctypes.POINTER(ctypes.c_double)
_i64 = ctypes.c_int64
_int = ctypes.c_int
_dbl = ctypes.c_double


def build() -> str:
    """Compile liboracle.so from flock_oracle.c with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        sig = {
            "fo_set_fma_mode": (None, [_int]),
            "fo_get_fma_mode": (_int, []),
            "fo_set_threads": (None, [_int]),
            "fo_max_threads": (_int, []),
            "fo_half_to_f32": (_dbl, [ctypes.c_uint16]),
            "fo_f32to16": (ctypes.c_uint16, [_dbl]),
            "fo_f16to32": (_dbl, [ctypes.c_uint16]),
            "fo_quant_row_q8": (None, [_f32p, _i64, _u8p]),
            "fo_quant_row_q4": (None, [_f32p, _i64, _u8p]),
            "fo_quant_matrix_q8": (None, [_f32p, _i64, _i64, _u8p]),
            "fo_quant_matrix_q4": (None, [_f32p, _i64, _i64, _u8p]),
            "fo_split_q8": (None, [_u8p, _i64, _i64, _u8p, _u8p]),
            "fo_split_q4": (None, [_u8p, _i64, _i64, _u8p, _u8p]),
            "fo_matmul_q8": (None, [_u8p, _f32p, _i64, _i64, _int, _f32p]),
            "fo_matmul_q4": (None, [_u8p, _f32p, _i64, _i64, _int, _f32p]),
            "fo_matmul_q8_batched": (None, [_u8p, _f32p, _i64, _i64, _int, _int, _f32p]),
            "fo_rmsnorm": (None, [_f32p, _f32p, _int, _int, _dbl, _int, _f32p]),
            "fo_rope_inv_freq": (None, [_int, _dbl, _f32p]),
            "fo_rope": (None, [_f32p, _int, _int, _int, _int, _f32p, _int, _f32p]),
            "fo_swiglu": (None, [_f32p, _f32p, _i64, _f32p]),
            "fo_add": (None, [_f32p, _f32p, _i64, _f32p]),
            "fo_attn": (None, [_f32p, _f32p, _f32p, _int, _int, _int, _int, _f32p]),
            "fo_embed": (None, [_u8p, _i32p, _int, _int, _f32p]),
            "fo_argmax": (_i64, [_f32p, _i64]),
            "fo_attn_prefill": (None, [_f32p, _f32p, _f32p, _int, _int, _int, _int, _int, _int,
                                       _int, _f32p]),
            "fo_cache_new": (ctypes.c_void_p, [_int, _int]),
            "fo_cache_free": (None, [ctypes.c_void_p]),
            "fo_cache_reset": (None, [ctypes.c_void_p]),
            "fo_cache_len": (_int, [ctypes.c_void_p]),
            "fo_cache_k": (_f32p, [ctypes.c_void_p]),
            "fo_cache_v": (_f32p, [ctypes.c_void_p]),
            "fo_cache_fill": (_int, [ctypes.c_void_p, _f32p, _f32p, _int]),
            "fo_cache_set_bf16": (None, [ctypes.c_void_p, _int]),
            "fo_bf16_round": (ctypes.c_float, [ctypes.c_float]),
            "fo_cache_set_fp8": (None, [ctypes.c_void_p, _int]),
            "fo_fp8_round": (ctypes.c_float, [ctypes.c_float]),
            "fo_layer_forward": (_int, [_f32p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                        _f32p]),
            "fo_layer_prefill": (_int, [_f32p, _int, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p, _f32p]),
            "fo_layer_prefill_tp": (_int, [_f32p, _int, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_void_p, _int, _f32p]),
            "fo_head": (_i64, [_f32p, _f32p, _u8p, _i64, _int, _dbl, _f32p, _f32p]),
            "fo_shard_ranges": (_int, [_i64, _int, _i64, _i64p, _i64p]),
            "fo_slice_rows": (None, [_u8p, _u8p, _i64, _i64, _i64, _i64, _u8p, _u8p]),
            "fo_slice_cols": (_int, [_u8p, _u8p, _i64, _i64, _i64, _i64, _u8p, _u8p]),
            "fo_slice_packed_cols": (_int, [_u8p, _i64, _i64, _i64, _i64, _u8p]),
            "fo_shard_matvec": (None, [_u8p, _f32p, _i64, _i64, _int, _f32p]),
            "fo_shard_reduce": (None, [_f32p, _int, _i64, _f32p]),
            "fo_sharded_col_matvec": (_int, [_u8p, _f32p, _i64, _i64, _int, _int, _f32p]),
            "fo_sharded_row_matvec": (_int, [_u8p, _f32p, _i64, _i64, _int, _int, _f32p]),
            "fo_reduce_shard_argmax": (_i64, [_f32p, _i64p, _i64p, _int]),
            "fo_mem_shard_plan": (_int, [_i64, _i64, _dbl, _dbl, _int, _int, _dbl, _dp, _dp,
                                         _i64p, _i32p]),
            "fo_dequant_q8": (None, [_u8p, _i64, _i64, _f32p]),
            "fo_requant_with_noise": (None, [_u8p, _i64, _i64, _u32p, _u8p]),
            "fo_wire_pack": (_i64, [_f32p, _i64, ctypes.c_uint32, ctypes.c_uint32,
                                    ctypes.c_uint32, _int, _int, _u8p]),
            "fo_wire_unpack": (_int, [_u8p, _i64, _f32p, _u32p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray, ty):
    return a.ctypes.data_as(ty)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint8)


# ------------------------------------------------------------------ settings

def set_fma_mode(ieee: bool) -> None:
    """False = literal JS fma32 (f64 add then f32 round); True = IEEE fmaf."""
    lib().fo_set_fma_mode(1 if ieee else 0)


def set_threads(n: int) -> None:
    lib().fo_set_threads(int(n))


def max_threads() -> int:
    return int(lib().fo_max_threads())


# ------------------------------------------------------------------- codecs

def half_to_f32(h: int) -> float:
    return lib().fo_half_to_f32(h)


def f32to16(v: float) -> int:
    return int(lib().fo_f32to16(float(v)))


def f16to32(h: int) -> float:
    return lib().fo_f16to32(h)


# --------------------------------------------------------------- quantizers

def quant_matrix_q8(w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    w = _f32(w)
    out = np.empty(rows * (cols // 32) * 34, np.uint8)
    lib().fo_quant_matrix_q8(_p(w, _f32p), rows, cols, _p(out, _u8p))
    return out


def quant_matrix_q4(w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    w = _f32(w)
    out = np.empty(rows * (cols // 32) * 18, np.uint8)
    lib().fo_quant_matrix_q4(_p(w, _f32p), rows, cols, _p(out, _u8p))
    return out


def split_q8(packed: np.ndarray, rows: int, cols: int):
    packed = _u8(packed)
    qs = np.empty(rows * cols, np.uint8)
    sc = np.empty(rows * (cols // 32) * 2, np.uint8)
    lib().fo_split_q8(_p(packed, _u8p), rows, cols, _p(qs, _u8p), _p(sc, _u8p))
    return qs, sc


def split_q4(packed: np.ndarray, rows: int, cols: int):
    packed = _u8(packed)
    qs = np.empty(rows * (cols // 32) * 16, np.uint8)
    sc = np.empty(rows * (cols // 32) * 2, np.uint8)
    lib().fo_split_q4(_p(packed, _u8p), rows, cols, _p(qs, _u8p), _p(sc, _u8p))
    return qs, sc


# ------------------------------------------------------------------- matvec

COOP = 64  # layer_ref.ts COOP_LANES / q8_coop.wgsl LANES
SERIAL = 0


def matmul_q8(packed, x, rows, cols, lanes=COOP) -> np.ndarray:
    packed, x = _u8(packed), _f32(x)
    out = np.empty(rows, np.float32)
    lib().fo_matmul_q8(_p(packed, _u8p), _p(x, _f32p), rows, cols, lanes, _p(out, _f32p))
    return out


def matmul_q4(packed, x, rows, cols, lanes=COOP) -> np.ndarray:
    packed, x = _u8(packed), _f32(x)
    out = np.empty(rows, np.float32)
    lib().fo_matmul_q4(_p(packed, _u8p), _p(x, _f32p), rows, cols, lanes, _p(out, _f32p))
    return out


def matmul_q8_batched(packed, x, rows, cols, n_tokens, lanes=COOP) -> np.ndarray:
    packed, x = _u8(packed), _f32(x)
    out = np.empty(n_tokens * rows, np.float32)
    lib().fo_matmul_q8_batched(_p(packed, _u8p), _p(x, _f32p), rows, cols, n_tokens, lanes,
                               _p(out, _f32p))
    return out


# ---------------------------------------------------------------------- ops

EPS = 9.999999974752427e-7  # layer.ts:125 QWEN3_06B.eps (f32 of 1e-6)


def rmsnorm(x, g, n, n_vecs, eps=EPS, wg=128) -> np.ndarray:
    x, g = _f32(x), _f32(g)
    out = np.empty(n * n_vecs, np.float32)
    lib().fo_rmsnorm(_p(x, _f32p), _p(g, _f32p), n, n_vecs, eps, wg, _p(out, _f32p))
    return out


def rope_inv_freq(head_dim=128, base=1e6) -> np.ndarray:
    out = np.empty(head_dim // 2, np.float32)
    lib().fo_rope_inv_freq(head_dim, base, _p(out, _f32p))
    return out


def rope(x, n_tokens, n_heads, head_dim, pos0, inv_freq, neox=True) -> np.ndarray:
    x, inv_freq = _f32(x), _f32(inv_freq)
    out = np.empty_like(x)
    lib().fo_rope(_p(x, _f32p), n_tokens, n_heads, head_dim, pos0, _p(inv_freq, _f32p),
                  1 if neox else 0, _p(out, _f32p))
    return out


def swiglu(gate, up) -> np.ndarray:
    gate, up = _f32(gate), _f32(up)
    out = np.empty_like(gate)
    lib().fo_swiglu(_p(gate, _f32p), _p(up, _f32p), gate.size, _p(out, _f32p))
    return out


def add(a, b) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    lib().fo_add(_p(a, _f32p), _p(b, _f32p), a.size, _p(out, _f32p))
    return out


def attn(q, k, v, n_heads, n_kv_heads, head_dim, n_keys) -> np.ndarray:
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty(n_heads * head_dim, np.float32)
    lib().fo_attn(_p(q, _f32p), _p(k, _f32p), _p(v, _f32p), n_heads, n_kv_heads, head_dim,
                  n_keys, _p(out, _f32p))
    return out


def embed(packed, ids, cols) -> np.ndarray:
    packed = _u8(packed)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    out = np.empty(ids.size * cols, np.float32)
    lib().fo_embed(_p(packed, _u8p), _p(ids, _i32p), ids.size, cols, _p(out, _f32p))
    return out


def argmax(x) -> int:
    x = _f32(x)
    return int(lib().fo_argmax(_p(x, _f32p), x.size))


def attn_prefill(q, k, v, n_heads, n_kv_heads, head_dim, n_queries, pos0, tile=64,
                 wg=128) -> np.ndarray:
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty(n_queries * n_heads * head_dim, np.float32)
    lib().fo_attn_prefill(_p(q, _f32p), _p(k, _f32p), _p(v, _f32p), n_heads, n_kv_heads,
                          head_dim, n_queries, pos0, tile, wg, _p(out, _f32p))
    return out


# -------------------------------------------------------------------- layer

class _Cfg(ctypes.Structure):
    _fields_ = [("hidden", _int), ("n_heads", _int), ("n_kv_heads", _int), ("head_dim", _int),
                ("ffn", _int), ("eps", _dbl), ("rope_base", _dbl), ("neox", _int)]


class _W(ctypes.Structure):
    _fields_ = [(n, _u8p) for n in ("q", "k", "v", "o", "gate", "up", "down")] + \
               [(n, _f32p) for n in ("attn_norm", "q_norm", "k_norm", "ffn_norm")]


Q8_NAMES = {"attn_q.weight": "q", "attn_k.weight": "k", "attn_v.weight": "v",
            "attn_output.weight": "o", "ffn_gate.weight": "gate", "ffn_up.weight": "up",
            "ffn_down.weight": "down"}
F32_NAMES = {"attn_norm.weight": "attn_norm", "attn_q_norm.weight": "q_norm",
             "attn_k_norm.weight": "k_norm", "ffn_norm.weight": "ffn_norm"}


class RefLayer:
    """layer_ref.ts layerForwardRef / layerPrefillRef with a RefCache (:24).
    tp > 1: o_proj and down become tp-shard input-split matvecs
    (shard_ref.ts:353), the arithmetic of a tensor-parallel layer.
    kv="bf16": every appended key/value is rounded to bf16 (nearest even), the
    cache a FLOCK_KV_BF16 layer keeps; kv="fp8": to e4m3 (fo_fp8_round, the
    FLOCK_KV_FP8 cache); attention then reads the rounded values."""

    def __init__(self, weights: dict, cfg: dict, max_keys: int = 4096, tp: int = 1,
                 kv: str = "f32"):
        if kv not in ("f32", "bf16", "fp8"):
            raise ValueError(f"kv must be 'f32', 'bf16' or 'fp8', not {kv!r}")
        self.tp = int(tp)
        self._keep = {}
        w = _W()
        for name, field in Q8_NAMES.items():
            a = _u8(weights[name]["packed"] if isinstance(weights[name], dict) else weights[name])
            self._keep[name] = a
            setattr(w, field, _p(a, _u8p))
        for name, field in F32_NAMES.items():
            a = _f32(weights[name])
            self._keep[name] = a
            setattr(w, field, _p(a, _f32p))
        self._w = w
        self.cfg = cfg
        self._c = _Cfg(cfg["hidden"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                       cfg["ffn"], cfg.get("eps", EPS), cfg.get("rope_base", 1e6),
                       1 if cfg.get("rope_pairing", "neox") == "neox" else 0)
        self.kvw = cfg["n_kv_heads"] * cfg["head_dim"]
        self._cache = lib().fo_cache_new(max_keys, self.kvw)
        lib().fo_cache_set_bf16(self._cache, 1 if kv == "bf16" else 0)
        if kv == "fp8":
            lib().fo_cache_set_fp8(self._cache, 1)

    def __del__(self):
        try:
            lib().fo_cache_free(self._cache)
        except Exception:
            pass

    @property
    def n_keys(self) -> int:
        return int(lib().fo_cache_len(self._cache))

    def reset(self) -> None:
        lib().fo_cache_reset(self._cache)

    def fill_cache(self, k: np.ndarray, v: np.ndarray) -> None:
        k, v = _f32(k), _f32(v)
        n = k.size // self.kvw
        if lib().fo_cache_fill(self._cache, _p(k, _f32p), _p(v, _f32p), n) != 0:
            raise ValueError("reference cache overflow")

    def cache(self):
        n = self.n_keys
        k = np.ctypeslib.as_array(lib().fo_cache_k(self._cache), shape=(max(n, 1) * self.kvw,))
        v = np.ctypeslib.as_array(lib().fo_cache_v(self._cache), shape=(max(n, 1) * self.kvw,))
        return k[: n * self.kvw].copy(), v[: n * self.kvw].copy()

    def forward(self, hidden: np.ndarray, n_tokens: int = 1) -> np.ndarray:
        hidden = _f32(hidden)
        out = np.empty(n_tokens * self.cfg["hidden"], np.float32)
        rc = lib().fo_layer_prefill_tp(_p(hidden, _f32p), n_tokens, ctypes.byref(self._w),
                                       ctypes.byref(self._c), self._cache, self.tp,
                                       _p(out, _f32p))
        if rc == -2:
            raise ValueError(f"cannot cut this layer into {self.tp} shards")
        if rc != 0:
            raise ValueError("reference cache overflow")
        return out


def head(last_row, out_norm, embd_packed, vocab, hidden, eps=EPS):
    """model.ts:307 encodeHead -> (token id, normed, logits)."""
    last_row, out_norm, embd_packed = _f32(last_row), _f32(out_norm), _u8(embd_packed)
    normed = np.empty(hidden, np.float32)
    logits = np.empty(vocab, np.float32)
    tid = lib().fo_head(_p(last_row, _f32p), _p(out_norm, _f32p), _p(embd_packed, _u8p), vocab,
                        hidden, eps, _p(normed, _f32p), _p(logits, _f32p))
    return int(tid), normed, logits


# ------------------------------------------------------------------- shards

def shard_ranges(total: int, n: int, align: int = 1):
    st = np.empty(max(n, 1), np.int64)
    ct = np.empty(max(n, 1), np.int64)
    rc = lib().fo_shard_ranges(total, n, align, _p(st, _i64p), _p(ct, _i64p))
    if rc:
        raise ValueError(f"shard_ranges rc={rc}")
    return [(int(s), int(c)) for s, c in zip(st[:n], ct[:n])]


def shard_reduce(parts: np.ndarray) -> np.ndarray:
    parts = _f32(parts)
    n_shards, n = parts.shape
    out = np.empty(n, np.float32)
    lib().fo_shard_reduce(_p(parts, _f32p), n_shards, n, _p(out, _f32p))
    return out


def sharded_col_matvec(packed, x, rows, cols, n_shards, lanes=COOP):
    packed, x = _u8(packed), _f32(x)
    out = np.empty(rows, np.float32)
    rc = lib().fo_sharded_col_matvec(_p(packed, _u8p), _p(x, _f32p), rows, cols, n_shards, lanes,
                                     _p(out, _f32p))
    if rc:
        raise ValueError(f"sharded_col_matvec rc={rc}")
    return out


def sharded_row_matvec(packed, x, rows, cols, n_shards, lanes=COOP):
    packed, x = _u8(packed), _f32(x)
    out = np.empty(rows, np.float32)
    rc = lib().fo_sharded_row_matvec(_p(packed, _u8p), _p(x, _f32p), rows, cols, n_shards, lanes,
                                     _p(out, _f32p))
    if rc:
        raise ValueError(f"sharded_row_matvec rc={rc}")
    return out


def reduce_shard_argmax(values, index, row_offset) -> int:
    values = _f32(values)
    index = np.ascontiguousarray(index, np.int64)
    row_offset = np.ascontiguousarray(row_offset, np.int64)
    return int(lib().fo_reduce_shard_argmax(_p(values, _f32p), _p(index, _i64p),
                                            _p(row_offset, _i64p), values.size))


def mem_shard_plan(rows, cols, n, direction="row", limit=128 * 1024 * 1024,
                   bytes_per_weight=1.0, scale_bytes_per_block=2.0):
    mb, un = ctypes.c_double(), ctypes.c_double()
    mn = ctypes.c_int64()
    fits = ctypes.c_int32()
    rc = lib().fo_mem_shard_plan(rows, cols, bytes_per_weight, scale_bytes_per_block, n,
                                 0 if direction == "row" else 1, float(limit), ctypes.byref(mb),
                                 ctypes.byref(un), ctypes.byref(mn), ctypes.byref(fits))
    if rc:
        raise ValueError(f"mem_shard_plan rc={rc}")
    return {"max_binding_bytes": mb.value, "unsharded_max_binding_bytes": un.value,
            "min_shards_for_limit": (mn.value or None), "fits": bool(fits.value)}


# ------------------------------------------------------------------ dequant

def dequant_q8(packed, rows, cols) -> np.ndarray:
    packed = _u8(packed)
    out = np.empty(rows * cols, np.float32)
    lib().fo_dequant_q8(_p(packed, _u8p), rows, cols, _p(out, _f32p))
    return out


def requant_with_noise(packed, rows, cols, state: int = 1):
    packed = _u8(packed)
    out = np.empty_like(packed)
    st = ctypes.c_uint32(state or 1)
    lib().fo_requant_with_noise(_p(packed, _u8p), rows, cols, ctypes.byref(st), _p(out, _u8p))
    return out, st.value


# --------------------------------------------------------------------- wire

def wire_pack(floats, seq, hidden, offset=0, reset=False, replay=False) -> bytes:
    floats = _f32(floats)
    out = np.empty(20 + floats.size * 2, np.uint8)
    n = lib().fo_wire_pack(_p(floats, _f32p), floats.size, seq, hidden, offset, int(reset),
                           int(replay), _p(out, _u8p))
    return out[:n].tobytes()


def wire_unpack(buf: bytes):
    a = np.frombuffer(buf, np.uint8).copy()
    out = np.empty((a.size - 20) // 2, np.float32)
    meta = np.empty(5, np.uint32)
    if lib().fo_wire_unpack(_p(a, _u8p), a.size, _p(out, _f32p), _p(meta, _u32p)) != 0:
        raise ValueError("not a flock frame")
    return out, {"seq": int(meta[0]), "hidden": int(meta[1]), "offset": int(meta[2]),
                 "reset": bool(meta[3]), "replay": bool(meta[4])}
