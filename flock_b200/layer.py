"""One Qwen3 decoder layer on the GPU -- the kernels/layer.ts surface.

    h1 = h + attn_output @ attention(rope(q_norm(Wq n(h))), rope(k_norm(Wk n(h))), Wv n(h))
    h2 = h1 + ffn_down @ (silu(ffn_gate @ n(h1)) * (ffn_up @ n(h1)))

``Layer.create`` takes packed GGUF Q8_0 bytes (repacked on the host, as
layer.ts:289 does); ``Layer.from_buffers`` takes tensors already on the GPU
(layer.ts:228).  ``encode`` / ``encode_prefill`` leave the output on the
device for the next layer; ``read_output`` fetches it (layer.ts:801).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace

import numpy as np

from . import _abi
from .lib import Device, GpuTensor

TENSOR_NAMES = ("attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
                "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight", "attn_norm.weight",
                "attn_q_norm.weight", "attn_k_norm.weight", "ffn_norm.weight")
Q8_NAMES = TENSOR_NAMES[:7]
F32_NAMES = TENSOR_NAMES[7:]


@dataclass(frozen=True)
class LayerConfig:
    """kernels/layer.ts:87 LayerConfig (+ which decode attention to run)."""
    hidden: int = 1024
    n_heads: int = 16
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 3072
    eps: float = 9.999999974752427e-7
    rope_base: float = 1e6
    max_keys: int = 2048
    max_prefill: int = 512
    rope_pairing: str = "neox"
    # "exact": attnRef's order (ops_ref.ts:135), bit-comparable;
    # "fast": split-K flash-decode, uncapped keys, 1e-5 relative tolerance.
    attention: str = "exact"
    # multi-token steps: "exact" (the reference's f32 order, bit-comparable) or
    # "tensor" (tcgen05 tensor cores, f16 operands, 1e-2 relative tolerance)
    prefill: str = "exact"
    # KV cache element type: "f32" (the reference's), "bf16" (half the bytes
    # per key) or "fp8" (e4m3, a quarter; magnitudes past 448 saturate);
    # appends round to nearest even; both need attention="fast" and
    # prefill="tensor"
    kv: str = "f32"
    # one-token matvecs: "exact" (cpuMatmulQ8F32(coop(64))'s order, bit-identical)
    # or "fast" (the decode LM head on the int8 tensor cores, reassociated,
    # 1e-3 relative tolerance)
    matvec: str = "exact"

    def to_c(self) -> _abi.LayerConfigC:
        if self.kv not in ("f32", "bf16", "fp8"):
            raise ValueError(f"kv must be 'f32', 'bf16' or 'fp8', not {self.kv!r}")
        if self.matvec not in ("exact", "fast"):
            raise ValueError(f"matvec must be 'exact' or 'fast', not {self.matvec!r}")
        return _abi.LayerConfigC(
            self.hidden, self.n_heads, self.n_kv_heads, self.head_dim, self.ffn, self.eps,
            self.rope_base, self.max_keys, self.max_prefill,
            _abi.FLOCK_ROPE_NEOX if self.rope_pairing == "neox" else _abi.FLOCK_ROPE_NORM,
            _abi.FLOCK_ATTN_EXACT if self.attention == "exact" else _abi.FLOCK_ATTN_FAST,
            _abi.FLOCK_PREFILL_TENSOR if self.prefill == "tensor" else _abi.FLOCK_PREFILL_EXACT,
            {"bf16": _abi.FLOCK_KV_BF16, "fp8": _abi.FLOCK_KV_FP8}.get(self.kv, _abi.FLOCK_KV_F32),
            _abi.FLOCK_MATVEC_FAST if self.matvec == "fast" else _abi.FLOCK_MATVEC_EXACT)

    def with_(self, **kw) -> "LayerConfig":
        return replace(self, **kw)


# kernels/layer.ts:119 QWEN3_06B
QWEN3_06B = LayerConfig()


def upload_layer(dev: Device, weights: dict) -> dict:
    """Packed LayerWeights (layer.ts:59) -> GpuTensors keyed by GGUF suffix."""
    out = {}
    for name, t in weights.items():
        if isinstance(t, dict):
            out[name] = GpuTensor.from_packed(dev, t["packed"], t["rows"], t["cols"])
        else:
            out[name] = GpuTensor.from_f32(dev, np.asarray(t, np.float32))
    return out


class Layer:
    def __init__(self, dev: Device, handle, cfg: LayerConfig, tensors: dict):
        self.dev, self.handle, self.cfg = dev, handle, cfg
        self._tensors = tensors  # the layer borrows them; keep them alive

    # ----------------------------------------------------------- construct
    @staticmethod
    def from_buffers(dev: Device, tensors: dict, cfg: LayerConfig = QWEN3_06B) -> "Layer":
        """kernels/layer.ts:228 -- missing tensors raise, naming them."""
        names = list(tensors.keys())
        c_names = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
        c_ts = (ctypes.c_void_p * len(names))(*[tensors[n].handle for n in names])
        h = ctypes.c_void_p()
        cfg_c = cfg.to_c()
        _abi.call("flock_layer_create", dev.handle, ctypes.byref(cfg_c), len(names), c_names,
                  c_ts, ctypes.byref(h))
        return Layer(dev, h, cfg, dict(tensors))

    @staticmethod
    def create(dev: Device, weights: dict, cfg: LayerConfig = QWEN3_06B) -> "Layer":
        """kernels/layer.ts:289 -- packed Q8_0 bytes repacked at upload."""
        return Layer.from_buffers(dev, upload_layer(dev, weights), cfg)

    def free(self) -> None:
        if self.handle:
            _abi.lib().flock_layer_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    # ------------------------------------------------------------- running
    def encode(self, hidden: np.ndarray | None = None) -> None:
        """kernels/layer.ts:571 -- one decode step, output stays on the GPU."""
        self.encode_prefill(1, hidden)

    def encode_prefill(self, n_tokens: int, hidden: np.ndarray | None = None) -> None:
        """kernels/layer.ts:685 -- n_tokens positions from nKeys."""
        p = None
        if hidden is not None:
            hidden = np.ascontiguousarray(hidden, np.float32)
            if hidden.size != n_tokens * self.cfg.hidden:
                raise ValueError(f"hidden is {hidden.size}, expected {n_tokens * self.cfg.hidden}")
            p = _abi.ptr(hidden, _abi._fp)
        _abi.call("flock_layer_encode", self.handle, p, n_tokens)

    def forward(self, hidden: np.ndarray) -> np.ndarray:
        """kernels/layer.ts:554 -- encode + readOutput."""
        n = np.asarray(hidden).size // self.cfg.hidden
        self.encode_prefill(n, hidden)
        return self.read_output(n)

    def read_output(self, n_tokens: int = 1) -> np.ndarray:
        out = np.empty(n_tokens * self.cfg.hidden, np.float32)
        _abi.call("flock_layer_read_output", self.handle, n_tokens, _abi.ptr(out, _abi._fp))
        return out

    def reset(self) -> None:
        _abi.call("flock_layer_reset", self.handle)

    def rewind(self, n_keys: int) -> None:
        _abi.call("flock_layer_rewind", self.handle, n_keys)

    @property
    def n_keys(self) -> int:
        n = ctypes.c_int()
        _abi.call("flock_layer_n_keys", self.handle, ctypes.byref(n))
        return n.value

    def cache_buffers(self) -> tuple[np.ndarray, np.ndarray]:
        """kernels/layer.ts:792 -- the KV cache [nKeys][nKV][hd], read back."""
        n = self.n_keys * self.cfg.n_kv_heads * self.cfg.head_dim
        k = np.empty(max(n, 1), np.float32)
        v = np.empty(max(n, 1), np.float32)
        _abi.call("flock_layer_read_cache", self.handle, _abi.ptr(k, _abi._fp),
                  _abi.ptr(v, _abi._fp))
        return k[:n], v[:n]

    def write_cache(self, k: np.ndarray, v: np.ndarray) -> None:
        """Append precomputed keys/values at the current position."""
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        n = k.size // (self.cfg.n_kv_heads * self.cfg.head_dim)
        _abi.call("flock_layer_write_cache", self.handle, _abi.ptr(k, _abi._fp),
                  _abi.ptr(v, _abi._fp), n)


def range_forward(layers: list, x: np.ndarray, seq: int, offset: int,
                  reset: bool = False) -> np.ndarray:
    """web/bird.html:544-620 runFrame: a held layer range over one frame."""
    x = np.ascontiguousarray(x, np.float32)
    hs = (ctypes.c_void_p * len(layers))(*[L.handle for L in layers])
    out = np.empty(seq * layers[0].cfg.hidden, np.float32)
    _abi.call("flock_range_forward", hs, len(layers), _abi.ptr(x, _abi._fp), seq, offset,
              1 if reset else 0, _abi.ptr(out, _abi._fp))
    return out
