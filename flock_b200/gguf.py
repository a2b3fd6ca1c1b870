"""GGUF model files: the directory, the byte planner and the streaming
loader of the C ABI (flock_gguf_*), and a Qwen3 model built straight from a
file -- web/js/gguf-dir.mjs readDirectory, server/gguf.mjs byteRanges,
web/js/gguf-stream.mjs streamTensorToGPU / loadLayersToGPU on B200.

GGUF shapes are [in, out]: a tensor's ``cols`` is shape[0] and ``rows`` the
product of the remaining dims.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _abi
from .layer import TENSOR_NAMES, LayerConfig
from .lib import Device, GpuTensor

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0 = 0, 1, 2, 8
STAGING = 4 << 20  # gguf-stream.mjs:45


@dataclass(frozen=True)
class TensorInfo:
    name: str
    dtype: int
    rows: int
    cols: int
    offset: int  # from the data start
    bytes: int


class GGUFFile:
    def __init__(self, path: str):
        h = ctypes.c_void_p()
        _abi.call("flock_gguf_open", str(path).encode(), ctypes.byref(h))
        self.handle, self.path = h, str(path)
        n, ds = ctypes.c_int64(), ctypes.c_int64()
        ver, nl = ctypes.c_int(), ctypes.c_int()
        _abi.call("flock_gguf_info", h, ctypes.byref(n), ctypes.byref(ds), ctypes.byref(ver),
                  ctypes.byref(nl))
        self.data_start, self.version = ds.value, ver.value
        self.n_layers = nl.value if nl.value >= 0 else None
        self.tensors: list[TensorInfo] = []
        name = ctypes.create_string_buffer(512)
        for i in range(n.value):
            dt, r, c, o, b = (ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64(),
                              ctypes.c_int64())
            _abi.call("flock_gguf_tensor_info", h, i, name, 512, ctypes.byref(dt), ctypes.byref(r),
                      ctypes.byref(c), ctypes.byref(o), ctypes.byref(b))
            self.tensors.append(TensorInfo(name.value.decode(), dt.value, r.value, c.value,
                                           o.value, b.value))
        self.by_name = {t.name: t for t in self.tensors}

    def close(self) -> None:
        if self.handle:
            _abi.lib().flock_gguf_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------ metadata
    def meta_int(self, key: str) -> int:
        v = ctypes.c_int64()
        _abi.call("flock_gguf_meta_int", self.handle, key.encode(), ctypes.byref(v))
        return v.value

    def meta_float(self, key: str) -> float:
        v = ctypes.c_double()
        _abi.call("flock_gguf_meta_f64", self.handle, key.encode(), ctypes.byref(v))
        return v.value

    def meta_str(self, key: str) -> str:
        b = ctypes.create_string_buffer(4096)
        _abi.call("flock_gguf_meta_str", self.handle, key.encode(), b, 4096)
        return b.value.decode()

    def layer_ranges(self, first: int, last: int, gap: int = 1 << 20) -> list[tuple[int, int]]:
        """server/gguf.mjs:78 byteRanges: absolute [start, end) ranges."""
        n = ctypes.c_int()
        rc = _abi.lib().flock_gguf_layer_ranges(self.handle, first, last, gap, None, None, 0,
                                                ctypes.byref(n))
        if rc not in (_abi.FLOCK_OK, _abi.FLOCK_E_LIMIT):
            _abi.check(rc)
        st = np.zeros(max(1, n.value), np.int64)
        en = np.zeros(max(1, n.value), np.int64)
        _abi.call("flock_gguf_layer_ranges", self.handle, first, last, gap,
                  _abi.ptr(st, _abi._i64p), _abi.ptr(en, _abi._i64p), st.size, ctypes.byref(n))
        return [(int(a), int(b)) for a, b in zip(st[:n.value], en[:n.value])]

    # -------------------------------------------------------------- tensors
    def split_host(self, name: str, chunk: int = STAGING) -> tuple[np.ndarray, np.ndarray]:
        """The incremental Q8_0/Q4_0 split into host planes (qs, scales)."""
        t = self.by_name[name]
        nb = t.rows * t.cols // 32
        qs = np.empty(nb * (32 if t.dtype == GGML_Q8_0 else 16), np.uint8)
        sc = np.empty(nb * 2, np.uint8)
        _abi.call("flock_gguf_split_host", self.handle, name.encode(), chunk,
                  _abi.ptr(qs, _abi._u8p), _abi.ptr(sc, _abi._u8p))
        return qs, sc

    def load_tensor(self, dev: Device, name: str, staging: int = STAGING) -> GpuTensor:
        """gguf-stream.mjs:281 streamTensorToGPU."""
        t = self.by_name.get(name)
        h = ctypes.c_void_p()
        _abi.call("flock_gguf_load_tensor", dev.handle, self.handle, name.encode(), staging,
                  ctypes.byref(h))
        if t.dtype in (GGML_F32, GGML_F16):
            return GpuTensor(dev, h, 1, t.rows * t.cols, _abi.FLOCK_F32)
        return GpuTensor(dev, h, t.rows, t.cols,
                         _abi.FLOCK_Q8_0 if t.dtype == GGML_Q8_0 else _abi.FLOCK_Q4_0)

    def load_layer(self, dev: Device, layer: int, staging: int = STAGING) -> dict:
        """gguf-stream.mjs:651 loadLayersToGPU for one layer: blk.<i>.* by suffix."""
        return {n: self.load_tensor(dev, f"blk.{layer}.{n}", staging) for n in TENSOR_NAMES}

    # ---------------------------------------------------------------- model
    def config(self, **kw) -> LayerConfig:
        """The layer shape from `<arch>.*` metadata (Qwen3 keys)."""
        arch = self.meta_str("general.architecture")

        def opt(key, default, f=self.meta_int):
            try:
                return f(f"{arch}.{key}")
            except _abi.FlockError:
                return default
        hidden = self.meta_int(f"{arch}.embedding_length")
        heads = self.meta_int(f"{arch}.attention.head_count")
        cfg = LayerConfig(
            hidden=hidden, n_heads=heads,
            n_kv_heads=opt("attention.head_count_kv", heads),
            head_dim=opt("attention.key_length", hidden // heads),
            ffn=self.meta_int(f"{arch}.feed_forward_length"),
            eps=opt("attention.layer_norm_rms_epsilon", 1e-6, self.meta_float),
            rope_base=opt("rope.freq_base", 1e6, self.meta_float))
        return cfg.with_(**kw) if kw else cfg

    @property
    def vocab(self) -> int:
        return self.by_name["token_embd.weight"].rows


def model_from_gguf(dev: Device, path: str, cfg: LayerConfig | None = None,
                    cut: int | None = None, staging: int = STAGING):
    """A Model whose weights stream from a GGUF file straight into device
    planes: layers 0..cut-1, token_embd, output_norm, and output (untied)."""
    from .model import Model
    g = GGUFFile(path)
    cfg = cfg or g.config()
    n = g.n_layers if g.n_layers is not None else 0
    cut = n if cut is None else cut
    layer_ts = [g.load_layer(dev, i, staging) for i in range(cut)]
    embd = g.load_tensor(dev, "token_embd.weight", staging)
    onorm = g.load_tensor(dev, "output_norm.weight", staging)
    out = g.load_tensor(dev, "output.weight", staging) if "output.weight" in g.by_name else None
    M = Model.from_tensors(dev, cfg, g.vocab, n, layer_ts, embd, onorm, out, cut)
    g.close()
    return M
