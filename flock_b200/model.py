"""A whole Qwen3 forward pass on the GPU -- the kernels/model.ts surface.

    token ids -> embedding -> layers -> output_norm -> logits -> argmax -> id

``Model.create(dev, m, cfg, cut=...)`` holds the embedding, layers
0..cut-1, output_norm and the (tied) head, as model.ts:109 does; the
coordinator half is ``encode_partial`` / ``project_hidden``.  Decode steps
replay one captured CUDA graph; ``decode_device`` feeds each chosen token
back on the device with no host round trip.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _abi
from .layer import QWEN3_06B, TENSOR_NAMES, LayerConfig, upload_layer
from .lib import Device, GpuTensor


class Model:
    def __init__(self, dev: Device, handle, cfg: LayerConfig, vocab: int, n_layers: int,
                 keep: list):
        self.dev, self.handle, self.cfg, self.vocab, self.n_layers = dev, handle, cfg, vocab, n_layers
        self._keep = keep
        # the one-token step's arguments, made once (the per-token loop of a
        # caller feeding back each id converts no arrays)
        self._one = (ctypes.c_int32 * 1)()
        self._next = ctypes.c_int32()
        self._next_ref = ctypes.byref(self._next)
        self._step_fn = _abi.lib().flock_model_step

    @staticmethod
    def create(dev: Device, m, cfg: LayerConfig = QWEN3_06B, cut: int | None = None) -> "Model":
        """kernels/model.ts:109 -- `m` is a RealModel-like object (layers,
        embd, output_norm, optional untied output); only layers < cut are
        uploaded."""
        n_layers = len(m.layers)
        cut = n_layers if cut is None else cut
        if not (0 <= cut <= n_layers):
            raise ValueError(f"cut {cut} is not in 0..{n_layers}")
        if m.hidden != cfg.hidden:
            raise ValueError(f"model hidden {m.hidden} != config {cfg.hidden}")
        layer_ts = [upload_layer(dev, m.layers[i]) for i in range(cut)]
        embd = GpuTensor.from_packed(dev, m.embd["packed"], m.embd["rows"], m.embd["cols"])
        onorm = GpuTensor.from_f32(dev, m.output_norm)
        out = None
        if getattr(m, "output", None) is not None:
            out = GpuTensor.from_packed(dev, m.output["packed"], m.output["rows"], m.output["cols"])
        return Model.from_tensors(dev, cfg, m.vocab, n_layers, layer_ts, embd, onorm, out, cut)

    @staticmethod
    def from_tensors(dev: Device, cfg: LayerConfig, vocab: int, n_layers: int, layer_ts: list,
                     embd: GpuTensor | None, out_norm: GpuTensor | None,
                     output: GpuTensor | None = None, cut: int | None = None) -> "Model":
        cut = len(layer_ts) if cut is None else cut
        flat = []
        for t in layer_ts:
            for name in TENSOR_NAMES:
                if name not in t:
                    raise ValueError(f"layer is missing 1 tensor(s): {name}")
                flat.append(t[name].handle)
        arr = (ctypes.c_void_p * max(1, len(flat)))(*flat)
        h = ctypes.c_void_p()
        cfg_c = cfg.to_c()
        _abi.call("flock_model_create", dev.handle, ctypes.byref(cfg_c), vocab, len(layer_ts),
                  arr, embd.handle if embd else None, out_norm.handle if out_norm else None,
                  output.handle if output else None, cut, ctypes.byref(h))
        return Model(dev, h, cfg, vocab, n_layers, [layer_ts, embd, out_norm, output])

    @staticmethod
    def create_tp(dev: Device, m, cfg: LayerConfig, comm, rank: int, world: int) -> "Model":
        """One rank of the tensor-parallel model over an NCCL communicator
        (flock_model_create_tp): this rank's slices of every layer, the
        whole embedding and output_norm, its vocab rows of the head."""
        from .tensor_parallel import local_config, slice_head, slice_layer
        lcfg = local_config(cfg, world)
        layer_ts = [upload_layer(dev, slice_layer(w, cfg, rank, world)) for w in m.layers]
        embd = GpuTensor.from_packed(dev, m.embd["packed"], m.embd["rows"], m.embd["cols"])
        onorm = GpuTensor.from_f32(dev, m.output_norm)
        head = getattr(m, "output", None) or m.embd
        hs = slice_head(head, rank, world)
        out = GpuTensor.from_packed(dev, hs["packed"], hs["rows"], hs["cols"])
        flat = [t[name].handle for t in layer_ts for name in TENSOR_NAMES]
        arr = (ctypes.c_void_p * max(1, len(flat)))(*flat)
        h = ctypes.c_void_p()
        cfg_c = lcfg[rank].to_c()
        _abi.call("flock_model_create_tp", dev.handle, ctypes.byref(cfg_c), m.vocab,
                  len(layer_ts), arr, embd.handle, onorm.handle, out.handle,
                  comm.handle if hasattr(comm, "handle") else comm, ctypes.byref(h))
        # the model holds the communicator: it is freed after the model (and
        # its captured graph with NCCL calls)
        return Model(dev, h, lcfg[rank], m.vocab, len(m.layers),
                     [layer_ts, embd, onorm, out, comm])

    def free(self) -> None:
        if self.handle:
            _abi.lib().flock_model_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    @staticmethod
    def _ids(ids) -> np.ndarray:
        return np.ascontiguousarray(np.atleast_1d(ids), np.int32)

    # -------------------------------------------------------------- decode
    def step(self, ids) -> int:
        """kernels/model.ts:387 -- feed ids, return the greedy next id."""
        if (isinstance(ids, (list, tuple)) and len(ids) == 1 and
                isinstance(ids[0], (int, np.integer)) and -2**31 <= int(ids[0]) < 2**31):
            self._one[0] = int(ids[0])
            _abi.check(self._step_fn(self.handle, self._one, 1, self._next_ref))
            return self._next.value
        ids = self._ids(ids)
        out = ctypes.c_int32()
        _abi.call("flock_model_step", self.handle, _abi.ptr(ids, _abi._i32p), ids.size,
                  ctypes.byref(out))
        return out.value

    def logits(self, ids) -> np.ndarray:
        """kernels/model.ts:400"""
        ids = self._ids(ids)
        out = np.empty(self.vocab, np.float32)
        _abi.call("flock_model_logits", self.handle, _abi.ptr(ids, _abi._i32p), ids.size,
                  _abi.ptr(out, _abi._fp))
        return out

    def hidden_state(self, ids) -> np.ndarray:
        """kernels/model.ts:409 -- last position, before output_norm."""
        ids = self._ids(ids)
        out = np.empty(self.cfg.hidden, np.float32)
        _abi.call("flock_model_hidden_state", self.handle, _abi.ptr(ids, _abi._i32p), ids.size,
                  _abi.ptr(out, _abi._fp))
        return out

    def normed_state(self, ids) -> np.ndarray:
        """kernels/model.ts:491 -- last position after output_norm."""
        ids = self._ids(ids)
        out = np.empty(self.cfg.hidden, np.float32)
        _abi.call("flock_model_normed_state", self.handle, _abi.ptr(ids, _abi._i32p), ids.size,
                  _abi.ptr(out, _abi._fp))
        return out

    def embed(self, ids) -> np.ndarray:
        """kernels/model.ts:546"""
        ids = self._ids(ids)
        out = np.empty(ids.size * self.cfg.hidden, np.float32)
        _abi.call("flock_model_embed", self.handle, _abi.ptr(ids, _abi._i32p), ids.size,
                  _abi.ptr(out, _abi._fp))
        return out

    def encode_partial(self, ids, offset: int | None = None) -> np.ndarray:
        """kernels/model.ts:437 -- every position's hidden after the held layers."""
        ids = self._ids(ids)
        out = np.empty(ids.size * self.cfg.hidden, np.float32)
        _abi.call("flock_model_encode_partial", self.handle, _abi.ptr(ids, _abi._i32p), ids.size,
                  -1 if offset is None else offset, _abi.ptr(out, _abi._fp))
        return out

    def project_hidden(self, flat: np.ndarray, seq: int) -> int:
        """kernels/model.ts:474 -- output_norm + head + argmax on the last row."""
        flat = np.ascontiguousarray(flat, np.float32)
        if flat.size < seq * self.cfg.hidden:
            raise ValueError(f"hidden state is {flat.size} floats, want {seq * self.cfg.hidden}")
        out = ctypes.c_int32()
        _abi.call("flock_model_project_hidden", self.handle, _abi.ptr(flat, _abi._fp), seq,
                  ctypes.byref(out))
        return out.value

    def generate(self, prompt, max_tokens: int, eos=()) -> list:
        """kernels/model.ts:572 -- greedy, one 4-byte readback per token."""
        prompt = self._ids(prompt)
        eos = np.ascontiguousarray(np.array(list(eos), np.int32))
        out = np.empty(max(1, max_tokens), np.int32)
        n = ctypes.c_int()
        _abi.call("flock_model_generate", self.handle, _abi.ptr(prompt, _abi._i32p), prompt.size,
                  max_tokens, _abi.ptr(eos, _abi._i32p) if eos.size else None, eos.size,
                  _abi.ptr(out, _abi._i32p), ctypes.byref(n))
        return out[: n.value].tolist()

    def decode_device(self, n_steps: int) -> np.ndarray:
        """Greedy decode with the chosen id fed back on the device."""
        out = np.empty(max(1, n_steps), np.int32)
        _abi.call("flock_model_decode_device", self.handle, n_steps, _abi.ptr(out, _abi._i32p))
        return out[:n_steps]

    def steps_amortized(self, ids) -> int:
        """kernels/model.ts:510 -- K decode steps behind one readback."""
        ids = self._ids(ids)
        for i in ids:
            tok = self.step([int(i)])
        return tok

    # --------------------------------------------------------------- state
    def reset(self) -> None:
        _abi.call("flock_model_reset", self.handle)

    def rewind(self, n_keys: int) -> None:
        _abi.call("flock_model_rewind", self.handle, n_keys)

    @property
    def pos(self) -> int:
        n = ctypes.c_int()
        _abi.call("flock_model_pos", self.handle, ctypes.byref(n))
        return n.value

    @property
    def held(self) -> int:
        n = ctypes.c_int()
        _abi.call("flock_model_held", self.handle, ctypes.byref(n))
        return n.value

    _MODES = {"kernels": _abi.FLOCK_DECODE_KERNELS, "persistent": _abi.FLOCK_DECODE_PERSISTENT,
              "eager": _abi.FLOCK_DECODE_EAGER, "stream": _abi.FLOCK_DECODE_STREAM}

    @property
    def decode_mode(self) -> str:
        """"kernels" (the captured kernel graph), "persistent" (one cooperative
        kernel per token), "stream" (one cooperative kernel per token with the
        weights streamed through shared-memory rings) or "eager" (the kernels
        launched from the host)."""
        n = ctypes.c_int()
        _abi.call("flock_model_get_decode_mode", self.handle, ctypes.byref(n))
        return {v: k for k, v in self._MODES.items()}[n.value]

    @decode_mode.setter
    def decode_mode(self, mode: str) -> None:
        if mode not in self._MODES:
            raise ValueError(f"decode mode {mode!r} is not one of {sorted(self._MODES)}")
        _abi.call("flock_model_set_decode_mode", self.handle, self._MODES[mode])

    @property
    def tp_exchange(self) -> str:
        """Tensor-parallel decode exchange: "peer" (NVLink peer memory) or "nccl"."""
        n = ctypes.c_int()
        _abi.call("flock_model_get_tp_exchange", self.handle, ctypes.byref(n))
        return "peer" if n.value == _abi.FLOCK_TP_PEER else "nccl"

    @tp_exchange.setter
    def tp_exchange(self, mode: str) -> None:
        if mode not in ("peer", "nccl"):
            raise ValueError(f"tp exchange {mode!r} is neither 'peer' nor 'nccl'")
        _abi.call("flock_model_set_tp_exchange", self.handle,
                  _abi.FLOCK_TP_PEER if mode == "peer" else _abi.FLOCK_TP_NCCL)

    def trace(self, enable: bool = True) -> None:
        """Record per-CTA phase timestamps in the persistent decode kernel."""
        _abi.call("flock_model_trace", self.handle, 1 if enable else 0)

    def read_trace(self) -> np.ndarray:
        """The last traced token's entries, [n_ctas, 10 + 10 * held] uint64 ns."""
        n, s = ctypes.c_int(), ctypes.c_int()
        rc = _abi.lib().flock_model_trace_read(self.handle, None, 0, ctypes.byref(n), ctypes.byref(s))
        if rc not in (0, _abi.FLOCK_E_LIMIT):
            _abi.check(rc)
        out = np.zeros((n.value, s.value), np.uint64)
        _abi.call("flock_model_trace_read", self.handle,
                  out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), out.size,
                  ctypes.byref(n), ctypes.byref(s))
        return out

    def set_token(self, token: int) -> None:
        """The id the next device-fed decode step consumes."""
        _abi.call("flock_model_set_token", self.handle, int(token))

    def current_token(self) -> int:
        """kernels/model.ts:541"""
        out = ctypes.c_int32()
        _abi.call("flock_model_current_token", self.handle, ctypes.byref(out))
        return out.value
