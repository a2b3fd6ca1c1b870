"""FLK1 frames (web/js/wire.mjs) through the C ABI: ``pack`` / ``unpack``
and ``range_forward_wire``, web/bird.html's runFrame for a held layer range
with the f16 payload converted on the device."""
from __future__ import annotations

import ctypes

import numpy as np

from . import _abi

FLAG_RESET, FLAG_REPLAY = 1, 2


def pack(x, seq: int, hidden: int, offset: int = 0, reset: bool = False,
         replay: bool = False) -> bytes:
    """wire.mjs:54 pack."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    out = np.empty(20 + 2 * x.size, np.uint8)
    n = ctypes.c_int64()
    flags = (FLAG_RESET if reset else 0) | (FLAG_REPLAY if replay else 0)
    _abi.call("flock_wire_pack", _abi.ptr(x, _abi._fp), x.size, seq, hidden, offset, flags,
              _abi.ptr(out, _abi._u8p), out.size, ctypes.byref(n))
    return out[:n.value].tobytes()


def unpack(frame: bytes) -> tuple[np.ndarray, dict]:
    """wire.mjs:79 unpack -> (f32 values, {seq, hidden, offset, reset, replay})."""
    b = np.frombuffer(frame, np.uint8).copy()
    out = np.empty(max(0, (b.size - 20) // 2), np.float32)
    meta = (ctypes.c_uint32 * 5)()
    _abi.call("flock_wire_unpack", _abi.ptr(b, _abi._u8p), b.size, _abi.ptr(out, _abi._fp),
              out.size, meta)
    return out, {"seq": meta[0], "hidden": meta[1], "offset": meta[2], "reset": bool(meta[3]),
                 "replay": bool(meta[4])}


def range_forward_wire(layers, frame: bytes) -> bytes:
    """bird.html:544 runFrame: a frame in, the range's output frame out."""
    b = np.frombuffer(frame, np.uint8).copy()
    out = np.empty(b.size, np.uint8)
    hs = (ctypes.c_void_p * len(layers))(*[L.handle for L in layers])
    n = ctypes.c_int64()
    _abi.call("flock_range_forward_wire", hs, len(layers), _abi.ptr(b, _abi._u8p), b.size,
              _abi.ptr(out, _abi._u8p), out.size, ctypes.byref(n))
    return out[:n.value].tobytes()
