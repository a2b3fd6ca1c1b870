"""An NCCL communicator of one rank, bound to that rank's device and stream
(flock_comm_init).  The 128-byte unique id comes from rank 0
(``Comm.unique_id()``) and reaches the other ranks by any host channel: a
queue, a torch.distributed gloo broadcast, a file."""
from __future__ import annotations

import ctypes

import numpy as np

from . import _abi
from .lib import Device


class Comm:
    def __init__(self, dev: Device, world: int, rank: int, uid: bytes, timeout_ms: int = 30000):
        self.dev, self.world, self.rank = dev, world, rank
        u = np.frombuffer(uid, np.uint8).copy()
        if u.size != 128:
            raise ValueError(f"an NCCL unique id is 128 bytes, got {u.size}")
        h = ctypes.c_void_p()
        _abi.call("flock_comm_init", dev.handle, world, rank, _abi.ptr(u, _abi._u8p), timeout_ms,
                  ctypes.byref(h))
        self.handle = h

    @staticmethod
    def unique_id() -> bytes:
        u = np.zeros(128, np.uint8)
        _abi.call("flock_comm_unique_id", _abi.ptr(u, _abi._u8p))
        return u.tobytes()

    def free(self) -> None:
        if self.handle:
            _abi.lib().flock_comm_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
