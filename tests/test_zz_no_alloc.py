"""The allocation-free greedy argmax (flock_argmax_noalloc), through the C ABI.

Callers that cannot allocate device memory (a serving framework owning the
GPU's memory, an allocation-free decode loop, an FFI caller with raw device
pointers) pass their own input and output buffers; the kernel's scratch is a
fixed array inside the library.  Checked against the oracle's argmaxRef
(kernels/head_ref.ts:65, lowest index among equal maxima) on random logits
and on a planted three-way tie, two calls in a row, so the second call also
proves the shared scratch is reset between calls.  Named to be collected
last.
"""
import ctypes

import numpy as np
import pytest

from flock_b200 import _abi, ops, synth
from flock_b200 import lib as flib

pytestmark = pytest.mark.gpu


def test_argmax_noalloc_matches_the_oracle(oracle):
    import torch

    dev = flib.get_device(0)
    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream()
    idx_out = torch.full((1,), -1, dtype=torch.int32, device="cuda:0")
    val_out = torch.zeros((1,), dtype=torch.float32, device="cuda:0")
    a = synth.normal(31, "logits-a", 151936) * 10
    b = np.full(151936, -1.0, np.float32)
    b[[40000, 900, 151000]] = 3.0  # a tie: the lowest index wins
    cases = [a, b]
    for x in cases:  # two calls in a row share the library's scratch
        xd = torch.from_numpy(x).to("cuda:0")
        _abi.call("flock_argmax_noalloc", ctypes.c_void_p(xd.data_ptr()), x.size,
                  ctypes.c_void_p(idx_out.data_ptr()), ctypes.c_void_p(val_out.data_ptr()),
                  ctypes.c_void_p(stream.cuda_stream))
        stream.synchronize()
        want_idx = oracle.argmax(x)
        assert int(idx_out.item()) == want_idx
        assert np.float32(val_out.item()).view(np.uint32) == x[want_idx].view(np.uint32)
        # and the allocating entry point agrees
        assert ops.argmax(dev, x)[0] == want_idx
    assert int(idx_out.item()) == 900


def test_argmax_noalloc_rejects_oversize():
    import torch

    x = torch.zeros((8,), dtype=torch.float32, device="cuda:0")
    o = torch.zeros((1,), dtype=torch.int32, device="cuda:0")
    v = torch.zeros((1,), dtype=torch.float32, device="cuda:0")
    with pytest.raises(_abi.FlockError, match="maximum"):
        _abi.call("flock_argmax_noalloc", ctypes.c_void_p(x.data_ptr()), 4194305,
                  ctypes.c_void_p(o.data_ptr()), ctypes.c_void_p(v.data_ptr()), None)
