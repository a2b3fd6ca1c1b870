"""Failure detection without a GPU fault: a bounded device-side wait that
runs out returns an error status the host reads, and the context stays
usable.

The tensor-parallel peer exchange (flock_peer.cu) is run as one rank of a
two-rank exchange whose peer never publishes its flag (a local buffer that
nothing writes): the exchange kernel gives up after its 50 ms limit and sets
the error word; the host check reports FLOCK_E_CUDA, and the failure is
sticky -- the rank is an exchange out of step with its peers, so every later
exchange is refused rather than summing partials of another step."""
import ctypes

import numpy as np
import pytest

from flock_b200 import _abi, ops
from flock_b200 import lib as flib
from flock_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


def test_peer_exchange_wait_runs_out_and_stays_failed(dev):
    first = ctypes.c_int(0)
    rc = _abi.lib().flock_op_peer_exchange_lone(dev.handle, 2, 1024, 50, 3, ctypes.byref(first))
    assert first.value == _abi.FLOCK_E_CUDA
    assert rc == _abi.FLOCK_E_CUDA
    assert "failed earlier" in _abi.last_error()
    # the context is still usable: a matvec right after is bit-exact
    w = synth.q8_tensor(3, "after", 64, 1024)
    t = flib.GpuTensor.from_packed(dev, w, 64, 1024)
    x = synth.normal(3, "x", 1024)
    y1 = ops.matvec(dev, t, x)
    y2 = ops.matvec(dev, t, x)
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))
    t.free()


def test_peer_exchange_lone_rejects_bad_arguments(dev):
    first = ctypes.c_int(0)
    for args in [(1, 1024, 50, 1), (2, 1023, 50, 1), (2, 1024, 0, 1), (2, 1024, 50, 0)]:
        rc = _abi.lib().flock_op_peer_exchange_lone(dev.handle, *args, ctypes.byref(first))
        assert rc == _abi.FLOCK_E_ARG
