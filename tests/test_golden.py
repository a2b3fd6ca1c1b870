"""The committed regression fixtures (tests/golden/oracle_pins.npz, written by
tests/golden/make_golden.py from the oracle on seeded inputs): the oracle
still reproduces every one bit for bit, and the C-ABI host codecs (FLK1
pack) and torch's f32 -> bf16 conversion agree with the pinned bytes."""
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden  # noqa: E402

from flock_b200 import synth, wire  # noqa: E402


@pytest.fixture(scope="module")
def pins():
    return make_golden.load()


def test_oracle_reproduces_every_pin(oracle, pins):
    now = make_golden.compute()
    assert sorted(now) == sorted(pins)
    for k, v in pins.items():
        assert now[k].dtype == v.dtype and now[k].shape == v.shape, k
        assert np.array_equal(np.ascontiguousarray(now[k]).view(np.uint8),
                              np.ascontiguousarray(v).view(np.uint8)), k


def test_host_wire_pack_matches_pin(pins):
    x = synth.normal(9, "wire", 1024) * 0.05
    got = wire.pack(x, seq=1, hidden=1024, offset=17, reset=True)
    assert got == pins["wire_frame"].tobytes()
    vals, meta = wire.unpack(got)
    assert meta["offset"] == 17 and meta["reset"] and meta["seq"] == 1
    assert np.abs(vals - x).max() <= np.abs(x).max() * 2 ** -11


def test_bf16_pin_matches_torch(pins):
    x = make_golden.bf16_bits_input()
    want = torch.from_numpy(x).to(torch.bfloat16).to(torch.float32).numpy()
    assert np.array_equal(pins["bf16_round"].view(np.uint32), want.view(np.uint32))


def test_small_layer_pin_is_a_real_step(pins):
    # the pinned decode outputs move the state and the cache holds three keys
    out = pins["small_layer_decode"].reshape(3, -1)
    assert np.all(np.isfinite(out)) and not np.allclose(out[0], out[1])
    kvw = make_golden.SMALL["n_kv_heads"] * make_golden.SMALL["head_dim"]
    assert pins["small_layer_k"].size == 3 * kvw == pins["small_layer_v"].size
