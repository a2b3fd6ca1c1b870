"""FLK1 frames (web/js/wire.mjs) through the C ABI against the oracle's
restatement: identical bytes from pack, identical values and header from
unpack, over ordinary activations and the edge values f32to16 treats
specially (subnormals, the f16 overflow boundary, infinities, NaN, signed
zero, round-half-to-even ties)."""
import numpy as np
import pytest

from flock_b200 import wire
from flock_b200._abi import FlockError


def edge_values():
    v = [0.0, -0.0, 1.0, -1.0, 65504.0, 65520.0, 65519.99, 1e6, -1e6, np.inf, -np.inf, np.nan,
         6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8, 1e-9, -3.1e-6,
         1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11, 1.0 + 2.0 ** -11 + 2.0 ** -20]
    return np.array(v, np.float32)


@pytest.mark.parametrize("kind", ["edge", "activations", "wide"])
def test_pack_matches_oracle(oracle, kind):
    rng = np.random.default_rng(3)
    x = {"edge": edge_values(),
         "activations": rng.standard_normal(4096).astype(np.float32) * 0.05,
         "wide": (rng.standard_normal(4096) * 10.0 ** rng.uniform(-9, 6, 4096)).astype(np.float32)}[kind]
    got = wire.pack(x, seq=3, hidden=7, offset=11, reset=True, replay=kind == "edge")
    want = oracle.wire_pack(x, 3, 7, 11, True, kind == "edge")
    assert got == want
    vals, meta = wire.unpack(got)
    ref, rmeta = oracle.wire_unpack(want)
    assert meta == rmeta
    assert np.array_equal(np.isnan(vals), np.isnan(ref))
    ok = ~np.isnan(ref)
    assert np.array_equal(vals[ok].view(np.uint32), ref[ok].view(np.uint32))


def test_unpack_rejects_foreign_bytes():
    good = wire.pack(np.ones(4, np.float32), 1, 4)
    with pytest.raises(FlockError, match="not a flock frame"):
        wire.unpack(b"FLK2" + good[4:])
    with pytest.raises(FlockError, match="not a flock frame"):
        wire.unpack(good[:19])
    vals, meta = wire.unpack(good)
    assert meta == {"seq": 1, "hidden": 4, "offset": 0, "reset": False, "replay": False}
    assert vals.tolist() == [1.0] * 4
