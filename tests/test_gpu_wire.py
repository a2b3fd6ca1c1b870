"""A held layer range driven by FLK1 frames (flock_range_forward_wire,
web/bird.html:544 runFrame): the output frame must be the bytes the
oracle gives for the same frames -- unpack, the layers in order (reset
clears, the offset must match), pack -- and a desynchronised offset is
refused without touching the caches."""
import numpy as np
import pytest

from flock_b200 import lib as flib
from flock_b200 import synth, wire
from flock_b200._abi import FlockError
from flock_b200.layer import QWEN3_06B, Layer

pytestmark = pytest.mark.gpu

CFG = dict(hidden=1024, n_heads=16, n_kv_heads=8, head_dim=128, ffn=3072)


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


def test_frames_match_oracle(dev, oracle):
    ws = [synth.layer_weights(60, i) for i in range(2)]
    layers = [Layer.create(dev, w, QWEN3_06B) for w in ws]
    oracle.set_fma_mode(True)
    try:
        refs = [oracle.RefLayer(w, CFG, 64) for w in ws]

        def ref_frame(frame):
            x, m = oracle.wire_unpack(frame)
            if m["reset"]:
                for r in refs:
                    r.reset()
            h = x
            for r in refs:
                h = r.forward(h, m["seq"])
            return oracle.wire_pack(h, m["seq"], m["hidden"], m["offset"], m["reset"], m["replay"])

        x = (synth.normal(61, "x", 4 * 1024) * 0.05).astype(np.float32)
        frames = [wire.pack(x, 4, 1024, 0, reset=True)]
        pos = 4
        for step in range(3):
            y = (synth.normal(62 + step, "y", 1024) * 0.05).astype(np.float32)
            frames.append(wire.pack(y, 1, 1024, pos, replay=step == 1))
            pos += 1
        for f in frames:
            got = wire.range_forward_wire(layers, f)
            assert got[:20] == f[:20]
            assert got == ref_frame(f)
    finally:
        oracle.set_fma_mode(False)
    assert layers[0].n_keys == 7
    with pytest.raises(FlockError, match="cache holds 7 positions, frame is at 3"):
        wire.range_forward_wire(layers, wire.pack(np.zeros(1024, np.float32), 1, 1024, 3))
    assert layers[0].n_keys == 7
    with pytest.raises(FlockError, match="values for seq"):
        wire.range_forward_wire(layers, wire.pack(np.zeros(512, np.float32), 1, 1024, 7))
    again = wire.range_forward_wire(layers, wire.pack(x, 4, 1024, 0, reset=True))
    assert layers[0].n_keys == 4 and len(again) == 20 + 8 * 1024
