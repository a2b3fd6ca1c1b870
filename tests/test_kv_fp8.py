"""The e4m3 rounding behind FLOCK_KV_FP8, on the CPU: the oracle's
fo_fp8_round against hand-checked values and against a nearest-code search
over the 253 finite E4M3FN values (ties to the even code), and the layer
config's mapping."""
import math

import numpy as np
import pytest

import oracle
from flock_b200 import _abi
from flock_b200.layer import QWEN3_06B


def _codes():
    """Every finite non-negative E4M3FN value, by code (0x00 .. 0x7E)."""
    vals = []
    for c in range(0x7F):
        e, m = c >> 3, c & 7
        vals.append(m * 2.0 ** -9 if e == 0 else (8 + m) * 2.0 ** (e - 10))
    return np.array(vals)


def _nearest(x: float) -> float:
    """Nearest finite e4m3 value by search, ties to the even code, saturating."""
    if math.isnan(x):
        return x
    a = abs(x)
    vals = _codes()
    if a >= vals[-1]:
        return math.copysign(vals[-1], x)
    d = np.abs(vals - a)
    best = np.flatnonzero(d == d.min())
    c = int(best[0]) if len(best) == 1 else int(best[best % 2 == 0][0])
    return math.copysign(float(vals[c]), x)


KNOWN = [(1.0, 1.0), (0.3, 0.3125), (448.0, 448.0), (464.0, 448.0), (500.0, 448.0),
         (-500.0, -448.0), (1e-4, 0.0), (1e-3, 2.0 ** -9), (2.0 ** -10, 0.0),
         (3 * 2.0 ** -10, 2.0 ** -8), (17.0, 16.0), (19.0, 20.0), (250.0, 256.0),
         (240.0, 240.0), (2.0 ** -6, 2.0 ** -6), (-0.0, -0.0), (float("inf"), 448.0),
         (float("-inf"), -448.0)]


@pytest.mark.parametrize("x,want", KNOWN)
def test_fp8_round_known_values(x, want):
    got = oracle.lib().fo_fp8_round(x)
    assert got == want and math.copysign(1.0, got) == math.copysign(1.0, want), (x, got, want)


def test_fp8_round_nan():
    assert math.isnan(oracle.lib().fo_fp8_round(float("nan")))


def test_fp8_round_matches_nearest_code_search():
    rng = np.random.default_rng(5)
    xs = np.concatenate([rng.standard_normal(4000) * s for s in (1e-3, 0.05, 1.0, 30.0, 300.0)]
                        + [_codes()[1:], -_codes()[1:],
                           (_codes()[1:-1] + _codes()[2:]) / 2])   # every midpoint: a tie
    xs = xs.astype(np.float32)
    for x in xs.tolist():
        assert oracle.lib().fo_fp8_round(x) == _nearest(x), x


def test_layer_config_fp8():
    c = QWEN3_06B.with_(attention="fast", prefill="tensor", kv="fp8").to_c()
    assert c.kv_dtype == _abi.FLOCK_KV_FP8 == 2
    with pytest.raises(ValueError):
        QWEN3_06B.with_(kv="fp16").to_c()


def test_ref_layer_rounds_every_append_fp8():
    from flock_b200 import synth
    s = synth.Shape(hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, ffn=512)
    cfg = dict(hidden=s.hidden, n_heads=s.n_heads, n_kv_heads=s.n_kv_heads, head_dim=s.head_dim,
               ffn=s.ffn)
    w = synth.layer_weights(11, 0, s)
    x = synth.normal(12, "h", s.hidden) * 0.05
    f = oracle.RefLayer(w, cfg, 64)
    q = oracle.RefLayer(w, cfg, 64, kv="fp8")
    f.forward(x, 1)
    q.forward(x, 1)
    fk, fv = f.cache()
    qk, qv = q.cache()
    rnd = np.vectorize(lambda v: oracle.lib().fo_fp8_round(float(v)), otypes=[np.float32])
    assert np.array_equal(qk, rnd(fk)) and np.array_equal(qv, rnd(fv))
    # every stored value is an e4m3 value
    assert np.array_equal(rnd(qk), qk) and np.array_equal(rnd(qv), qv)
