"""Cross-check the C oracle against the JS-semantics transliteration (oracle/jsref.py).

Two independent restatements of the same TypeScript must agree bit for bit on
small seeded cases; a disagreement is a restatement error in one of them.
Also measures how often the literal fma32 (f64 add, then f32 round) differs
from an IEEE single-rounding fmaf on the shapes of data each chain sees, so a
GPU-vs-oracle difference can be attributed.  CPU only.
"""
import numpy as np
import pytest

from flock_b200 import synth
from oracle import jsref


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_quantizers_match(oracle):
    w = (synth.normal(1, "q", 8 * 64) * 0.05)
    w[3] = 0.0
    w[64:96] = 0.0  # an all-zero block: d == 0 path
    for r in range(8):
        row = w[r * 64:(r + 1) * 64]
        assert bytes(oracle.quant_matrix_q8(row, 1, 64)) == jsref.quant_row_q8(row)
        assert bytes(oracle.quant_matrix_q4(row, 1, 64)) == jsref.quant_row_q4(row)


def test_f32to16_matches(oracle):
    vals = np.concatenate([synth.normal(2, "h", 2000) * s for s in (1e-6, 1e-3, 1.0, 1e4, 7e4)])
    for v in vals:
        assert oracle.f32to16(float(v)) == jsref.f32to16(float(v))


@pytest.mark.parametrize("lanes", [0, 64, 8])
@pytest.mark.parametrize("rows,cols", [(3, 32), (5, 96), (2, 1024)])
def test_matmul_matches(oracle, rows, cols, lanes):
    x = synth.normal(3, "x", cols)
    p8 = synth.q8_tensor(3, "w8", rows, cols)
    p4 = synth.q4_tensor(3, "w4", rows, cols)
    assert np.array_equal(_bits(oracle.matmul_q8(p8, x, rows, cols, lanes)),
                          _bits(jsref.cpu_matmul_q8(bytes(p8), x, rows, cols, lanes)))
    assert np.array_equal(_bits(oracle.matmul_q4(p4, x, rows, cols, lanes)),
                          _bits(jsref.cpu_matmul_q4(bytes(p4), x, rows, cols, lanes)))


def test_rmsnorm_matches(oracle):
    for n, nv in [(1024, 1), (128, 3), (96, 2)]:
        x = synth.normal(4, f"x{n}", n * nv)
        g = synth.gain(4, f"g{n}", n)
        assert np.array_equal(_bits(oracle.rmsnorm(x, g, n, nv)),
                              _bits(jsref.rmsnorm(x, g, n, nv, oracle.EPS)))


@pytest.mark.parametrize("neox", [True, False])
def test_rope_matches(oracle, neox):
    inv_c = oracle.rope_inv_freq(128, 1e6)
    inv_j = jsref.rope_inv_freq(128, 1e6)
    assert np.array_equal(_bits(inv_c), _bits(inv_j))
    x = synth.normal(5, "r", 2 * 3 * 128)
    a = oracle.rope(x, 2, 3, 128, 137, inv_c, neox)
    b = jsref.rope(x, 2, 3, 128, 137, inv_j, neox)
    assert np.array_equal(_bits(a), _bits(b))


def test_swiglu_and_embed_match(oracle):
    g = synth.normal(6, "g", 512) * 4
    u = synth.normal(6, "u", 512)
    assert np.array_equal(_bits(oracle.swiglu(g, u)), _bits(jsref.swiglu(g, u)))
    packed = synth.q8_tensor(6, "e", 10, 64)
    ids = [3, 0, 9, 3]
    assert np.array_equal(_bits(oracle.embed(packed, ids, 64)),
                          _bits(jsref.embed(bytes(packed), ids, 64)))


def test_attention_matches(oracle):
    nH, nKV, hd, nk = 4, 2, 128, 9
    q = synth.normal(7, "q", nH * hd)
    k = synth.normal(7, "k", nk * nKV * hd)
    v = synth.normal(7, "v", nk * nKV * hd)
    assert np.array_equal(_bits(oracle.attn(q, k, v, nH, nKV, hd, nk)),
                          _bits(jsref.attn(q, k, v, nH, nKV, hd, nk)))


def test_attention_prefill_matches(oracle):
    nH, nKV, hd, nq, pos0 = 2, 1, 128, 3, 70  # crosses a 64-key tile boundary
    nk = pos0 + nq
    q = synth.normal(8, "q", nq * nH * hd)
    k = synth.normal(8, "k", nk * nKV * hd)
    v = synth.normal(8, "v", nk * nKV * hd)
    assert np.array_equal(_bits(oracle.attn_prefill(q, k, v, nH, nKV, hd, nq, pos0)),
                          _bits(jsref.attn_prefill(q, k, v, nH, nKV, hd, nq, pos0)))


def test_argmax_and_ranges_match(oracle):
    x = synth.normal(9, "a", 5000)
    assert oracle.argmax(x) == jsref.argmax(x)
    for total, n, align in [(1024, 3, 32), (151936, 8, 1), (30, 4, 1)]:
        assert oracle.shard_ranges(total, n, align) == jsref.shard_ranges(total, n, align)


def _fma_disagreements(a, b, c):
    """How often fround(a*b+c in f64) != fmaf(a,b,c), over float64 arrays of f32 values."""
    a64, b64, c64 = (np.asarray(t, np.float32).astype(np.float64) for t in (a, b, c))
    js = (a64 * b64 + c64).astype(np.float32)
    # IEEE fmaf via exact products: a*b is exact in f64; the sum is exact in
    # longdouble (64-bit mantissa) for these magnitudes, then one rounding to f32.
    ld = (a64.astype(np.longdouble) * b64.astype(np.longdouble) + c64.astype(np.longdouble))
    ieee = ld.astype(np.float32)
    return int(np.count_nonzero(js.view(np.uint32) != ieee.view(np.uint32)))


def test_fma32_equals_fmaf_on_int8_products():
    # Matvec chains multiply an int8 (<= 8 significant bits) by an f32: the
    # product has <= 32 bits, so product + accumulator is exact in f64 and the
    # literal fma32 is a single rounding -- identical to the GPU's fmaf.
    rng = np.random.default_rng(0)
    n = 2_000_000
    q = rng.integers(-128, 128, n).astype(np.float32)
    x = rng.standard_normal(n).astype(np.float32)
    acc = (rng.standard_normal(n) * 30).astype(np.float32)
    assert _fma_disagreements(q, x, acc) == 0
