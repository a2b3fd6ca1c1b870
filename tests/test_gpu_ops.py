"""Op-level parity of the sm_100a kernels against the CPU oracle, through the
C ABI.  Mirrors kernels/test_coop.ts, test_ops.ts and test_head.ts."""
import numpy as np
import pytest

from flock_b200 import lib as flib
from flock_b200 import ops, synth
from gpu_util import abs_err_scaled, bits, n_mismatch, rel_err

pytestmark = pytest.mark.gpu

EPS = 9.999999974752427e-7
VOCAB = 151936
# kernels/test_coop.ts:113-121 shapes, plus the model's other projections
SHAPES = [(64, 32), (30, 1024), (128, 1024), (1024, 1024), (2048, 1024), (3072, 1024),
          (1024, 3072), (1024, 2048), (37, 96), (5, 4096),
          # the 8B shape's large-matrix path (two rows per step, packed fold)
          (4096, 4096), (4097, 2048), (4096, 12288)]


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_matvec_q8_bit_exact(dev, oracle, rows, cols):
    # kernels/test_coop.ts:131-136: err === 0 against cpuMatmulQ8F32(coop(64))
    packed = synth.q8_tensor(1, f"w{rows}x{cols}", rows, cols)
    x = synth.normal(1, f"x{cols}", cols)
    w = flib.GpuTensor.from_packed(dev, packed, rows, cols)
    got = ops.matvec(dev, w, x)
    want = oracle.matmul_q8(packed, x, rows, cols)
    assert n_mismatch(got, want) == 0, rel_err(got, want)


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_matvec_q4_bit_exact(dev, oracle, rows, cols):
    packed = synth.q4_tensor(2, f"w{rows}x{cols}", rows, cols)
    x = synth.normal(2, f"x{cols}", cols)
    w = flib.GpuTensor.from_packed(dev, packed, rows, cols, flib.FLOCK_Q4_0)
    got = ops.matvec(dev, w, x)
    want = oracle.matmul_q4(packed, x, rows, cols)
    assert n_mismatch(got, want) == 0, rel_err(got, want)


def test_matvec_quantized_from_f32(dev, oracle):
    # the reference's own data path: randVec weights -> quantMatrixQ8 -> splitQ8
    rows, cols = 256, 1024
    w32 = flib.rand_vec(rows * cols, 0.05, seed=3)
    x = flib.rand_vec(cols, 1.0, seed=4)
    for q8 in (True, False):
        packed = flib.quant_matrix_q8(w32, rows, cols) if q8 else flib.quant_matrix_q4(w32, rows, cols)
        w = flib.GpuTensor.from_packed(dev, packed, rows, cols,
                                       flib.FLOCK_Q8_0 if q8 else flib.FLOCK_Q4_0)
        want = (oracle.matmul_q8 if q8 else oracle.matmul_q4)(packed, x, rows, cols)
        assert n_mismatch(ops.matvec(dev, w, x), want) == 0


def test_matvec_batched_tokens(dev, oracle):
    # kernels/q8_coop.wgsl:28-43 batching: per token identical to the decode matvec
    rows, cols, n = 512, 1024, 7
    packed = synth.q8_tensor(5, "wb", rows, cols)
    x = synth.normal(5, "xb", n * cols)
    w = flib.GpuTensor.from_packed(dev, packed, rows, cols)
    got = ops.matvec(dev, w, x, n)
    want = oracle.matmul_q8_batched(packed, x, rows, cols, n)
    assert n_mismatch(got, want) == 0


def test_matvec_lm_head_bit_exact(dev, oracle):
    rows, cols = VOCAB, 1024
    packed = synth.q8_tensor(6, "head", rows, cols)
    x = synth.normal(6, "hx", cols)
    w = flib.GpuTensor.from_packed(dev, packed, rows, cols)
    got = ops.matvec(dev, w, x)
    want = oracle.matmul_q8(packed, x, rows, cols)
    assert n_mismatch(got, want) == 0


@pytest.mark.parametrize("n,nv", [(1024, 1), (128, 16), (128, 8), (1024, 5), (96, 3), (4096, 1)])
def test_rmsnorm_bit_exact(dev, oracle, n, nv):
    # kernels/test_ops.ts:92-135 (the reference asserts < 3e-7; this is exact)
    x = synth.normal(7, f"x{n}{nv}", n * nv)
    g = synth.gain(7, f"g{n}", n)
    got = ops.rmsnorm(dev, x, g, n, nv, EPS)
    want = oracle.rmsnorm(x, g, n, nv, EPS)
    assert n_mismatch(got, want) == 0, rel_err(got, want)


@pytest.mark.parametrize("pairing", ["neox", "norm"])
@pytest.mark.parametrize("nt,nh,pos0", [(1, 16, 0), (1, 16, 137), (1, 8, 137), (7, 16, 0),
                                        (3, 8, 4000)])
def test_rope(dev, oracle, pairing, nt, nh, pos0):
    # kernels/test_ops.ts:190-225: absErrScaled < 4e-7; cos/sin here are the
    # f64 functions rounded once, like fr(Math.cos), so mismatches are rare
    inv = oracle.rope_inv_freq(128, 1e6)
    x = synth.normal(8, f"r{nt}{nh}{pos0}", nt * nh * 128)
    got = ops.rope(dev, x, nt, nh, 128, pos0, inv, pairing)
    want = oracle.rope(x, nt, nh, 128, pos0, inv, pairing == "neox")
    assert abs_err_scaled(got, want, float(np.abs(x).max())) < 4e-7
    assert n_mismatch(got, want) <= max(1, x.size // 10000)


@pytest.mark.parametrize("pairing", ["neox", "norm"])
def test_rope_planted_pairing(dev, oracle, pairing):
    # kernels/test_ops.ts:229-263
    inv = oracle.rope_inv_freq(128, 1e6)
    x = np.zeros(128, np.float32)
    x[0] = 1
    got = ops.rope(dev, x, 1, 1, 128, 1, inv, pairing)
    partner, other = (64, 1) if pairing == "neox" else (1, 64)
    assert abs(got[0] - np.cos(inv[0])) < 1e-6 and abs(got[partner] - np.sin(inv[0])) < 1e-6
    assert got[other] == 0


def test_swiglu_and_add(dev, oracle):
    # kernels/test_ops.ts:266-288: swiglu < 1e-6, add === 0
    g = synth.normal(9, "g", 3072 * 3) * 4
    u = synth.normal(9, "u", 3072 * 3)
    got = ops.swiglu(dev, g, u)
    want = oracle.swiglu(g, u)
    assert rel_err(got, want) < 1e-6
    assert n_mismatch(got, want) <= 2
    a = synth.normal(9, "a", 5000)
    assert n_mismatch(ops.add(dev, a, u[:5000]), oracle.add(a, u[:5000])) == 0


@pytest.mark.parametrize("nk", [1, 2, 63, 257, 2048])
def test_attention_exact(dev, oracle, nk):
    # kernels/test_ops.ts:315-355: relErr(..., 1e-3) < 1e-4; here the order is
    # attnRef's, so only f32-FMA vs the JS double-rounded fma32 can differ
    nH, nKV, hd = 16, 8, 128
    q = synth.normal(10, f"q{nk}", nH * hd)
    k = synth.normal(10, f"k{nk}", nk * nKV * hd)
    v = synth.normal(10, f"v{nk}", nk * nKV * hd)
    got = ops.attention(dev, q, k, v, nH, nKV, hd, nk, "exact")
    want = oracle.attn(q, k, v, nH, nKV, hd, nk)
    assert rel_err(got, want, 1e-3) < 1e-4
    oracle.set_fma_mode(True)
    try:
        want_ieee = oracle.attn(q, k, v, nH, nKV, hd, nk)
    finally:
        oracle.set_fma_mode(False)
    assert n_mismatch(got, want_ieee) <= max(2, got.size // 1000)


@pytest.mark.parametrize("nk", [1, 17, 257, 2048, 4608])
def test_attention_fast(dev, oracle, nk):
    # the split-K flash-decode: reassociated, no key cap (4608 > the WGSL 2048)
    nH, nKV, hd = 16, 8, 128
    q = synth.normal(11, f"q{nk}", nH * hd)
    k = synth.normal(11, f"k{nk}", nk * nKV * hd)
    v = synth.normal(11, f"v{nk}", nk * nKV * hd)
    got = ops.attention(dev, q, k, v, nH, nKV, hd, nk, "fast")
    want = oracle.attn(q, k, v, nH, nKV, hd, nk)
    # stated tolerance of the reassociated path: 1e-5 of the output scale, and
    # the north star's f32-decode bound (max rel err <= 1e-3, 1e-3 floor)
    assert abs_err_scaled(got, want) < 1e-5
    assert rel_err(got, want, 1e-3) < 1e-3


def test_attention_gqa_map(dev):
    # kernels/test_ops.ts:357-394
    nH, nKV, hd = 4, 2, 128
    q = np.zeros(nH * hd, np.float32)
    k = np.zeros(nKV * hd, np.float32)
    v = np.concatenate([np.full(hd, 7, np.float32), np.full(hd, -3, np.float32)])
    for mode in ("exact", "fast"):
        got = ops.attention(dev, q, k, v, nH, nKV, hd, 1, mode).reshape(nH, hd)
        for h, want in enumerate([7, 7, -3, -3]):
            assert np.all(got[h] == want), mode


@pytest.mark.parametrize("nq,pos0", [(1, 0), (2, 0), (7, 3), (13, 60), (65, 0), (3, 900)])
def test_attention_prefill(dev, oracle, nq, pos0):
    # kernels/test_head.ts:262-390 / test_prefill.ts: streaming order, tolerance
    nH, nKV, hd = 16, 8, 128
    nk = pos0 + nq
    q = synth.normal(12, f"q{nq}{pos0}", nq * nH * hd)
    k = synth.normal(12, f"k{nq}{pos0}", nk * nKV * hd)
    v = synth.normal(12, f"v{nq}{pos0}", nk * nKV * hd)
    got = ops.attention_prefill(dev, q, k, v, nH, nKV, hd, nq, pos0)
    want = oracle.attn_prefill(q, k, v, nH, nKV, hd, nq, pos0)
    assert abs_err_scaled(got, want) < 2e-6
    oracle.set_fma_mode(True)
    try:
        want_ieee = oracle.attn_prefill(q, k, v, nH, nKV, hd, nq, pos0)
    finally:
        oracle.set_fma_mode(False)
    assert n_mismatch(got, want_ieee) <= max(2, got.size // 1000)


def test_embed_bit_exact(dev, oracle):
    # kernels/test_head.ts: embed exact (gather from the split layout vs the
    # reference's decode of the 34-byte layout)
    V, H = 4096, 1024
    packed = synth.q8_tensor(13, "embd", V, H)
    t = flib.GpuTensor.from_packed(dev, packed, V, H)
    ids = [0, 1, 4095, 17, 17, 2048]
    assert n_mismatch(ops.embed(dev, t, ids), oracle.embed(packed, ids, H)) == 0


@pytest.mark.parametrize("at", [0, 1, 255, 256, 257, 151935, 75000])
def test_argmax_planted(dev, at):
    # kernels/test_head.ts:208-215
    x = np.array([-1 - (i % 7) * 0.001 for i in range(VOCAB)], np.float32)
    x[at] = 5
    assert ops.argmax(dev, x)[0] == at


def test_argmax_ties_negative_random(dev, oracle):
    # kernels/test_head.ts:219-256
    x = np.full(VOCAB, -1, np.float32)
    x[900] = x[40000] = x[151000] = 3
    assert ops.argmax(dev, x)[0] == 900
    n = VOCAB
    neg = np.array([-100 - (n - i) * 1e-3 for i in range(n)], np.float32)
    assert ops.argmax(dev, neg)[0] == oracle.argmax(neg)
    for n in (256, 1000, 4096, VOCAB):
        r = synth.normal(14, f"a{n}", n) * 10
        assert ops.argmax(dev, r)[0] == oracle.argmax(r)


def test_raw_buffer_roundtrip(dev):
    """kernels/lib.ts:548 storageBuffer / :576 readBack through the C ABI: a
    34-byte (not 4-aligned) upload reads back byte-for-byte, the pad is zero,
    and a range past the end is refused."""
    import ctypes

    from flock_b200 import _abi
    data = np.arange(34, dtype=np.uint8)
    h = ctypes.c_void_p()
    _abi.call("flock_tensor_from_bytes", dev.handle, data.ctypes.data, 34, ctypes.byref(h))
    try:
        out = np.zeros(36, np.uint8)
        _abi.call("flock_tensor_read", h, 0, 36, out.ctypes.data)
        assert np.array_equal(out[:34], data) and not out[34:].any()
        part = np.zeros(8, np.uint8)
        _abi.call("flock_tensor_read", h, 10, 8, part.ctypes.data)
        assert np.array_equal(part, data[10:18])
        assert _abi.lib().flock_tensor_read(h, 30, 8, part.ctypes.data) == _abi.FLOCK_E_LIMIT
    finally:
        _abi.lib().flock_tensor_free(h)
