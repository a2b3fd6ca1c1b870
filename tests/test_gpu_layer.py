"""One Qwen3 layer on the GPU vs layer_ref.ts (kernels/test_layer.ts,
test_prefill.ts, test_frombuffers.ts), including benchmark config 0: decode at
position 256 over a 256-key N(0,1) cache."""
import numpy as np
import pytest

from flock_b200 import lib as flib
from flock_b200 import synth
from flock_b200._abi import FlockError
from flock_b200.layer import QWEN3_06B, Layer
from gpu_util import abs_err_scaled, n_mismatch

pytestmark = pytest.mark.gpu

S = synth.QWEN3_06B
CFG = dict(hidden=S.hidden, n_heads=S.n_heads, n_kv_heads=S.n_kv_heads, head_dim=S.head_dim,
           ffn=S.ffn)


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def weights():
    return synth.layer_weights(100, 24)


def _ref(oracle, weights, ieee=False, cap=4096):
    oracle.set_fma_mode(ieee)
    return oracle.RefLayer(weights, CFG, cap)


def _fwd(oracle, ref, x, n, ieee):
    oracle.set_fma_mode(ieee)
    try:
        return ref.forward(x, n)
    finally:
        oracle.set_fma_mode(False)


@pytest.mark.parametrize("mode", ["exact", "fast"])
def test_config0_decode_at_256(dev, oracle, weights, mode):
    kvw = S.n_kv_heads * S.head_dim
    kc = synth.normal(101, "kcache", 256 * kvw)
    vc = synth.normal(101, "vcache", 256 * kvw)
    x = synth.normal(101, "x", S.hidden)
    L = Layer.create(dev, weights, QWEN3_06B.with_(attention=mode))
    L.write_cache(kc, vc)
    assert L.n_keys == 256
    got = L.forward(x)
    js = _ref(oracle, weights)
    js.fill_cache(kc, vc)
    want = _fwd(oracle, js, x, 1, False)
    if mode == "exact":
        assert abs_err_scaled(got, want) < 1e-6  # kernels/test_layer.ts:86-174
        ie = _ref(oracle, weights, True)
        ie.fill_cache(kc, vc)
        want_ieee = _fwd(oracle, ie, x, 1, True)
        assert n_mismatch(got, want_ieee) == 0
    else:
        assert abs_err_scaled(got, want) < 1e-5
    # the appended key/value (position 256) is bit-identical in both modes
    k, v = L.cache_buffers()
    rk, rv = js.cache()
    assert L.n_keys == 257
    assert np.array_equal(v, rv)
    assert n_mismatch(k[256 * kvw:], rk[256 * kvw:]) <= 2


def test_fast_decode_over_long_cache(dev, oracle, weights):
    """8192 keys: past 2048 keys of capacity the split-K attention runs up to 64
    splits (three CTAs per SM), combined two splits per lane."""
    kvw = S.n_kv_heads * S.head_dim
    kc = synth.normal(107, "k8k", 8192 * kvw)
    vc = synth.normal(107, "v8k", 8192 * kvw)
    L = Layer.create(dev, weights, QWEN3_06B.with_(attention="fast", max_keys=8200))
    L.write_cache(kc, vc)
    ref = _ref(oracle, weights, cap=8200)
    ref.fill_cache(kc, vc)
    for step in range(2):
        x = synth.normal(107, f"x{step}", S.hidden)
        got = L.forward(x)
        want = _fwd(oracle, ref, x, 1, False)
        assert abs_err_scaled(got, want) < 1e-5
    assert L.n_keys == 8194


@pytest.mark.parametrize("mode", ["exact", "fast"])
def test_four_decode_steps(dev, oracle, weights, mode):
    L = Layer.create(dev, weights, QWEN3_06B.with_(attention=mode))
    ref = _ref(oracle, weights)
    for step in range(4):
        x = synth.normal(102, f"s{step}", S.hidden) * 0.5
        got = L.forward(x)
        want = _fwd(oracle, ref, x, 1, False)
        assert abs_err_scaled(got, want) < (1e-6 if mode == "exact" else 1e-5)
        assert abs_err_scaled(got, x) > 1e-3  # not a pass-through
    assert L.n_keys == 4


@pytest.mark.parametrize("n", [1, 2, 7, 13, 64, 65])
def test_prefill_vs_reference(dev, oracle, weights, n):
    # kernels/test_prefill.ts:46-58 (< 2e-6)
    x = synth.normal(103, f"p{n}", n * S.hidden) * 0.05
    L = Layer.create(dev, weights)
    L.encode_prefill(n, x)
    got = L.read_output(n)
    want = _fwd(oracle, _ref(oracle, weights), x, n, False)
    assert abs_err_scaled(got, want) < 2e-6
    want_ieee = _fwd(oracle, _ref(oracle, weights, True), x, n, True)
    assert n_mismatch(got, want_ieee) <= max(2, got.size // 2000)


def test_prefill_equals_decode_kv_cache(dev, weights):
    # kernels/test_prefill.ts:80-135: bit-identical KV cache
    n = 9
    x = synth.normal(104, "pd", n * S.hidden) * 0.05
    A = Layer.create(dev, weights)
    A.encode_prefill(n, x)
    outA = A.read_output(n)
    B = Layer.create(dev, weights)
    outB = np.concatenate([B.forward(x[i * S.hidden:(i + 1) * S.hidden]) for i in range(n)])
    ka, va = A.cache_buffers()
    kb, vb = B.cache_buffers()
    assert np.array_equal(ka, kb) and np.array_equal(va, vb)
    assert abs_err_scaled(outA, outB) < 2e-6


def test_prefill_then_decode_at_900(dev, oracle, weights):
    # kernels/test_prefill.ts:143-185 and the pos0 = 900 RoPE liveness (:211-262),
    # over a preloaded 900-key cache so the oracle stays cheap
    kvw = S.n_kv_heads * S.head_dim
    kc = synth.normal(105, "k900", 900 * kvw)
    vc = synth.normal(105, "v900", 900 * kvw)
    L = Layer.create(dev, weights)
    L.write_cache(kc, vc)
    ref = _ref(oracle, weights)
    ref.fill_cache(kc, vc)
    pre = synth.normal(105, "pre", 3 * S.hidden) * 0.05
    L.encode_prefill(3, pre)
    got_pre = L.read_output(3)
    want_pre = _fwd(oracle, ref, pre, 3, False)
    assert abs_err_scaled(got_pre, want_pre) < 2e-6
    x = synth.normal(105, "dec", S.hidden)
    got = L.forward(x)
    want = _fwd(oracle, ref, x, 1, False)
    assert abs_err_scaled(got, want) < 2e-6
    assert L.n_keys == 904


def test_guards(dev, weights):
    # kernels/test_prefill.ts:292-307 and layer.ts:575 KV full
    L = Layer.create(dev, weights, QWEN3_06B.with_(max_keys=8, max_prefill=4))
    with pytest.raises(FlockError, match="maxPrefill"):
        L.encode_prefill(5, np.zeros(5 * S.hidden, np.float32))
    with pytest.raises(ValueError, match="expected"):
        L.encode_prefill(2, np.zeros(S.hidden, np.float32))
    L.encode_prefill(4, np.zeros(4 * S.hidden, np.float32))
    L.encode_prefill(4, np.zeros(4 * S.hidden, np.float32))
    with pytest.raises(FlockError, match="KV cache full"):
        L.encode(np.zeros(S.hidden, np.float32))


def test_from_buffers_equals_create(dev, weights):
    # kernels/test_frombuffers.ts:58-135
    x = synth.normal(106, "fb", 3 * S.hidden) * 0.05
    A = Layer.create(dev, weights)
    tensors = {}
    for name, t in weights.items():
        if isinstance(t, dict):
            qs, sc = flib.split_q8(t["packed"], t["rows"], t["cols"])
            tensors[name] = flib.GpuTensor.from_split(dev, qs, sc, t["rows"], t["cols"])
        else:
            tensors[name] = flib.GpuTensor.from_f32(dev, t)
    B = Layer.from_buffers(dev, tensors)
    assert np.array_equal(A.forward(x), B.forward(x))
    assert np.array_equal(A.forward(x[:S.hidden]), B.forward(x[:S.hidden]))


def test_missing_tensor_is_named(dev, weights):
    tensors = {n: (flib.GpuTensor.from_packed(dev, t["packed"], t["rows"], t["cols"])
                   if isinstance(t, dict) else flib.GpuTensor.from_f32(dev, t))
               for n, t in weights.items() if n != "ffn_up.weight"}
    with pytest.raises(FlockError, match="ffn_up.weight"):
        Layer.from_buffers(dev, tensors)
