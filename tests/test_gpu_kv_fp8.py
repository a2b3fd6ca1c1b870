"""The e4m3 KV cache (kv="fp8", FLOCK_KV_FP8) on the GPU against the oracle
layer with the same rounding (RefLayer(kv="fp8"), fo_fp8_round: nearest
E4M3FN, ties to even, saturating at 448): a preloaded cache is stored
rounded and read back exactly; decode steps over the e4m3 rows within the
fast-attention bound 1e-5 absErrScaled with the appended rows equal to the
oracle's; the tensor-core prefill within its 1e-2 bound; the persistent
decode kernel bit-identical to the kernel graph; a model close to the f32
cache's within fp8's own rounding; the streaming engine and the exact
kernels refuse it."""
import numpy as np
import pytest

from flock_b200 import lib as flib
from flock_b200 import synth
from flock_b200._abi import FlockError
from flock_b200.layer import QWEN3_06B, Layer
from flock_b200.model import Model
from gpu_util import abs_err_scaled, bits, n_mismatch

pytestmark = pytest.mark.gpu

S = synth.QWEN3_06B
CFG = dict(hidden=S.hidden, n_heads=S.n_heads, n_kv_heads=S.n_kv_heads, head_dim=S.head_dim,
           ffn=S.ffn)
KVW = S.n_kv_heads * S.head_dim
F8 = QWEN3_06B.with_(attention="fast", prefill="tensor", kv="fp8")
F32 = QWEN3_06B.with_(attention="fast", prefill="tensor")


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def weights():
    return synth.layer_weights(110, 24)


def _ref(oracle, weights, cap=4096):
    oracle.set_fma_mode(False)
    return oracle.RefLayer(weights, CFG, cap, kv="fp8")


def _fp8_np(oracle, x):
    f = oracle.lib().fo_fp8_round
    return np.array([f(float(v)) for v in np.asarray(x, np.float32)], np.float32)


def test_write_rounds_read_widens(dev, oracle, weights):
    kc = synth.normal(411, "k", 16 * KVW) * np.float32(40.0)   # past 448 too
    vc = synth.normal(411, "v", 16 * KVW) * np.float32(1e-2)   # into the subnormals
    L = Layer.create(dev, weights, F8)
    L.write_cache(kc, vc)
    k, v = L.cache_buffers()
    assert np.array_equal(bits(k), bits(_fp8_np(oracle, kc)))
    assert np.array_equal(bits(v), bits(_fp8_np(oracle, vc)))


@pytest.mark.parametrize("n_cache", [256, 8192])
def test_decode_over_preloaded_cache(dev, oracle, weights, n_cache):
    kc = synth.normal(412, f"k{n_cache}", n_cache * KVW)
    vc = synth.normal(412, f"v{n_cache}", n_cache * KVW)
    L = Layer.create(dev, weights, F8.with_(max_keys=n_cache + 8))
    L.write_cache(kc, vc)
    ref = _ref(oracle, weights, n_cache + 8)
    ref.fill_cache(kc, vc)
    for step in range(3):
        x = synth.normal(413, f"x{step}", S.hidden)
        got = L.forward(x)
        want = ref.forward(x, 1)
        e = abs_err_scaled(got, want)
        print(f"{n_cache} keys, step {step}: absErrScaled {e:.2e}")
        assert e < 1e-5
    k, v = L.cache_buffers()
    rk, rv = ref.cache()
    assert L.n_keys == n_cache + 3
    assert np.array_equal(bits(k[:n_cache * KVW]), bits(rk[:n_cache * KVW]))
    assert np.array_equal(bits(v), bits(rv))
    assert n_mismatch(k[n_cache * KVW:], rk[n_cache * KVW:]) <= 2


@pytest.mark.parametrize("n", [16, 130])
def test_tensor_prefill_fp8(dev, oracle, weights, n):
    x = synth.normal(414, f"p{n}", n * S.hidden).astype(np.float32)
    L = Layer.create(dev, weights, F8)
    L.encode_prefill(n, x)
    got = L.read_output(n)
    ref = _ref(oracle, weights)
    want = ref.forward(x, n)
    e = abs_err_scaled(got - x, want - x)
    print(f"prefill {n}: layer contribution absErrScaled {e:.2e}")
    assert e <= 1e-2
    # then decode on the rows the prefill stored
    y = synth.normal(414, "dec", S.hidden).astype(np.float32)
    got_y = L.forward(y)
    want_y = ref.forward(y, 1)
    assert abs_err_scaled(got_y - y, want_y - y) <= 1e-2


def test_persistent_bit_identical_fp8(dev):
    m = synth.model(210, n_layers=2, vocab=4096)
    a = Model.create(dev, m, F8)
    b = Model.create(dev, m, F8)
    a.decode_mode = "persistent"
    assert a.decode_mode == "persistent" and b.decode_mode == "kernels"
    ids = synth.uniform_ids(17, "long", 1500, 4096).tolist()
    for M in (a, b):
        for i in range(0, 1500, 500):
            M.step(ids[i:i + 500])
    got = a.decode_device(12)
    want = b.decode_device(12)
    assert got.tolist() == want.tolist()
    la, lb = a.logits([int(got[-1])]), b.logits([int(want[-1])])
    assert np.array_equal(bits(la), bits(lb))


def test_model_fp8_close_to_f32(dev):
    """fp8 keeps 3 mantissa bits (relative rounding up to 2^-4 per element):
    the logits move by its own rounding, not by an error of the path."""
    m = synth.model(211, n_layers=2, vocab=4096)
    a = Model.create(dev, m, F8)
    b = Model.create(dev, m, F32)
    prompt = synth.uniform_ids(18, "prompt", 300, 4096).tolist()
    worst = abs_err_scaled(a.logits(prompt), b.logits(prompt))
    for t in (5, 77, 4000):
        worst = max(worst, abs_err_scaled(a.logits([t]), b.logits([t])))
    print(f"fp8 vs f32 cache logits: absErrScaled {worst:.2e}")
    assert worst <= 5e-2
    assert a.pos == b.pos == 303


def test_stream_engine_refuses_fp8(dev):
    m = synth.model(212, n_layers=2, vocab=4096)
    M = Model.create(dev, m, F8)
    M.decode_mode = "stream"
    assert M.decode_mode == "kernels"


@pytest.mark.parametrize("over", [dict(attention="exact"), dict(prefill="exact")])
def test_exact_kernels_refuse_fp8(dev, weights, over):
    with pytest.raises(FlockError) as e:
        Layer.create(dev, weights, F8.with_(**over))
    assert e.value.code == -8 and "fp8" in str(e.value)
