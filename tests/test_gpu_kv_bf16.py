"""The bf16 KV cache (kv="bf16", FLOCK_KV_BF16) on the GPU against the oracle
layer with the same rounding (RefLayer(kv="bf16")): a preloaded cache is
stored rounded and read back exactly; decode steps (split-K attention over
the bf16 rows) within the fast-attention bound 1e-5 absErrScaled with the
appended rows equal to the oracle's; tensor-core prefill within its 1e-2
bound; the persistent decode kernel bit-identical to the kernel graph; and
the exact kernels, which read f32, refuse the option."""
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
BF = QWEN3_06B.with_(attention="fast", prefill="tensor", kv="bf16")
F32 = QWEN3_06B.with_(attention="fast", prefill="tensor")


def bf16_np(x):
    w = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    w = ((w + 0x7FFF + ((w >> 16) & 1)) >> 16) << 16
    return w.astype(np.uint32).view(np.float32)


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def weights():
    return synth.layer_weights(100, 24)


def _ref(oracle, weights, cap=4096):
    oracle.set_fma_mode(False)
    return oracle.RefLayer(weights, CFG, cap, kv="bf16")


def test_write_rounds_read_widens(dev, weights):
    kc = synth.normal(401, "k", 64 * KVW)
    vc = synth.normal(401, "v", 64 * KVW)
    L = Layer.create(dev, weights, BF)
    L.write_cache(kc, vc)
    k, v = L.cache_buffers()
    assert np.array_equal(bits(k), bits(bf16_np(kc)))
    assert np.array_equal(bits(v), bits(bf16_np(vc)))


@pytest.mark.parametrize("n_cache", [256, 8192])
def test_decode_over_preloaded_cache(dev, oracle, weights, n_cache):
    kc = synth.normal(402, f"k{n_cache}", n_cache * KVW)
    vc = synth.normal(402, f"v{n_cache}", n_cache * KVW)
    L = Layer.create(dev, weights, BF.with_(max_keys=n_cache + 8))
    L.write_cache(kc, vc)
    ref = _ref(oracle, weights, n_cache + 8)
    ref.fill_cache(kc, vc)
    for step in range(3):
        x = synth.normal(403, f"x{step}", S.hidden)
        got = L.forward(x)
        want = ref.forward(x, 1)
        assert abs_err_scaled(got, want) < 1e-5
    k, v = L.cache_buffers()
    rk, rv = ref.cache()
    assert L.n_keys == n_cache + 3
    assert np.array_equal(bits(k[:n_cache * KVW]), bits(rk[:n_cache * KVW]))
    assert np.array_equal(bits(v), bits(rv))
    assert n_mismatch(k[n_cache * KVW:], rk[n_cache * KVW:]) <= 2
    assert not np.any(bits(k) & 0xFFFF) and not np.any(bits(v) & 0xFFFF)


@pytest.mark.parametrize("n", [16, 130])
def test_tensor_prefill_bf16(dev, oracle, weights, n):
    x = synth.normal(404, f"p{n}", n * S.hidden).astype(np.float32)
    L = Layer.create(dev, weights, BF)
    L.encode_prefill(n, x)
    got = L.read_output(n)
    ref = _ref(oracle, weights)
    want = ref.forward(x, n)
    assert abs_err_scaled(got - x, want - x) <= 1e-2
    k, v = L.cache_buffers()
    rk, rv = ref.cache()
    assert abs_err_scaled(k, rk[:n * KVW]) <= 1e-2
    assert abs_err_scaled(v, rv[:n * KVW]) <= 1e-2
    assert not np.any(bits(k) & 0xFFFF) and not np.any(bits(v) & 0xFFFF)
    # then decode on the rows the prefill stored
    y = synth.normal(404, "dec", S.hidden).astype(np.float32)
    B = Layer.create(dev, weights, F32)
    B.encode_prefill(n, x)
    assert abs_err_scaled(L.forward(y) - y, B.forward(y) - y) <= 1e-2


def test_persistent_bit_identical_bf16(dev):
    m = synth.model(200, n_layers=2, vocab=4096)
    a = Model.create(dev, m, BF)
    b = Model.create(dev, m, BF)
    a.decode_mode = "persistent"
    assert a.decode_mode == "persistent" and b.decode_mode == "kernels"
    ids = synth.uniform_ids(7, "long", 1500, 4096).tolist()
    for M in (a, b):
        for i in range(0, 1500, 500):
            M.step(ids[i:i + 500])
    got = a.decode_device(12)
    want = b.decode_device(12)
    assert got.tolist() == want.tolist()
    la, lb = a.logits([int(got[-1])]), b.logits([int(want[-1])])
    assert np.array_equal(bits(la), bits(lb))


def test_model_bf16_close_to_f32(dev):
    m = synth.model(201, n_layers=2, vocab=4096)
    a = Model.create(dev, m, BF)
    b = Model.create(dev, m, F32)
    prompt = synth.uniform_ids(8, "prompt", 300, 4096).tolist()
    assert abs_err_scaled(a.logits(prompt), b.logits(prompt)) <= 1e-2
    for t in (5, 77, 4000):
        assert abs_err_scaled(a.logits([t]), b.logits([t])) <= 1e-2
    assert a.pos == b.pos == 303


@pytest.mark.parametrize("over", [dict(attention="exact"), dict(prefill="exact")])
def test_exact_kernels_refuse_bf16(dev, weights, over):
    with pytest.raises(FlockError) as e:
        Layer.create(dev, weights, BF.with_(**over))
    assert e.value.code == -8 and "bf16" in str(e.value)
