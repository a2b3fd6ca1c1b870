"""Prefill with the tcgen05 tensor-core matmuls (prefill="tensor") against the
reference's exact f32 prefill (layer_ref.ts / head_ref.ts attnPrefillRef
order on the oracle), within the tensor-core prefill bound: max relative error
1e-2 as absErrScaled (ops_ref.ts:206), on the layer output, on the layer's
own contribution (output - input), on the KV rows it appends, and on model
logits.  Single-token steps keep the exact path."""
import numpy as np
import pytest

from flock_b200 import lib as flib
from flock_b200 import synth
from flock_b200.layer import QWEN3_06B, Layer
from flock_b200.model import Model
from gpu_util import abs_err_scaled

pytestmark = pytest.mark.gpu

S = synth.QWEN3_06B
CFG = dict(hidden=S.hidden, n_heads=S.n_heads, n_kv_heads=S.n_kv_heads, head_dim=S.head_dim,
           ffn=S.ffn)
TENSOR = QWEN3_06B.with_(prefill="tensor")


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def weights():
    return synth.layer_weights(100, 24)


@pytest.mark.parametrize("n", [2, 16, 64, 200])
def test_tensor_prefill_layer(dev, oracle, weights, n):
    x = synth.normal(103, f"p{n}", n * S.hidden).astype(np.float32)
    L = Layer.create(dev, weights, TENSOR)
    L.encode_prefill(n, x)
    got = L.read_output(n)
    oracle.set_fma_mode(False)
    ref = oracle.RefLayer(weights, CFG, 4096)
    want = ref.forward(x, n)
    assert abs_err_scaled(got, want) <= 1e-2
    assert abs_err_scaled(got - x, want - x) <= 1e-2
    kc, vc = L.cache_buffers()
    kvw = S.n_kv_heads * S.head_dim
    rk, rv = ref.cache()
    assert abs_err_scaled(kc[:n * kvw], rk[:n * kvw]) <= 1e-2
    assert abs_err_scaled(vc[:n * kvw], rv[:n * kvw]) <= 1e-2


def test_tensor_prefill_then_exact_decode(dev, oracle, weights):
    """After a tensor-core prefill, single-token steps run the exact path."""
    n = 24
    x = synth.normal(104, "pre", n * S.hidden).astype(np.float32)
    A = Layer.create(dev, weights, TENSOR)
    B = Layer.create(dev, weights)
    A.encode_prefill(n, x)
    B.encode_prefill(n, x)
    y = synth.normal(104, "dec", S.hidden).astype(np.float32)
    ya, yb = A.forward(y), B.forward(y)
    assert abs_err_scaled(ya, yb) <= 1e-2
    assert A.n_keys == B.n_keys == n + 1


def test_tensor_prefill_model_logits(dev):
    m = synth.model(200, n_layers=2, vocab=4096)
    exact = Model.create(dev, m, QWEN3_06B)
    tc = Model.create(dev, m, TENSOR)
    prompt = synth.uniform_ids(5, "prompt", 100, 4096).tolist()
    le = exact.logits(prompt)
    lt = tc.logits(prompt)
    assert abs_err_scaled(lt, le) <= 1e-2
    assert exact.pos == tc.pos == 100


def test_tensor_prefill_chunks_past_max_prefill(dev):
    """model.ts:235 encodeTokens: prompts longer than maxPrefill run in chunks."""
    m = synth.model(201, n_layers=2, vocab=4096)
    cfg = TENSOR.with_(max_prefill=64)
    a = Model.create(dev, m, cfg)
    b = Model.create(dev, m, QWEN3_06B.with_(max_prefill=64))
    prompt = synth.uniform_ids(6, "long", 150, 4096).tolist()
    assert abs_err_scaled(a.logits(prompt), b.logits(prompt)) <= 1e-2
    assert a.pos == 150


def test_tensor_prefill_over_long_cache(dev, oracle, weights):
    """pos0 = 900: 130 queries over 1030 keys (two query tiles, nine key tiles)."""
    kvw = S.n_kv_heads * S.head_dim
    kc = synth.normal(105, "k900", 900 * kvw)
    vc = synth.normal(105, "v900", 900 * kvw)
    L = Layer.create(dev, weights, TENSOR)
    L.write_cache(kc, vc)
    oracle.set_fma_mode(False)
    ref = oracle.RefLayer(weights, CFG, 4096)
    ref.fill_cache(kc, vc)
    n = 130
    x = synth.normal(106, "p130", n * S.hidden).astype(np.float32)
    L.encode_prefill(n, x)
    got = L.read_output(n)
    want = ref.forward(x, n)
    assert abs_err_scaled(got - x, want - x) <= 1e-2
    assert L.n_keys == 1030
