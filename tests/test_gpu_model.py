"""Whole-model greedy decode vs the oracle composed the way kernels/model.ts
wires it (embed -> layers -> output_norm -> tied head -> argmax), and the
coordinator split (kernels/test_split.ts)."""
import numpy as np
import pytest

from flock_b200 import lib as flib
from flock_b200 import synth
from flock_b200._abi import FlockError
from flock_b200.layer import QWEN3_06B, Layer, range_forward
from flock_b200.model import Model
from gpu_util import n_mismatch

pytestmark = pytest.mark.gpu

S = synth.QWEN3_06B
CFG = dict(hidden=S.hidden, n_heads=S.n_heads, n_kv_heads=S.n_kv_heads, head_dim=S.head_dim,
           ffn=S.ffn)


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


class OracleModel:
    """model.ts step() on the CPU oracle."""

    def __init__(self, oracle, m, ieee=False):
        self.o, self.m, self.ieee = oracle, m, ieee
        self.layers = [oracle.RefLayer(w, CFG, 4096) for w in m.layers]

    def step(self, ids):
        o = self.o
        o.set_fma_mode(self.ieee)
        try:
            n = len(ids)
            h = o.embed(self.m.embd["packed"], ids, S.hidden)
            for L in self.layers:
                h = L.forward(h, n)
            last = h[(n - 1) * S.hidden:]
            tok, normed, logits = o.head(last, self.m.output_norm, self.m.embd["packed"],
                                         self.m.vocab, S.hidden)
        finally:
            o.set_fma_mode(False)
        self.logits = logits
        return tok


@pytest.fixture(scope="module")
def small():
    return synth.model(200, n_layers=2, vocab=4096)


@pytest.mark.parametrize("mode", ["exact", "fast"])
def test_small_model_greedy_ids(dev, oracle, small, mode):
    M = Model.create(dev, small, QWEN3_06B.with_(attention=mode))
    ref = OracleModel(oracle, small, ieee=True)
    prompt = [5, 99, 4000, 17, 17, 3]
    got = [M.step(prompt)]
    want = [ref.step(prompt)]
    for _ in range(6):
        got.append(M.step([got[-1]]))
        want.append(ref.step([want[-1]]))
    assert got == want


def test_small_model_logits_exact(dev, oracle, small):
    M = Model.create(dev, small, QWEN3_06B)
    ref = OracleModel(oracle, small, ieee=True)
    prompt = [7, 8, 9, 10]
    lg = M.logits(prompt)
    ref.step(prompt)
    assert n_mismatch(lg, ref.logits) == 0
    assert int(np.argmax(lg)) == int(np.argmax(ref.logits))


def test_decode_device_matches_host_loop(dev, small):
    A = Model.create(dev, small)
    B = Model.create(dev, small)
    prompt = [1, 2, 3, 4, 5]
    first = A.step(prompt)
    assert B.step(prompt) == first
    host = [first]
    for _ in range(10):
        host.append(A.step([host[-1]]))
    dev_ids = B.decode_device(10)
    assert [first] + dev_ids.tolist() == host
    assert A.pos == B.pos == len(prompt) + 10


def test_coordinator_split_equals_whole(dev, small):
    # kernels/test_split.ts:42-195: cut model + layer range == whole model
    whole = Model.create(dev, small)
    coord = Model.create(dev, small, cut=1)
    bird = [Layer.create(dev, small.layers[1])]
    prompt = [11, 22, 33, 44]
    want = whole.generate(prompt, 6)
    got = []
    ids, offset = prompt, 0
    for _ in range(6):
        flat = coord.encode_partial(ids, offset)
        flat = range_forward(bird, flat, len(ids), offset)
        tok = coord.project_hidden(flat, len(ids))
        got.append(tok)
        offset += len(ids)
        ids = [tok]
    assert got == want
    with pytest.raises(FlockError, match="offset"):
        coord.encode_partial([1], 0)


def test_generate_eos_and_rewind(dev, small):
    M = Model.create(dev, small)
    out = M.generate([1, 2, 3], 5)
    assert len(out) == 5
    M.reset()
    assert M.pos == 0
    out2 = M.generate([1, 2, 3], 5, eos=[out[2]])
    assert out2 == out[:out.index(out[2])]


def test_objects_outlive_device_close(small):
    """Closing a device drops only the caller's reference: models and tensors
    made on it keep working and free cleanly afterwards."""
    d = flib.get_device(0)
    t = flib.GpuTensor.from_f32(d, np.ones(64, np.float32))
    M = Model.create(d, small)
    first = M.step([1, 2, 3])
    d.close()
    assert M.step([first]) >= 0
    M.free()
    t.free()


def test_full_06b_model_greedy_ids(dev, oracle):
    """benchmark config 2 shape (28 layers, vocab 151936, tied head), short run."""
    m = synth.model(300)
    M = Model.create(dev, m, QWEN3_06B)
    ref = OracleModel(oracle, m, ieee=False)
    prompt = synth.uniform_ids(300, "prompt", 8, S.vocab).tolist()
    got = [M.step(prompt)]
    want = [ref.step(prompt)]
    for _ in range(2):
        got.append(M.step([got[-1]]))
        want.append(ref.step([want[-1]]))
    assert got == want


S8 = synth.QWEN3_8B
CFG8 = dict(hidden=S8.hidden, n_heads=S8.n_heads, n_kv_heads=S8.n_kv_heads,
            head_dim=S8.head_dim, ffn=S8.ffn)


@pytest.fixture(scope="module")
def small8b():
    return synth.model(210, S8, n_layers=2, vocab=4096)


def _cfg8(**kw):
    from flock_b200.layer import LayerConfig
    return LayerConfig(hidden=S8.hidden, n_heads=S8.n_heads, n_kv_heads=S8.n_kv_heads,
                       head_dim=S8.head_dim, ffn=S8.ffn, **kw)


def test_8b_shape_greedy_ids(dev, oracle, small8b):
    """Config 4's layer shape (hidden 4096, GQA group 4, ffn 12288, untied
    head) on 2 layers: greedy ids equal the oracle's, exact attention."""
    m = small8b
    M = Model.create(dev, m, _cfg8())
    oracle.set_fma_mode(True)
    try:
        layers = [oracle.RefLayer(w, CFG8, 256) for w in m.layers]

        def ref_step(ids):
            n = len(ids)
            h = oracle.embed(m.embd["packed"], ids, S8.hidden)
            for L in layers:
                h = L.forward(h, n)
            tok, _, _ = oracle.head(h[(n - 1) * S8.hidden:], m.output_norm, m.output["packed"],
                                    m.vocab, S8.hidden)
            return int(tok)

        prompt = [5, 4000, 17, 123]
        got = [M.step(prompt)]
        want = [ref_step(prompt)]
        for _ in range(3):
            got.append(M.step([got[-1]]))
            want.append(ref_step([want[-1]]))
    finally:
        oracle.set_fma_mode(False)
    assert got == want


def test_8b_shape_persistent_equals_kernels(dev, small8b):
    """The persistent decode kernel at the 8B shape (K = 4096 / 12288 staging
    through shared memory, GQA group 4) is bit-identical to the kernel graph."""
    a = Model.create(dev, small8b, _cfg8(attention="fast"))
    b = Model.create(dev, small8b, _cfg8(attention="fast"))
    a.decode_mode = "persistent"
    if a.decode_mode != "persistent":
        pytest.skip("persistent kernel does not fit this shape")
    for M in (a, b):
        M.step([9, 8, 7, 6, 5])
    la, lb = a.logits([a.current_token()]), b.logits([b.current_token()])
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    assert a.decode_device(6).tolist() == b.decode_device(6).tolist()


def test_8b_shape_tensor_prefill(dev, small8b):
    """Tensor-core prefill at the 8B shape (K up to 12288) within 1e-2."""
    from gpu_util import abs_err_scaled
    a = Model.create(dev, small8b, _cfg8(prefill="tensor"))
    b = Model.create(dev, small8b, _cfg8())
    prompt = synth.uniform_ids(8, "p8", 300, 4096).tolist()
    assert abs_err_scaled(a.logits(prompt), b.logits(prompt)) <= 1e-2
