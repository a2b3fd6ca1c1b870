"""GGUF files streamed into device planes (flock_gguf_load_tensor): a model
built from a file equals the model built from the same packed weights bit
for bit, at the default 4 MiB staging and at a staging size that splits
every row into its own flush; f16 norm gains are widened exactly."""
import numpy as np
import pytest

import gguf_writer as gw
from flock_b200 import lib as flib
from flock_b200 import ops, synth
from flock_b200.gguf import GGUFFile, model_from_gguf
from flock_b200.layer import QWEN3_06B
from flock_b200.model import Model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def small():
    return synth.model(41, n_layers=2, vocab=4096)


@pytest.mark.parametrize("staging", [4 << 20, 2000])
def test_model_from_gguf_equals_packed(dev, small, tmp_path, staging):
    p = str(tmp_path / "m.gguf")
    gw.write_model(p, small)
    a = model_from_gguf(dev, p, QWEN3_06B, staging=staging)
    b = Model.create(dev, small, QWEN3_06B)
    prompt = [3, 77, 4000, 12]
    la, lb = a.logits(prompt), b.logits(prompt)
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    assert a.generate([5], 4) == b.generate([5], 4)


def test_tensor_planes_and_f16_norms(dev, small, tmp_path):
    import copy
    p = str(tmp_path / "h.gguf")
    gw.write_model(p, small, f16_norms=True)
    g = GGUFFile(p)
    t = small.layers[0]["ffn_up.weight"]
    x = synth.normal(3, "x", t["cols"]).astype(np.float32)
    a = g.load_tensor(dev, "blk.0.ffn_up.weight", staging=777)
    b = flib.GpuTensor.from_packed(dev, t["packed"], t["rows"], t["cols"])
    ya, yb = ops.matvec(dev, a, x), ops.matvec(dev, b, x)
    assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32))
    # f16 gains widen exactly: the file's model equals one whose f32 gains
    # were rounded to f16 first
    r16 = lambda v: np.asarray(v, np.float32).astype(np.float16).astype(np.float32)  # noqa: E731
    m16 = copy.copy(small)
    m16.layers = [{k: (v if isinstance(v, dict) else r16(v)) for k, v in w.items()}
                  for w in small.layers]
    m16.output_norm = r16(small.output_norm)
    A = model_from_gguf(dev, p, QWEN3_06B)
    B = Model.create(dev, m16, QWEN3_06B)
    la, lb = A.logits([9, 8, 7]), B.logits([9, 8, 7])
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
