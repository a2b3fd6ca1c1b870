"""The CUDA path against the committed oracle fixtures
(tests/golden/oracle_pins.npz): the Q8_0 / Q4_0 matvecs bit for bit, and the
smoke scenario (2-layer Qwen3-0.6B-shape model, vocab 4096, 4-token prompt
and 3 greedy steps) with identical ids and bit-identical prefill logits."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden  # noqa: E402

from flock_b200 import lib as flib  # noqa: E402
from flock_b200 import ops, synth  # noqa: E402
from flock_b200.layer import QWEN3_06B  # noqa: E402
from flock_b200.model import Model  # noqa: E402
from gpu_util import n_mismatch  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def pins():
    return make_golden.load()


def test_matvecs_equal_pins(dev, pins):
    packed = synth.q8_tensor(1, "w1024x1024", 1024, 1024)
    w = flib.GpuTensor.from_packed(dev, packed, 1024, 1024)
    got = ops.matvec(dev, w, synth.normal(1, "x1024", 1024))
    assert n_mismatch(got, pins["q8_1024x1024"]) == 0
    packed = synth.q4_tensor(2, "w3072x1024", 3072, 1024)
    w = flib.GpuTensor.from_packed(dev, packed, 3072, 1024, flib.FLOCK_Q4_0)
    got = ops.matvec(dev, w, synth.normal(2, "x1024", 1024))
    assert n_mismatch(got, pins["q4_3072x1024"]) == 0


def test_smoke_scenario_equals_pins(dev, pins):
    m = synth.model(7, n_layers=2, vocab=4096)
    M = Model.create(dev, m, QWEN3_06B)
    ids = [M.step(make_golden.SMOKE_PROMPT)]
    for _ in range(3):
        ids.append(M.step([ids[-1]]))
    assert ids == pins["smoke_ids"].tolist()
    M.rewind(0)
    lg = M.logits(make_golden.SMOKE_PROMPT)
    assert n_mismatch(lg, pins["smoke_prefill_logits"]) == 0
