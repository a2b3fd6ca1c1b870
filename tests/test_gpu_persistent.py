"""The persistent decode kernel (one cooperative launch per token) against the
per-op kernel graph: same ids, bit-identical logits and hidden state, at
short and long contexts, on the toy and on the full Qwen3-0.6B shape.

Both engines run fast (split-K) attention; the per-op fast path is itself
checked against the oracle in test_gpu_model.py / test_gpu_layer.py."""
import numpy as np
import pytest

from flock_b200 import lib as flib
from flock_b200 import synth
from flock_b200.layer import QWEN3_06B
from flock_b200.model import Model

pytestmark = pytest.mark.gpu

FAST = QWEN3_06B.with_(attention="fast")


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def small():
    return synth.model(200, n_layers=2, vocab=4096)


def _pair(dev, m, cfg=FAST):
    a = Model.create(dev, m, cfg)
    b = Model.create(dev, m, cfg)
    assert b.decode_mode == "kernels"   # the default engine
    a.decode_mode = "persistent"
    assert a.decode_mode == "persistent"
    assert b.decode_mode == "kernels"
    return a, b


def _bits(x):
    return np.asarray(x, dtype=np.float32).view(np.uint32)


def test_persistent_logits_bit_identical(dev, small):
    a, b = _pair(dev, small)
    prompt = [5, 99, 4000, 17, 17, 3]
    ta, tb = a.step(prompt), b.step(prompt)
    assert ta == tb
    for _ in range(8):
        la, lb = a.logits([ta]), b.logits([tb])
        assert np.array_equal(_bits(la), _bits(lb))
        ta, tb = int(np.argmax(la)), int(np.argmax(lb))
        assert a.current_token() == ta
    assert a.pos == b.pos == len(prompt) + 8


def test_persistent_hidden_state_bit_identical(dev, small):
    a, b = _pair(dev, small)
    for M in (a, b):
        M.step([1, 2, 3])
        M.step([M.current_token()])
    # hidden_state runs through the per-op path; its input cache rows were
    # written by the persistent kernel in `a` and by the kernel graph in `b`
    ha = a.hidden_state([42])
    hb = b.hidden_state([42])
    assert np.array_equal(_bits(ha), _bits(hb))


def test_persistent_long_context(dev, small):
    """More keys than splits x 64, so every split streams several K/V tiles."""
    a, b = _pair(dev, small)
    ids = synth.uniform_ids(7, "long", 1500, 4096).tolist()
    for M in (a, b):
        for i in range(0, 1500, 500):
            M.step(ids[i:i + 500])
    got = a.decode_device(12)
    want = b.decode_device(12)
    assert got.tolist() == want.tolist()
    la, lb = a.logits([int(got[-1])]), b.logits([int(want[-1])])
    assert np.array_equal(_bits(la), _bits(lb))


def test_persistent_long_cache_splits(dev, small):
    """A cache of over 2048 keys: up to 64 splits, several per SM, which the
    persistent kernel's CTAs take in turn."""
    a, b = _pair(dev, small, FAST.with_(max_keys=4200, prefill="tensor"))
    ids = synth.uniform_ids(9, "long4k", 4000, 4096).tolist()
    for M in (a, b):
        for i in range(0, 4000, 500):
            M.step(ids[i:i + 500])
    got = a.decode_device(8)
    want = b.decode_device(8)
    assert got.tolist() == want.tolist()
    la, lb = a.logits([int(got[-1])]), b.logits([int(want[-1])])
    assert np.array_equal(_bits(la), _bits(lb))


def test_split_counts_bit_identical(dev, small):
    """Teacher-forced one-token steps from position 40 to 330 cross every
    decode-attention split count from 2 to 11 (one split per 32 keys; the
    first step right after a 40-token prompt, whose position the first layer
    advances by 40): every step's logits must be bit-identical between the
    kernel graph and the persistent kernel, which stage, split and combine
    the attention in their own launches."""
    a, b = _pair(dev, small)
    prompt = synth.uniform_ids(11, "ac-prompt", 40, 4096).tolist()
    forced = synth.uniform_ids(11, "ac-forced", 290, 4096).tolist()
    assert a.step(prompt) == b.step(prompt)
    for i, t in enumerate(forced):
        la, lb = a.logits([t]), b.logits([t])
        assert np.array_equal(_bits(la), _bits(lb)), f"position {40 + i}"
    assert a.pos == b.pos == 330


def test_engine_switches_around_multi_step_graphs(dev, small):
    """Device-fed runs of 8 or more steps launch the kernel graph's 8-step
    capture; switching the engine drops both captures and a later run
    captures them again, and freeing the model releases them.  Ids follow a
    model that stays on the persistent kernel, step for step."""
    a = Model.create(dev, small, FAST)
    ref = Model.create(dev, small, FAST)
    ref.decode_mode = "persistent"
    for M in (a, ref):
        M.step([4, 8, 15, 16, 23])
    got = a.decode_device(10).tolist()          # one 8-step launch + 2 single steps
    a.decode_mode = "persistent"
    got += a.decode_device(9).tolist()
    a.decode_mode = "kernels"
    got += a.decode_device(16).tolist()         # captured again
    got.append(a.step([got[-1]]))              # the one-step graph after the run graph
    want = ref.decode_device(35).tolist()
    want.append(ref.step([want[-1]]))
    assert got == want
    assert a.pos == ref.pos == 5 + 36
    a.free()
    ref.free()


def test_persistent_decode_device_history(dev, small):
    a, b = _pair(dev, small)
    for M in (a, b):
        M.step([9, 8, 7, 6])
    da, db = a.decode_device(20), b.decode_device(20)
    assert da.tolist() == db.tolist()
    assert a.pos == b.pos == 24


def test_mode_switch_mid_sequence(dev, small):
    a, b = _pair(dev, small)
    ref = Model.create(dev, small, FAST)
    ref.decode_mode = "persistent"
    for M in (a, b, ref):
        M.step([3, 1, 4, 1, 5])
    a.decode_device(3)
    b.decode_device(3)
    ref.decode_device(3)
    a.decode_mode, b.decode_mode = "kernels", "persistent"
    assert a.decode_device(5).tolist() == b.decode_device(5).tolist() == ref.decode_device(5).tolist()


def test_exact_attention_uses_kernel_graph(dev, small):
    M = Model.create(dev, small, QWEN3_06B)
    M.decode_mode = "persistent"
    assert M.decode_mode == "kernels"   # exact attention is not fused into the persistent kernel


def test_persistent_full_06b(dev):
    """The bench shape: 28 layers, 151936-row tied head."""
    m = synth.model(300)
    a, b = _pair(dev, m)
    prompt = synth.uniform_ids(300, "prompt", 64, synth.QWEN3_06B.vocab).tolist()
    ta, tb = a.step(prompt), b.step(prompt)
    assert ta == tb
    la, lb = a.logits([ta]), b.logits([tb])
    assert np.array_equal(_bits(la), _bits(lb))
    assert a.decode_device(16).tolist() == b.decode_device(16).tolist()


def test_phase_trace(dev, small):
    a, b = _pair(dev, small)
    for M in (a, b):
        M.step([2, 4, 6])
    a.trace(True)
    got = a.decode_device(3)
    tr = a.read_trace().astype(np.int64)
    a.trace(False)
    assert got.tolist() == b.decode_device(3).tolist()
    assert tr.shape[1] == 10 + 10 * a.held and tr.shape[0] % dev.sm_count == 0  # 1-2 CTAs per SM
    tr = tr[:, :4 + 10 * a.held]                      # the stamps
    assert (tr > 0).all()
    assert (np.diff(tr, axis=1) >= 0).all()          # stamps in program order per CTA
    # no CTA leaves a grid barrier before every CTA has reached it
    for c in range(3, tr.shape[1] - 2, 2):
        assert tr[:, c].min() >= tr[:, c - 1].max()
