"""Parity at exactly the configuration bench.py times (benchmark config 2):
the 28-layer Qwen3-0.6B-shaped Q8_0 model with the tied 151936 x 1024 head,
seed 0, split-K ("fast") decode attention, a 64-token prompt, then
device-fed greedy decode -- against the oracle's kernels/model.ts
composition (embed -> layers -> output_norm -> head -> argmax) on the same
seeded inputs.  Also config 3's tensor-core prefill of a 512-token prompt
against the exact f32 prefill.

Tolerances (north star): greedy ids identical token for token; logits within
max relative error 1e-3 for the f32 decode and 1e-2 for the f16 tensor-core
prefill.  Relative error is taken against max(|ref|, floor): for the f32
decode the floor is 1e-3 * max|ref| (logits that cross zero have no
meaningful relative error of their own); the f16 prefill's error is absolute
in nature (about 1e-3 of the logit scale, from the f16 operand rounding), so
its relative bar applies to the logits within 10x of the largest (floor
0.1 * max|ref|) and its absErrScaled must stay under 1e-2.
kernels/lib.ts:322 maxRelErr (floor 1e-6) and ops_ref.ts:206 absErrScaled
are printed beside them.

Random weights make the greedy continuation collapse onto one repeated token
after a few steps, so the decode path is also checked teacher-forced: a
fixed sequence of distinct tokens fed one decode step at a time, every
step's logits against the oracle's."""
import numpy as np
import pytest

from flock_b200 import lib as flib
from flock_b200 import synth
from flock_b200.layer import QWEN3_06B
from flock_b200.model import Model
from gpu_util import abs_err_scaled, rel_err

pytestmark = pytest.mark.gpu

S = synth.QWEN3_06B
CFG = dict(hidden=S.hidden, n_heads=S.n_heads, n_kv_heads=S.n_kv_heads, head_dim=S.head_dim,
           ffn=S.ffn)
SEED = 0          # bench.py's seed
PROMPT = 64       # bench.py's prompt length
N_DECODE = 32     # device-fed greedy tokens compared id for id


N_FORCED = 8      # teacher-forced decode steps


def bench_rel_err(got, want, floor_frac=1e-3) -> float:
    want = np.asarray(want, np.float64)
    return rel_err(got, want, floor=floor_frac * float(np.abs(want).max()))


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def model0():
    return synth.model(SEED)


@pytest.fixture(scope="module")
def oracle_run(oracle, model0):
    """The oracle's greedy run: logits after the prompt and after every
    decode token, and the ids."""
    m = model0
    layers = [oracle.RefLayer(w, CFG, PROMPT + N_DECODE + 8) for w in m.layers]
    prompt = synth.uniform_ids(SEED, "prompt", PROMPT, S.vocab).tolist()

    def step(ids):
        h = oracle.embed(m.embd["packed"], ids, S.hidden)
        for L in layers:
            h = L.forward(h, len(ids))
        tok, _, logits = oracle.head(h[(len(ids) - 1) * S.hidden:], m.output_norm,
                                     m.embd["packed"], m.vocab, S.hidden)
        return int(tok), np.array(logits, np.float32)

    ids, logits = [], []
    tok, lg = step(prompt)
    ids.append(tok)
    logits.append(lg)
    for _ in range(N_DECODE):
        tok, lg = step([ids[-1]])
        ids.append(tok)
        logits.append(lg)
    # teacher-forced: fresh caches, the prompt, then the forced tokens
    for L in layers:
        L.reset()
    step(prompt)
    forced = synth.uniform_ids(SEED, "forced", N_FORCED, S.vocab).tolist()
    forced_logits = [step([t])[1] for t in forced]
    return prompt, ids, logits, forced, forced_logits


@pytest.mark.parametrize("mode", ["kernels", "stream", "kernels+fast-matvec"])
def test_bench_config_greedy_ids_and_logits(dev, model0, oracle_run, mode):
    """'kernels+fast-matvec': the kernel graph with the LM head on the int8
    tensor cores (matvec="fast"), held to the same 1e-3 bar."""
    prompt, want_ids, want_logits, forced, forced_logits = oracle_run
    matvec = "fast" if mode.endswith("+fast-matvec") else "exact"
    mode = mode.split("+")[0]
    if mode not in Model._MODES:
        pytest.skip(f"decode mode {mode} is not built")
    M = Model.create(dev, model0, QWEN3_06B.with_(attention="fast", matvec=matvec,
                                                  max_keys=PROMPT + N_DECODE + 8))
    M.decode_mode = mode
    if M.decode_mode != mode:
        pytest.skip(f"decode mode {mode} unavailable for this shape")
    # prompt: the logits of its last position, then its greedy id
    lg0 = M.logits(prompt)
    first = int(np.argmax(lg0))
    assert first == want_ids[0]
    e0 = bench_rel_err(lg0, want_logits[0])
    print(f"prompt logits: rel {e0:.2e} (floor 1e-3*amax), maxRelErr "
          f"{rel_err(lg0, want_logits[0]):.2e}, absErrScaled "
          f"{abs_err_scaled(lg0, want_logits[0]):.2e}")
    assert e0 <= 1e-3
    # device-fed decode exactly as bench.py runs it
    got = M.decode_device(N_DECODE - 1).tolist()
    assert [first] + got == want_ids[:N_DECODE]
    # the last decode token's logits through the public API
    lgN = M.logits([got[-1]])
    assert int(np.argmax(lgN)) == want_ids[N_DECODE]
    eN = bench_rel_err(lgN, want_logits[N_DECODE])
    print(f"token {N_DECODE} logits: rel {eN:.2e}, maxRelErr "
          f"{rel_err(lgN, want_logits[N_DECODE]):.2e}, absErrScaled "
          f"{abs_err_scaled(lgN, want_logits[N_DECODE]):.2e}")
    assert eN <= 1e-3
    # teacher-forced decode steps from the prompt's cache
    M.rewind(PROMPT)
    worst = 0.0
    for t, want in zip(forced, forced_logits):
        lg = M.logits([t])
        assert int(np.argmax(lg)) == int(np.argmax(want))
        worst = max(worst, bench_rel_err(lg, want))
    print(f"{N_FORCED} forced steps: worst rel {worst:.2e}")
    assert worst <= 1e-3
    M.free()


def test_config3_tensor_prefill_first_token(dev, model0):
    """bench.py's config-3 line: the 512-token prompt through the tcgen05 f16
    prefill gives the exact f32 prefill's first id, logits within the f16
    bars above."""
    prompt = synth.uniform_ids(SEED, "prompt512", 512, S.vocab).tolist()
    cfg = QWEN3_06B.with_(attention="fast", max_keys=576, max_prefill=512)
    tc = Model.create(dev, model0, cfg.with_(prefill="tensor"))
    ex = Model.create(dev, model0, cfg)
    lt, le = tc.logits(prompt), ex.logits(prompt)
    assert int(np.argmax(lt)) == int(np.argmax(le))
    e = bench_rel_err(lt, le, floor_frac=0.1)
    a = abs_err_scaled(lt, le)
    print(f"512-token prefill logits: rel {e:.2e} (floor 0.1*amax), rel "
          f"{bench_rel_err(lt, le):.2e} (floor 1e-3*amax), absErrScaled {a:.2e}")
    assert e <= 1e-2
    assert a <= 1e-2
    tc.free()
    ex.free()
