"""The tensor-parallel model (flock_model_create_tp) on the GPU.

* one rank (a 1-rank NCCL communicator): the exchange is a copy and the
  rank-order sum of one partial is the partial itself, so logits and ids are
  bit-identical to the single-GPU model, in every decode mode;
* two ranks on two GPUs (skipped with fewer): the o_proj / down partials are
  exchanged (NVLink peer memory for decode steps, or an NCCL all-gather) and
  summed in rank order and the head's maxima reduced, so the
  gathered logits equal the oracle's tensor-parallel model (RefLayer(tp=2),
  shardedColMatvecRef per projection) bit for bit, and the ids follow; the
  device-fed decode graph (NCCL inside the captured graph) gives the ids of
  the host-launched steps.
"""
import multiprocessing as mp

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PROMPT = [5, 99, 4000, 17, 3]
LONG = [(37 * i + 11) % 4096 for i in range(200)]
N_DECODE = 5
CFG = dict(hidden=1024, n_heads=16, n_kv_heads=8, head_dim=128, ffn=3072)


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _oracle_run(oracle, m, tp, prompt, n_decode):
    """Greedy ids and last logits of the oracle model with tp-shard layers."""
    oracle.set_fma_mode(True)
    try:
        layers = [oracle.RefLayer(w, CFG, 256, tp=tp) for w in m.layers]
        ids, out, lg = list(prompt), [], None
        for _ in range(1 + n_decode):
            n = len(ids)
            h = oracle.embed(m.embd["packed"], ids, 1024)
            for L in layers:
                h = L.forward(h, n)
            tok, _, lg = oracle.head(h[(n - 1) * 1024:], m.output_norm, m.embd["packed"], m.vocab,
                                     1024)
            out.append(int(tok))
            ids = [int(tok)]
    finally:
        oracle.set_fma_mode(False)
    return out, lg


def test_one_rank_equals_single_gpu_model():
    from flock_b200 import lib as flib
    from flock_b200 import synth
    from flock_b200.comm import Comm
    from flock_b200.layer import QWEN3_06B
    from flock_b200.model import Model
    dev = flib.get_device(0)
    m = synth.model(200, n_layers=2, vocab=4096)
    for attention in ("exact", "fast"):
        cfg = QWEN3_06B.with_(attention=attention)
        ref = Model.create(dev, m, cfg)
        T = Model.create_tp(dev, m, cfg, Comm(dev, 1, 0, Comm.unique_id()), 0, 1)
        assert T.decode_mode == "kernels"
        T.decode_mode = "persistent"  # not available with tensor parallelism
        assert T.decode_mode == "kernels"
        la, lb = ref.logits(PROMPT), T.logits(PROMPT)
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
        want = ref.decode_device(N_DECODE).tolist()
        assert T.decode_device(N_DECODE).tolist() == want
        T.decode_mode = "eager"
        assert T.decode_mode == "eager"
        nxt = [ref.step([want[-1]])]
        assert T.step([want[-1]]) == nxt[0]
        assert T.tp_exchange == "peer"
        T.tp_exchange = "nccl"
        assert T.tp_exchange == "nccl"
        assert T.step([nxt[0]]) == ref.step([nxt[0]])
        T.free()
        ref.free()


def test_one_rank_tensor_prefill_equals_single_gpu():
    """Tensor-core prefill with the o_proj / down partials stored and summed
    by the exchange: the same sum res + o as the residual epilogue."""
    from flock_b200 import lib as flib
    from flock_b200 import synth
    from flock_b200.comm import Comm
    from flock_b200.layer import QWEN3_06B
    from flock_b200.model import Model
    dev = flib.get_device(0)
    m = synth.model(200, n_layers=2, vocab=4096)
    cfg = QWEN3_06B.with_(prefill="tensor", attention="fast")
    ref = Model.create(dev, m, cfg)
    T = Model.create_tp(dev, m, cfg, Comm(dev, 1, 0, Comm.unique_id()), 0, 1)
    prompt = synth.uniform_ids(5, "tp", 200, 4096).tolist()
    la, lb = ref.logits(prompt), T.logits(prompt)
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))


def _rank(rank, world, q_uid, q_out):
    try:
        q_out.put((rank, _rank_body(rank, world, q_uid)))
    except Exception as e:  # report instead of leaving the parent waiting
        q_out.put((rank, f"rank {rank} failed: {e!r}"))


def _rank_body(rank, world, q_uid):
    from flock_b200 import lib as flib
    from flock_b200 import synth
    from flock_b200.comm import Comm
    from flock_b200.layer import QWEN3_06B
    from flock_b200.model import Model
    dev = flib.get_device(rank)
    m = synth.model(200, n_layers=2, vocab=4096)
    if rank == 0:
        uid = Comm.unique_id()
        for _ in range(world - 1):
            q_uid.put(uid)
    else:
        uid = q_uid.get(timeout=60)
    # one communicator per rank (a unique id bootstraps exactly one), shared
    # by the models built one after another
    comm = Comm(dev, world, rank, uid, 30000)
    res = {}
    for attention in ("exact", "fast"):
        M = Model.create_tp(dev, m, QWEN3_06B.with_(attention=attention), comm, rank, world)
        M.decode_mode = "eager"
        ids = [M.step(PROMPT)]
        for _ in range(N_DECODE - 1):
            ids.append(M.step([ids[-1]]))
        lg = M.logits([ids[-1]])
        M.reset()
        M.decode_mode = "kernels"
        graph = [M.step(PROMPT)] + M.decode_device(N_DECODE - 1).tolist()
        res[attention] = (ids, lg, graph)
        M.free()
    M = Model.create_tp(dev, m, QWEN3_06B.with_(prefill="tensor"), comm, rank, world)
    res["tensor_prefill"] = M.logits(LONG)
    M.free()
    # the two decode exchanges (NVLink peer memory, NCCL) give the same bits
    M = Model.create_tp(dev, m, QWEN3_06B.with_(attention="fast"), comm, rank, world)
    res["default_exchange"] = M.tp_exchange
    for mode in ("peer", "nccl"):
        M.tp_exchange = mode
        M.reset()
        ids = [M.step(PROMPT)] + M.decode_device(N_DECODE - 1).tolist()
        res[f"xchg_{mode}"] = (ids, M.logits([ids[-1]]))
    M.free()
    comm.free()
    return res


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_two_rank_tp_matches_oracle(oracle):
    from flock_b200 import synth
    ctx = mp.get_context("spawn")
    q_uid, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, q_uid, q_out)) for r in range(2)]
    res = {}
    try:
        for p in procs:
            p.start()
        for _ in range(2):
            r, v = q_out.get(timeout=600)
            res[r] = v
            assert not isinstance(v, str), v
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    m = synth.model(200, n_layers=2, vocab=4096)
    want, want_lg = _oracle_run(oracle, m, 2, PROMPT, N_DECODE)
    for attention in ("exact", "fast"):
        ids0, lg0, graph0 = res[0][attention]
        ids1, lg1, graph1 = res[1][attention]
        assert ids0 == ids1 == graph0 == graph1
        assert np.array_equal(lg0.view(np.uint32), lg1.view(np.uint32))
        if attention == "exact":
            assert ids0 + [int(np.argmax(lg0))] == want
            assert np.array_equal(lg0.view(np.uint32), want_lg.view(np.uint32))
        else:  # fast attention: 1e-5 relative tolerance per step
            assert ids0 == want[:N_DECODE]
    for r in (0, 1):
        assert res[r]["default_exchange"] == "peer"
        (ip, lp), (inc, lnc) = res[r]["xchg_peer"], res[r]["xchg_nccl"]
        assert ip == inc == res[0]["fast"][2]
        assert np.array_equal(lp.view(np.uint32), lnc.view(np.uint32))
    from gpu_util import abs_err_scaled
    _, want_long = _oracle_run(oracle, m, 2, LONG, 0)
    assert abs_err_scaled(res[0]["tensor_prefill"], want_long) <= 1e-2
    assert np.array_equal(res[0]["tensor_prefill"].view(np.uint32),
                          res[1]["tensor_prefill"].view(np.uint32))
