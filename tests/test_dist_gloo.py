"""The N > 1 path on CPU ranks over gloo (127.0.0.1, world size 2):

* the layer-range pipeline protocol of flock_pipeline_step -- stage 0 embeds
  and runs its layers, each stage receives the hidden state from the previous
  one, runs its range and sends it on, the last stage sends it back to stage
  0 for the head (kernels/test_split.ts: coordinator + bird == whole model) --
  with the oracle as the compute, so the pipelined greedy ids must equal the
  single-process ones exactly;
* a rank that leaves after the rendezvous: the survivor's receive ends in an
  error within the process group's timeout instead of hanging.
"""
import multiprocessing as mp
import socket

import numpy as np
import pytest

from flock_b200.pipeline import stage_ranges, token_route

CFG = dict(hidden=1024, n_heads=16, n_kv_heads=8, head_dim=128, ffn=3072)
PROMPT = [5, 99, 4000, 17]
N_DECODE = 3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _greedy_ids(m, layer_ranges, rank, world, send, recv):
    """One stage's part of PROMPT + N_DECODE greedy steps; rank 0 returns ids."""
    import oracle
    H = CFG["hidden"]
    a, b = layer_ranges[rank]
    layers = [oracle.RefLayer(m.layers[i], CFG, 64) for i in range(a, b)]
    ids, out = list(PROMPT), []
    for step in range(1 + N_DECODE):
        n = len(PROMPT) if step == 0 else 1
        if rank == 0:
            h = oracle.embed(m.embd["packed"], ids, H)
        else:
            h = recv(n * H, rank - 1)
        for L in layers:
            h = L.forward(h, n)
        if world > 1:
            send(h, (rank + 1) % world)
            if rank == 0:
                h = recv(n * H, world - 1)
        if rank == 0:
            tok, _, _ = oracle.head(h[(n - 1) * H:], m.output_norm, m.embd["packed"], m.vocab, H)
            out.append(int(tok))
            ids = [int(tok)]
    return out


def _pipeline_worker(rank, world, port, q):
    import os
    from datetime import timedelta

    import torch
    import torch.distributed as dist
    from flock_b200 import synth
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        m = synth.model(200, n_layers=3, vocab=4096)

        def send(h, dst):
            dist.send(torch.from_numpy(np.ascontiguousarray(h, np.float32)), dst=dst)

        def recv(n, src):
            t = torch.empty(n, dtype=torch.float32)
            dist.recv(t, src=src)
            return t.numpy()

        out = _greedy_ids(m, stage_ranges(3, world, first=1), rank, world, send, recv)
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def _leaver_worker(rank, world, port, q):
    import os
    import time
    from datetime import timedelta

    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    if rank == 1:
        q.put((1, "left"))
        q.close()
        q.join_thread()  # the item is sent before the process disappears
        os._exit(0)  # leaves between steps, nothing in flight
    t0 = time.time()
    try:
        # a bounded wait: a blocking recv would not notice the peer is gone
        dist.irecv(torch.empty(1024), src=1).wait(timeout=timedelta(seconds=3))
        q.put((0, "received?"))
    except Exception as e:  # the peer is gone: an error, not a hang
        q.put((0, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))
    q.close()
    q.join_thread()
    os._exit(0)


def _run(target, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    res = {}
    try:
        for p in procs:
            p.start()
        for _ in range(world):
            r, v = q.get(timeout=180)
            res[r] = v
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    return res


def test_stage_ranges():
    assert stage_ranges(28, 1) == [(0, 28)]
    assert stage_ranges(28, 2) == [(0, 4), (4, 28)]
    assert stage_ranges(28, 4) == [(0, 4), (4, 12), (12, 20), (20, 28)]
    # 24 layers over 7 stages: the remainder (3) goes to the earlier stages
    assert stage_ranges(28, 8) == [(0, 4), (4, 8), (8, 12), (12, 16), (16, 19), (19, 22),
                                   (22, 25), (25, 28)]
    assert stage_ranges(36, 8)[0] == (0, 4) and stage_ranges(36, 8)[-1][1] == 36
    for n, w in [(28, 3), (28, 5), (36, 7), (3, 3)]:
        r = stage_ranges(n, w)
        assert r[0][0] == 0 and r[-1][1] == n and all(b > a for a, b in r)
        assert all(r[i][1] == r[i + 1][0] for i in range(w - 1))
    with pytest.raises(ValueError):
        stage_ranges(2, 3)
    assert token_route(3) == [(0, 1), (1, 2), (2, 0)]


def test_pipeline_protocol_two_ranks_matches_one(oracle):
    from flock_b200 import synth
    m = synth.model(200, n_layers=3, vocab=4096)
    want = _greedy_ids(m, stage_ranges(3, 1), 0, 1, None, None)
    got = _run(_pipeline_worker, 2)
    assert got[0] == want
    assert got[1] == []


def test_rank_leaving_ends_in_error_not_hang():
    res = _run(_leaver_worker, 2)
    assert res[1] == "left"
    assert res[0].startswith("error after")
