"""The layer-range pipeline on two GPUs (flock_pipeline_step over NCCL
send/recv) against one GPU running the whole model: identical greedy ids,
for a prompt and for device-fed decode steps.  Needs 2 GPUs; skipped
otherwise.  Each rank is a spawned process bound to its own GPU."""
import multiprocessing as mp

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PROMPT = [11, 22, 33, 44, 55]
N_DECODE = 6


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _rank(rank, world, q_uid, q_out):
    import ctypes

    from flock_b200 import _abi, synth
    from flock_b200 import lib as flib
    from flock_b200.layer import QWEN3_06B, upload_layer
    from flock_b200.model import Model
    from flock_b200.pipeline import stage_ranges
    dev = flib.get_device(rank)
    m = synth.model(200, n_layers=4, vocab=4096)
    cfg = QWEN3_06B.with_(attention="fast")
    uid = np.zeros(128, np.uint8)
    if rank == 0:
        _abi.call("flock_comm_unique_id", _abi.ptr(uid, _abi._u8p))
        for _ in range(world - 1):
            q_uid.put(uid.tobytes())
    else:
        uid = np.frombuffer(q_uid.get(timeout=60), np.uint8).copy()
    comm = ctypes.c_void_p()
    _abi.call("flock_comm_init", dev.handle, world, rank, _abi.ptr(uid, _abi._u8p), 30000,
              ctypes.byref(comm))
    a, b = stage_ranges(4, world, first=1)[rank]
    lts = [upload_layer(dev, m.layers[i]) for i in range(a, b)]
    if rank == 0:
        embd = flib.GpuTensor.from_packed(dev, m.embd["packed"], m.embd["rows"], m.embd["cols"])
        onorm = flib.GpuTensor.from_f32(dev, m.output_norm)
        M = Model.from_tensors(dev, cfg, m.vocab, b - a, lts, embd, onorm)
    else:
        M = Model.from_tensors(dev, cfg, m.vocab, b - a, lts, None, None)
    nxt = ctypes.c_int32()
    ids = np.asarray(PROMPT, np.int32)
    _abi.call("flock_pipeline_step", M.handle, comm, _abi.ptr(ids, _abi._i32p) if rank == 0 else None,
              len(PROMPT), 1, ctypes.byref(nxt))
    out = [nxt.value]
    for _ in range(N_DECODE):  # device-fed: ids[0] carries the token to the next step
        _abi.call("flock_pipeline_step", M.handle, comm, None, 1, 1, ctypes.byref(nxt))
        out.append(nxt.value)
    if rank == 0:
        whole = Model.create(dev, m, cfg)
        want = [whole.step(PROMPT)]
        for _ in range(N_DECODE):
            want.append(whole.step([want[-1]]))
        q_out.put((0, out, want))
    else:
        q_out.put((rank, None, None))
    _abi.lib().flock_comm_free(comm)


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_two_gpu_pipeline_matches_one_gpu():
    ctx = mp.get_context("spawn")
    q_uid, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, q_uid, q_out)) for r in range(2)]
    res = {}
    try:
        for p in procs:
            p.start()
        for _ in range(2):
            r, got, want = q_out.get(timeout=300)
            res[r] = (got, want)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    got, want = res[0]
    assert got == want
