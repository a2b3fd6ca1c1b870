"""Tensor-parallel host logic on CPU: the shard ranges and weight slicing of
flock_b200.tensor_parallel against the oracle's shardRanges /
shardedColMatvecRef, and the whole per-token protocol of
flock_model_create_tp -- every rank runs its slice of a layer, the o_proj and
down partials are all-gathered (gloo, world size 2 and 4, 127.0.0.1) and
summed in rank order, the head's (value, index) maxima are reduced by
reduceShardArgmax -- with the oracle as the compute.  Every rank's hidden
states must equal the oracle's tensor-parallel layer (RefLayer(tp=N)) bit
for bit, and the ids the whole model's."""
import multiprocessing as mp
import socket

import numpy as np
import pytest

from flock_b200 import synth
from flock_b200.layer import QWEN3_06B
from flock_b200.tensor_parallel import (head_ranges, local_config, shard_ranges, slice_cols,
                                        slice_head, slice_layer, slice_rows)

CFG = dict(hidden=1024, n_heads=16, n_kv_heads=8, head_dim=128, ffn=3072)
PROMPT = [5, 99, 4000]
N_DECODE = 2


def test_shard_ranges_match_oracle(oracle):
    for total, n, align in [(151936, 8, 1), (3072, 3, 32), (12288, 8, 32), (4096, 5, 32),
                            (7, 7, 1), (100, 3, 1)]:
        assert shard_ranges(total, n, align) == [tuple(map(int, r)) for r in
                                                 oracle.shard_ranges(total, n, align)]
    with pytest.raises(ValueError):
        shard_ranges(64, 3, 32)
    with pytest.raises(ValueError):
        shard_ranges(100, 3, 32)


def test_slices_reassemble():
    t = {"rows": 96, "cols": 256, "packed": synth.q8_tensor(3, "t", 96, 256)}
    rows = [slice_rows(t, s, c)["packed"] for s, c in shard_ranges(96, 3)]
    assert np.array_equal(np.concatenate(rows), t["packed"])
    cols = [slice_cols(t, s, c)["packed"].reshape(96, -1) for s, c in shard_ranges(256, 4, 32)]
    assert np.array_equal(np.concatenate(cols, axis=1).reshape(-1), t["packed"])
    with pytest.raises(ValueError):
        slice_cols(t, 16, 32)


def test_local_config_shapes():
    for world in (1, 2, 4, 8):
        cs = local_config(QWEN3_06B, world)
        assert sum(c.n_kv_heads for c in cs) == 8 and sum(c.ffn for c in cs) == 3072
        assert all(c.n_heads == 2 * c.n_kv_heads and c.hidden == 1024 for c in cs)
    assert head_ranges(QWEN3_06B, 4) == [(0, 2), (2, 2), (4, 2), (6, 2)]
    with pytest.raises(ValueError):
        local_config(QWEN3_06B, 3)  # 8 KV heads over 3 ranks


def test_8b_shape_slices():
    """Config 4b's shape over 2 / 4 / 8 ranks: whole KV heads with their GQA
    groups, ffn cut in 32-aligned pieces, and the slices reassemble the layer."""
    s8 = synth.QWEN3_8B
    cfg = QWEN3_06B.with_(hidden=s8.hidden, n_heads=s8.n_heads, n_kv_heads=s8.n_kv_heads,
                          ffn=s8.ffn)
    for world in (2, 4, 8):
        cs = local_config(cfg, world)
        assert all(c.n_heads == 4 * c.n_kv_heads for c in cs)
        assert sum(c.n_kv_heads for c in cs) == 8 and sum(c.ffn for c in cs) == 12288
        assert all(c.ffn % 32 == 0 for c in cs)
    # reassembly on a small layer of the same head structure
    small = QWEN3_06B.with_(hidden=256, n_heads=8, n_kv_heads=2, head_dim=128, ffn=512)
    w = {}
    for name, (rows, cols) in {"attn_q.weight": (1024, 256), "attn_k.weight": (256, 256),
                               "attn_v.weight": (256, 256), "attn_output.weight": (256, 1024),
                               "ffn_gate.weight": (512, 256), "ffn_up.weight": (512, 256),
                               "ffn_down.weight": (256, 512)}.items():
        w[name] = {"rows": rows, "cols": cols, "packed": synth.q8_tensor(5, name, rows, cols)}
    parts = [slice_layer(w, small, r, 2) for r in range(2)]
    for name in ("attn_q.weight", "attn_k.weight", "attn_v.weight", "ffn_gate.weight",
                 "ffn_up.weight"):
        assert np.array_equal(np.concatenate([p[name]["packed"] for p in parts]), w[name]["packed"])
    for name in ("attn_output.weight", "ffn_down.weight"):
        rows = w[name]["rows"]
        glued = np.concatenate([p[name]["packed"].reshape(rows, -1) for p in parts], axis=1)
        assert np.array_equal(glued.reshape(-1), w[name]["packed"])


def test_col_slices_sum_to_sharded_matvec(oracle):
    """o_proj on two ranks: each rank's matvec of its column slice, summed in
    rank order == shardedColMatvecRef."""
    w = synth.layer_weights(7, 0, synth.QWEN3_06B)["attn_output.weight"]
    x = synth.normal(8, "x", 2048).astype(np.float32)
    parts = []
    for s, c in shard_ranges(2048, 2, 32):
        sl = slice_cols(w, s, c)
        parts.append(oracle.matmul_q8(sl["packed"], x[s:s + c], 1024, c))
    got = oracle.shard_reduce(np.stack(parts))
    want = oracle.sharded_col_matvec(w["packed"], x, 1024, 2048, 2)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_ref_layer_tp_is_close_to_whole(oracle):
    w = synth.layer_weights(9, 0, synth.QWEN3_06B)
    h = synth.normal(10, "h", 3 * 1024).astype(np.float32)
    a = oracle.RefLayer(w, CFG, 16)
    b = oracle.RefLayer(w, CFG, 16, tp=1)
    c = oracle.RefLayer(w, CFG, 16, tp=2)
    ya, yb, yc = a.forward(h, 3), b.forward(h, 3), c.forward(h, 3)
    assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32))
    assert np.max(np.abs(yc - ya)) <= 1e-5 * np.max(np.abs(ya))
    with pytest.raises(ValueError, match="shards"):
        oracle.RefLayer(w, CFG, 16, tp=200).forward(h, 3)


# ------------------------------------------------------------ gloo protocol

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _RankLayer:
    """One rank's slice of a layer, composed from oracle ops in
    layerPrefillRef order (layer_ref.ts:103); `reduce` sums partials."""

    def __init__(self, oracle, w, rank, world):
        self.o = oracle
        self.c = local_config(QWEN3_06B, world)[rank]
        self.w = slice_layer(w, QWEN3_06B, rank, world)
        self.inv = oracle.rope_inv_freq(128, 1e6)
        self.k = np.zeros(0, np.float32)
        self.v = np.zeros(0, np.float32)

    def forward(self, h, n, reduce):
        o, c, w = self.o, self.c, self.w
        H, hd, nH, nKV, F = 1024, 128, c.n_heads, c.n_kv_heads, c.ffn
        qw, kvw = nH * hd, nKV * hd
        pos0 = self.k.size // kvw
        nh = o.rmsnorm(h, w["attn_norm.weight"], H, n)
        q = o.matmul_q8_batched(w["attn_q.weight"]["packed"], nh, qw, H, n)
        k = o.matmul_q8_batched(w["attn_k.weight"]["packed"], nh, kvw, H, n)
        v = o.matmul_q8_batched(w["attn_v.weight"]["packed"], nh, kvw, H, n)
        qn = o.rmsnorm(q, w["attn_q_norm.weight"], hd, n * nH)
        kn = o.rmsnorm(k, w["attn_k_norm.weight"], hd, n * nKV)
        q = o.rope(qn, n, nH, hd, pos0, self.inv)
        k = o.rope(kn, n, nKV, hd, pos0, self.inv)
        self.k = np.concatenate([self.k, k])
        self.v = np.concatenate([self.v, v])
        if n == 1:
            att = o.attn(q, self.k, self.v, nH, nKV, hd, pos0 + 1)
        else:
            att = o.attn_prefill(q, self.k, self.v, nH, nKV, hd, n, pos0, 64, 128)
        part = o.matmul_q8_batched(w["attn_output.weight"]["packed"], att, H, qw, n)
        h2 = o.add(h, reduce(part))
        nh = o.rmsnorm(h2, w["ffn_norm.weight"], H, n)
        g = o.matmul_q8_batched(w["ffn_gate.weight"]["packed"], nh, F, H, n)
        u = o.matmul_q8_batched(w["ffn_up.weight"]["packed"], nh, F, H, n)
        part = o.matmul_q8_batched(w["ffn_down.weight"]["packed"], o.swiglu(g, u), H, F, n)
        return o.add(h2, reduce(part))


def _tp_worker(rank, world, port, q):
    import os
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        m = synth.model(200, n_layers=2, vocab=4096)
        layers = [_RankLayer(oracle, w, rank, world) for w in m.layers]
        hs = slice_head(m.embd, rank, world)
        off = shard_ranges(m.vocab, world, 1)[rank][0]

        def reduce(part):  # all-gather, then the serial sum in rank order
            got = [torch.empty(part.size, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(got, torch.from_numpy(np.ascontiguousarray(part, np.float32)))
            return oracle.shard_reduce(np.stack([g.numpy() for g in got]))

        ids, out, hidden = list(PROMPT), [], []
        for step in range(1 + N_DECODE):
            n = len(ids)
            h = oracle.embed(m.embd["packed"], ids, 1024)
            for L in layers:
                h = L.forward(h, n, reduce)
            hidden.append(h)
            last = h[(n - 1) * 1024:]
            normed = oracle.rmsnorm(last, m.output_norm, 1024, 1)
            lg = oracle.matmul_q8(hs["packed"], normed, hs["rows"], 1024)
            i = oracle.argmax(lg)
            vals = [torch.empty(1, dtype=torch.float32) for _ in range(world)]
            idx = [torch.empty(1, dtype=torch.int64) for _ in range(world)]
            dist.all_gather(vals, torch.tensor([lg[i]], dtype=torch.float32))
            dist.all_gather(idx, torch.tensor([i + off], dtype=torch.int64))
            tok = oracle.reduce_shard_argmax(np.array([v.item() for v in vals], np.float32),
                                             np.array([x.item() for x in idx], np.int64),
                                             np.zeros(world, np.int64))
            out.append(int(tok))
            ids = [int(tok)]
        q.put((rank, (out, hidden)))
    finally:
        dist.destroy_process_group()


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
            r, v = q.get(timeout=300)
            res[r] = v
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    return res


@pytest.mark.parametrize("world", [2, 4])
def test_tp_protocol(oracle, world):
    res = _run(_tp_worker, world)
    m = synth.model(200, n_layers=2, vocab=4096)
    layers = [oracle.RefLayer(w, CFG, 16, tp=world) for w in m.layers]
    ids, want, want_h = list(PROMPT), [], []
    for _ in range(1 + N_DECODE):
        n = len(ids)
        h = oracle.embed(m.embd["packed"], ids, 1024)
        for L in layers:
            h = L.forward(h, n)
        want_h.append(h)
        tok, _, _ = oracle.head(h[(n - 1) * 1024:], m.output_norm, m.embd["packed"], m.vocab, 1024)
        want.append(int(tok))
        ids = [int(tok)]
    for r in range(world):
        got, hidden = res[r]
        assert got == want
        for a, b in zip(hidden, want_h):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
