"""Writes tests/golden/oracle_pins.npz: regression fixtures from the oracle.

The reference (TypeScript + WGSL under Deno/WebGPU) cannot execute on these
machines, so no reference-produced vectors exist.  These fixtures are the
oracle's own outputs on seeded inputs (regenerated bit for bit from
flock_b200.synth): tests/test_golden.py checks that the oracle still
reproduces them and that the C-ABI host codecs match, and
tests/test_gpu_golden.py checks the CUDA path against them.  They pin the
restatement and the kernels against drift, not against the reference.

    python tests/golden/make_golden.py          # rewrite the fixtures
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PATH = os.path.join(HERE, "oracle_pins.npz")

SMOKE_PROMPT = [3, 1000, 4095, 7]
SMALL = dict(hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, ffn=512)


def bf16_bits_input() -> np.ndarray:
    rng = np.random.default_rng(21)
    return np.concatenate([rng.standard_normal(192).astype(np.float32),
                           (rng.standard_normal(64) * 1e-38).astype(np.float32)])


def compute() -> dict:
    import oracle
    from flock_b200 import synth

    out = {}
    # Q8_0 / Q4_0 matvec in the coop(64) order (the inputs of test_gpu_ops' cases)
    packed = synth.q8_tensor(1, "w1024x1024", 1024, 1024)
    out["q8_1024x1024"] = oracle.matmul_q8(packed, synth.normal(1, "x1024", 1024), 1024, 1024)
    packed = synth.q4_tensor(2, "w3072x1024", 3072, 1024)
    out["q4_3072x1024"] = oracle.matmul_q4(packed, synth.normal(2, "x1024", 1024), 3072, 1024)

    # the smoke scenario: 2-layer 0.6B-shape model, vocab 4096, IEEE-FMA mode
    s = synth.QWEN3_06B
    m = synth.model(7, n_layers=2, vocab=4096)
    cfg = dict(hidden=s.hidden, n_heads=s.n_heads, n_kv_heads=s.n_kv_heads,
               head_dim=s.head_dim, ffn=s.ffn)
    oracle.set_fma_mode(True)
    try:
        refs = [oracle.RefLayer(w, cfg, 64) for w in m.layers]

        def step(ids):
            h = oracle.embed(m.embd["packed"], ids, s.hidden)
            for L in refs:
                h = L.forward(h, len(ids))
            return oracle.head(h[(len(ids) - 1) * s.hidden:], m.output_norm, m.embd["packed"],
                               m.vocab, s.hidden)

        tok, _, logits = step(SMOKE_PROMPT)
        ids = [tok]
        for _ in range(3):
            ids.append(step([ids[-1]])[0])
    finally:
        oracle.set_fma_mode(False)
    out["smoke_prefill_logits"] = logits.astype(np.float32)
    out["smoke_ids"] = np.array(ids, np.int32)

    # three decode steps of a small layer (literal fma32 mode), and its cache
    w = synth.layer_weights(11, 0, synth.Shape(**SMALL))
    L = oracle.RefLayer(w, SMALL, 16)
    outs = [L.forward(synth.normal(12, f"s{i}", SMALL["hidden"]) * 0.5, 1) for i in range(3)]
    out["small_layer_decode"] = np.concatenate(outs)
    out["small_layer_k"], out["small_layer_v"] = L.cache()

    # FLK1 frame (wire.mjs pack) and bf16 rounding (the bf16 KV cache's)
    x = synth.normal(9, "wire", 1024) * 0.05
    out["wire_frame"] = np.frombuffer(oracle.wire_pack(x, seq=1, hidden=1024, offset=17,
                                                       reset=True), np.uint8).copy()
    xb = bf16_bits_input()
    lib = oracle.lib()
    out["bf16_round"] = np.array([lib.fo_bf16_round(float(v)) for v in xb], np.float32)
    return out


def load() -> dict:
    with np.load(PATH) as z:
        return {k: z[k] for k in z.files}


if __name__ == "__main__":
    np.savez_compressed(PATH, **compute())
    print(f"wrote {PATH} ({os.path.getsize(PATH)} bytes)")
