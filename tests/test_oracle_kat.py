"""Pin the CPU oracle on the reference tests' own constructed known-answer cases.

The reference's tests draw their data from unseeded Math.random, so the only
fixed answers they hold are the constructed cases: planted maxima and ties,
planted RoPE inputs, the GQA head map, byte-preservation of the repack, the
shard planner's partition rules and capacity numbers.  Each test below cites
the reference test it restates.  CPU only.
"""
import math
import struct

import numpy as np
import pytest

from flock_b200 import synth

VOCAB = 151936


def test_split_q8_preserves_every_byte(oracle):
    # kernels/test_coop.ts:191-209
    rows, cols = 37, 1024
    w = np.random.default_rng(1).uniform(-0.05, 0.05, rows * cols).astype(np.float32)
    packed = oracle.quant_matrix_q8(w, rows, cols)
    qs, sc = oracle.split_q8(packed, rows, cols)
    nb = cols // 32
    p = packed.reshape(rows, nb, 34)
    assert np.array_equal(sc.reshape(rows, nb, 2), p[:, :, 0:2])
    assert np.array_equal(qs.reshape(rows, nb, 32), p[:, :, 2:])


def test_split_q4_preserves_every_byte(oracle):
    # kernels/lib.ts:142 -- same contract for the 18-byte layout
    rows, cols = 13, 256
    packed = synth.q4_tensor(3, "t", rows, cols)
    qs, sc = oracle.split_q4(packed, rows, cols)
    p = packed.reshape(rows * cols // 32, 18)
    assert np.array_equal(sc.reshape(-1, 2), p[:, 0:2])
    assert np.array_equal(qs.reshape(-1, 16), p[:, 2:])


def test_token_embd_repacked_size(oracle):
    # kernels/lib.ts:340-343: token_embd 151936 x 1024 repacks to a 155582464-byte qs plane
    plan = oracle.mem_shard_plan(VOCAB, 1024, 1, "row")
    assert plan["unsharded_max_binding_bytes"] == 155582464
    assert not plan["fits"]


def test_q4_nibble_mapping(oracle):
    # kernels/lib.ts:57-63 and :295-301: byte i = weight i (low) | weight i+16 (high)
    block = bytearray(18)
    block[0:2] = struct.pack("<H", 0x3C00)  # scale 1.0
    for i in range(16):
        lo, hi = i, 15 - i
        block[2 + i] = lo | (hi << 4)
    packed = np.frombuffer(bytes(block), np.uint8)
    for col in range(32):
        x = np.zeros(32, np.float32)
        x[col] = 1.0
        y = oracle.matmul_q4(packed, x, 1, 32)[0]
        want = (col - 8) if col < 16 else ((15 - (col - 16)) - 8)
        assert y == want, (col, y, want)


@pytest.mark.parametrize("at", [0, 1, 255, 256, 257, 151935, 75000])
def test_argmax_planted_max(oracle, at):
    # kernels/test_head.ts:208-215
    x = np.array([-1 - (i % 7) * 0.001 for i in range(VOCAB)], np.float32)
    x[at] = 5
    assert oracle.argmax(x) == at


def test_argmax_ties_lowest_index(oracle):
    # kernels/test_head.ts:219-230
    x = np.full(VOCAB, -1, np.float32)
    x[900] = x[40000] = x[151000] = 3
    assert oracle.argmax(x) == 900


def test_argmax_all_negative(oracle):
    # kernels/test_head.ts:246-256: largest = least negative = last index
    n = VOCAB
    x = np.array([-100 - (n - i) * 1e-3 for i in range(n)], np.float32)
    assert oracle.argmax(x) == n - 1


@pytest.mark.parametrize("neox", [True, False])
def test_rope_pairing_planted(oracle, neox):
    # kernels/test_ops.ts:229-263: x[0]=1, position 1; sine lands on the partner
    hd = 128
    inv = oracle.rope_inv_freq(hd, 1e6)
    x = np.zeros(hd, np.float32)
    x[0] = 1
    out = oracle.rope(x, 1, 1, hd, 1, inv, neox=neox)
    theta = float(inv[0])
    partner, other = (64, 1) if neox else (1, 64)
    assert abs(out[0] - math.cos(theta)) < 1e-6
    assert abs(out[partner] - math.sin(theta)) < 1e-6
    assert out[other] == 0


def test_gqa_head_map(oracle):
    # kernels/test_ops.ts:357-394: q head h reads kv head h / (nH/nKV)
    nH, nKV, hd = 4, 2, 128
    q = np.zeros(nH * hd, np.float32)
    k = np.zeros(nKV * hd, np.float32)
    v = np.concatenate([np.full(hd, 7, np.float32), np.full(hd, -3, np.float32)])
    out = oracle.attn(q, k, v, nH, nKV, hd, 1).reshape(nH, hd)
    for h, want in enumerate([7, 7, -3, -3]):
        assert np.all(out[h] == want)


def test_f32to16_known_values(oracle):
    # web/js/wire.mjs:309 -- RNE, overflow to inf, subnormals, signed zero
    cases = [(1.0, 0x3C00), (-2.0, 0xC000), (65504.0, 0x7BFF), (65520.0, 0x7C00),
             (1e10, 0x7C00), (0.0, 0x0000), (-0.0, 0x8000), (2.0 ** -24, 0x0001),
             (2.0 ** -25, 0x0000), (1.5 * 2.0 ** -25, 0x0001), (2.0 ** -14, 0x0400),
             (1.0 + 2.0 ** -11, 0x3C00), (1.0 + 3 * 2.0 ** -11, 0x3C02),
             (math.inf, 0x7C00), (-math.inf, 0xFC00)]
    for v, want in cases:
        assert oracle.f32to16(v) == want, (v, hex(oracle.f32to16(v)), hex(want))
    assert oracle.f32to16(float("nan")) & 0x7E00 == 0x7E00


def test_half_to_f32_clamps_inf(oracle):
    # kernels/lib.ts:33: kernels clamp inf to the largest finite f32
    assert oracle.half_to_f32(0x7C00) == 3.4028235e38
    assert oracle.half_to_f32(0x0001) == 2.0 ** -24
    assert oracle.half_to_f32(0x3C00) == 1.0


def test_shard_ranges_partition(oracle):
    # kernels/test_shard.ts:90-133 cases; exact partition, spread <= one unit
    cases = [(1024, 1, 32), (1024, 2, 32), (1024, 3, 32), (1024, 4, 32), (1024, 5, 32),
             (1024, 7, 32), (3072, 3, 32), (151936, 8, 1), (30, 4, 1)]
    for total, n, align in cases:
        rs = oracle.shard_ranges(total, n, align)
        assert len(rs) == n and rs[0][0] == 0 and sum(c for _, c in rs) == total
        for i in range(1, n):
            assert rs[i][0] == rs[i - 1][0] + rs[i - 1][1]
        counts = [c for _, c in rs]
        assert all(c % align == 0 and c > 0 for c in counts)
        assert max(counts) - min(counts) <= align


def test_shard_ranges_remainder_first(oracle):
    # kernels/shard_ref.ts:90-95: the remainder is spread over the FIRST shards, so
    # the largest is ceil(total / n).  (That docstring quotes 35476 for 248320 / 7;
    # its own formula gives 35475 = ceil(248320 / 7), which is what is asserted.)
    rs = oracle.shard_ranges(248320, 7, 1)
    assert [c for _, c in rs] == [35475, 35475] + [35474] * 5
    with pytest.raises(ValueError):
        oracle.shard_ranges(1024, 100, 32)  # test_shard.ts:142-153 "only 32 units"


def test_mem_shard_plan_14b_head(oracle):
    # kernels/test_shard_mem.ts:60-113 (Q6_K 210/256 bytes per weight, no scale plane)
    MiB = 1024 * 1024
    bpw = 210 / 256
    whole = oracle.mem_shard_plan(151936, 5120, 1, "row", 128 * MiB, bpw, 0)
    assert abs(whole["unsharded_max_binding_bytes"] / 1e6 - 638) < 5
    assert not whole["fits"]
    p8 = oracle.mem_shard_plan(151936, 5120, 8, "row", 128 * MiB, bpw, 0)
    assert p8["fits"] and p8["min_shards_for_limit"] <= 8
    c8 = oracle.mem_shard_plan(151936, 5120, 8, "col", 128 * MiB, bpw, 0)
    assert c8["fits"]
    assert abs(c8["max_binding_bytes"] - p8["max_binding_bytes"]) / p8["max_binding_bytes"] < 0.01


def test_mem_shard_plan_minimum_is_minimal(oracle):
    # kernels/test_shard_mem.ts:120-165
    MiB = 1024 * 1024
    tensors = [(151936, 1024, 1.0, 2.0), (151936, 5120, 210 / 256, 0.0), (248320, 5120, 1.0, 2.0)]
    for rows, cols, bpw, sbb in tensors:
        for lim in (64 * MiB, 128 * MiB, 256 * MiB, 1024 * MiB):
            n = oracle.mem_shard_plan(rows, cols, 1, "row", lim, bpw, sbb)["min_shards_for_limit"]
            assert n is not None
            assert oracle.mem_shard_plan(rows, cols, n, "row", lim, bpw, sbb)["fits"]
            if n > 1:
                assert not oracle.mem_shard_plan(rows, cols, n - 1, "row", lim, bpw, sbb)["fits"]


def _planted_head(vocab, hidden, rows):
    w = np.zeros(vocab * hidden, np.float32)
    for r in range(vocab):
        w[r * hidden] = 0.1 + (r % 17) * 0.01
    for r in rows:
        w[r * hidden] = 1.0
    return w


def test_sharded_argmax_ties_across_boundaries(oracle):
    # kernels/test_shard_head.ts:108-190
    vocab, hidden, n = 2048, 64, 4
    rg = oracle.shard_ranges(vocab, n, 1)
    start = [s for s, _ in rg]
    end = [s + c for s, c in rg]
    cases = [([start[1] + 5, start[3] + 9], start[1] + 5),
             ([start[0] + 1, end[3] - 1], start[0] + 1),
             ([start[2] + 3, start[2] + 400], start[2] + 3),
             ([end[1] - 1, start[2]], end[1] - 1)]
    x = np.zeros(hidden, np.float32)
    x[0] = 7.0
    for rows, want in cases:
        packed = oracle.quant_matrix_q8(_planted_head(vocab, hidden, rows), vocab, hidden)
        logits = oracle.sharded_row_matvec(packed, x, vocab, hidden, n)
        assert logits[rows[0]] == logits[rows[1]]
        assert oracle.argmax(logits) == want
        vals, idx, off = [], [], []
        for s, c in rg:
            part = logits[s:s + c]
            vals.append(part.max())
            idx.append(oracle.argmax(part))
            off.append(s)
        assert oracle.reduce_shard_argmax(vals, idx, off) == want


def test_row_shards_bit_identical(oracle):
    # kernels/test_shard.ts:244-280: output-split == unsharded, bit for bit
    rows, cols = 301, 1024
    packed = synth.q8_tensor(5, "w", rows, cols)
    x = synth.normal(5, "x", cols)
    full = oracle.matmul_q8(packed, x, rows, cols)
    for n in (1, 2, 3, 4, 7):
        assert np.array_equal(oracle.sharded_row_matvec(packed, x, rows, cols, n), full)


def test_col_shards_order_model(oracle):
    # kernels/test_shard.ts:282-346: input-split == its own order model; close to unsharded
    rows, cols = 64, 3072
    packed = synth.q8_tensor(6, "w", rows, cols)
    x = synth.normal(6, "x", cols)
    full = oracle.matmul_q8(packed, x, rows, cols)
    for n in (2, 3, 4):
        got = oracle.sharded_col_matvec(packed, x, rows, cols, n)
        rg = oracle.shard_ranges(cols, n, 32)
        parts = []
        for s, c in rg:
            sl = packed.reshape(rows, cols // 32, 34)[:, s // 32:(s + c) // 32].reshape(-1)
            parts.append(oracle.matmul_q8(sl, x[s:s + c], rows, c))
        assert np.array_equal(got, oracle.shard_reduce(np.stack(parts)))
        scale = np.abs(full).max()
        assert np.abs(got - full).max() / scale < 1e-5


def test_prefill_kv_cache_equals_decode(oracle):
    # kernels/test_prefill.ts:80-135: prefill leaves the SAME cache N decode steps write
    s = synth.Shape(hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, ffn=512)
    w = synth.layer_weights(7, 0, s)
    cfg = dict(hidden=s.hidden, n_heads=s.n_heads, n_kv_heads=s.n_kv_heads, head_dim=s.head_dim,
               ffn=s.ffn)
    n = 5
    x = synth.normal(7, "h", n * s.hidden) * 0.05
    A = oracle.RefLayer(w, cfg, 64)
    out_pre = A.forward(x, n)
    B = oracle.RefLayer(w, cfg, 64)
    outs = [B.forward(x[i * s.hidden:(i + 1) * s.hidden], 1) for i in range(n)]
    ka, va = A.cache()
    kb, vb = B.cache()
    assert np.array_equal(ka, kb) and np.array_equal(va, vb)
    dec = np.concatenate(outs)
    assert np.abs(out_pre - dec).max() / np.abs(dec).max() < 2e-6


def test_wire_roundtrip(oracle):
    # web/js/wire.mjs:344-371
    x = synth.normal(9, "wire", 1024) * 0.05
    buf = oracle.wire_pack(x, seq=3, hidden=1024, offset=17, reset=True)
    assert buf[:4] == b"FLK1" and len(buf) == 20 + 2048
    y, meta = oracle.wire_unpack(buf)
    assert meta == {"seq": 3, "hidden": 1024, "offset": 17, "reset": True, "replay": False}
    assert np.abs(y - x).max() <= np.abs(x).max() * 2 ** -11


def test_requant_noise_changes_weights(oracle):
    # kernels/dequant.ts:35-58: plain round trip is idempotent, the noisy one is not
    rows, cols = 8, 256
    w = synth.normal(2, "w", rows * cols) * 0.05
    packed = oracle.quant_matrix_q8(w, rows, cols)
    again = oracle.quant_matrix_q8(oracle.dequant_q8(packed, rows, cols), rows, cols)
    assert np.array_equal(again, packed)
    noisy, _ = oracle.requant_with_noise(packed, rows, cols, 1)
    assert not np.array_equal(noisy, packed)
