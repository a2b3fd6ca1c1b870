"""Product host-side logic against the oracle: quantizers (kernels/lib.ts:40-110)
and the shard planner (kernels/shard_ref.ts:97-567).  CPU only."""
import numpy as np
import pytest

from flock_b200 import lib as flib
from flock_b200 import shard, synth


@pytest.mark.parametrize("scale", [0.05, 1.0, 1e-7, 300.0])
def test_quant_q8_matches_reference(oracle, scale):
    rows, cols = 17, 256
    w = synth.normal(1, f"q8{scale}", rows * cols) * scale
    w[5] = 0.0
    w[64:96] = 0.0          # all-zero block
    w[100] = 127 * scale    # exact multiples / halves
    assert np.array_equal(flib.quant_matrix_q8(w, rows, cols), oracle.quant_matrix_q8(w, rows, cols))


@pytest.mark.parametrize("scale", [0.05, 1.0, 1e-7])
def test_quant_q4_matches_reference(oracle, scale):
    rows, cols = 13, 128
    w = synth.normal(2, f"q4{scale}", rows * cols) * scale
    w[32:64] = 0.0
    w[7] = 3 * scale  # equal magnitudes: the first one keeps its sign
    w[9] = -3 * scale
    assert np.array_equal(flib.quant_matrix_q4(w, rows, cols), oracle.quant_matrix_q4(w, rows, cols))


def test_half_to_f32(oracle):
    for h in [0, 1, 0x3C00, 0x7BFF, 0x7C00, 0xFC00, 0x7E01, 0x8001, 0x0400, 0x3555]:
        assert flib.half_to_f32(h) == oracle.half_to_f32(h)


@pytest.mark.parametrize("total,n,align", [(1024, 1, 32), (1024, 3, 32), (1024, 7, 32),
                                           (3072, 3, 32), (151936, 8, 1), (30, 4, 1),
                                           (248320, 7, 1)])
def test_shard_ranges_match(oracle, total, n, align):
    got = [(r.start, r.count) for r in shard.shard_ranges(total, n, align)]
    assert got == oracle.shard_ranges(total, n, align)


def test_shard_ranges_errors():
    with pytest.raises(ValueError, match="units"):
        shard.shard_ranges(1024, 100, 32)
    with pytest.raises(ValueError, match="multiple"):
        shard.shard_ranges(1000, 2, 32)
    with pytest.raises(ValueError, match="32"):
        shard.slice_cols(np.zeros(64, np.uint8), np.zeros(4, np.uint8), 1, 64, 0, 16)


@pytest.mark.parametrize("rows,cols,n,d,lim,bpw,sbb", [
    (151936, 1024, 1, "row", 128 << 20, 1.0, 2.0),
    (151936, 5120, 8, "row", 128 << 20, 210 / 256, 0.0),
    (151936, 5120, 8, "col", 128 << 20, 210 / 256, 0.0),
    (248320, 5120, 3, "row", 64 << 20, 1.0, 2.0),
])
def test_mem_shard_plan_matches(oracle, rows, cols, n, d, lim, bpw, sbb):
    a = shard.mem_shard_plan(rows, cols, n, d, lim, bpw, sbb)
    b = oracle.mem_shard_plan(rows, cols, n, d, lim, bpw, sbb)
    for k in ("max_binding_bytes", "unsharded_max_binding_bytes", "min_shards_for_limit", "fits"):
        assert a[k] == b[k], k


def test_slicers_reassemble(oracle):
    rows, cols = 37, 1024
    packed = synth.q8_tensor(3, "s", rows, cols)
    qs, sc = flib.split_q8(packed, rows, cols)
    parts = [shard.slice_cols(qs, sc, rows, cols, r.start, r.end)
             for r in shard.shard_ranges(cols, 3, 32)]
    q2 = np.concatenate([p[0].reshape(rows, -1) for p in parts], axis=1).reshape(-1)
    s2 = np.concatenate([p[1].reshape(rows, -1) for p in parts], axis=1).reshape(-1)
    assert np.array_equal(q2, qs) and np.array_equal(s2, sc)
    rparts = [shard.slice_rows(qs, sc, rows, cols, r.start, r.end)
              for r in shard.shard_ranges(rows, 4, 1)]
    assert np.array_equal(np.concatenate([p[0] for p in rparts]), qs)


def test_reduce_shard_argmax_ties():
    # shard_ref.ts:414-418: tie across shards -> lowest global index
    assert shard.reduce_shard_argmax([(3.0, 5, 0), (3.0, 1, 100)]) == 5
    assert shard.reduce_shard_argmax([(2.0, 5, 0), (3.0, 1, 100)]) == 101
    assert shard.reduce_shard_argmax([(3.0, 9, 200), (3.0, 5, 100)]) == 105
