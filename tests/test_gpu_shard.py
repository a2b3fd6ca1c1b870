"""Sharded matvec and sharded LM head on one device vs the reference's
shard_ref.ts order models (kernels/test_shard.ts, test_shard_head.ts,
test_shard_mem.ts)."""
import numpy as np
import pytest

from flock_b200 import lib as flib
from flock_b200 import ops, shard, synth
from flock_b200._abi import FlockError
from gpu_util import n_mismatch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


@pytest.mark.parametrize("n", [1, 2, 3, 4, 7])
def test_row_shards_bit_identical(dev, oracle, n):
    rows, cols = 301, 1024
    packed = synth.q8_tensor(20, "w", rows, cols)
    qs, sc = flib.split_q8(packed, rows, cols)
    x = synth.normal(20, "x", cols)
    sm = shard.ShardedMatvec.create(dev, qs, sc, rows, cols, n, "row")
    got = sm.run(x)
    full = ops.matvec(dev, flib.GpuTensor.from_split(dev, qs, sc, rows, cols), x)
    assert np.array_equal(got, full)
    assert n_mismatch(got, oracle.sharded_row_matvec(packed, x, rows, cols, n)) == 0


@pytest.mark.parametrize("rows,cols,n", [(64, 3072, 2), (64, 3072, 3), (1024, 3072, 4),
                                         (96, 1024, 7)])
def test_col_shards_match_order_model(dev, oracle, rows, cols, n):
    packed = synth.q8_tensor(21, "w", rows, cols)
    qs, sc = flib.split_q8(packed, rows, cols)
    x = synth.normal(21, "x", cols)
    sm = shard.ShardedMatvec.create(dev, qs, sc, rows, cols, n, "col")
    got = sm.run(x)
    assert n_mismatch(got, oracle.sharded_col_matvec(packed, x, rows, cols, n)) == 0
    parts = sm.partials()
    for rg, p in zip(sm.ranges, parts):
        sl = packed.reshape(rows, cols // 32, 34)[:, rg.start // 32:rg.end // 32].reshape(-1)
        assert n_mismatch(p, oracle.matmul_q8(sl, x[rg.start:rg.end], rows, rg.count)) == 0
    assert sm.wire_bytes_per_call() == n * rows * 4


def test_binding_limit_refused(dev):
    rows, cols = 4096, 1024
    packed = synth.q8_tensor(22, "w", rows, cols)
    qs, sc = flib.split_q8(packed, rows, cols)
    with pytest.raises(FlockError, match="limit"):
        shard.ShardedMatvec.create(dev, qs, sc, rows, cols, 2, "row", binding_limit=1 << 20)
    sm = shard.ShardedMatvec.create(dev, qs, sc, rows, cols, 4, "row", binding_limit=1 << 20)
    assert sm.run(np.ones(cols, np.float32)).shape == (rows,)


def _planted(vocab, hidden, rows):
    w = np.zeros(vocab * hidden, np.float32)
    w[np.arange(vocab) * hidden] = 0.1 + (np.arange(vocab) % 17) * 0.01
    for r in rows:
        w[r * hidden] = 1.0
    return w


def test_sharded_head_ties(dev):
    # kernels/test_shard_head.ts:108-190
    vocab, hidden, n = 2048, 64, 4
    rg = shard.shard_ranges(vocab, n, 1)
    cases = [([rg[1].start + 5, rg[3].start + 9], rg[1].start + 5),
             ([rg[0].start + 1, rg[3].end - 1], rg[0].start + 1),
             ([rg[2].start + 3, rg[2].start + 400], rg[2].start + 3),
             ([rg[1].end - 1, rg[2].start], rg[1].end - 1)]
    x = np.zeros(hidden, np.float32)
    x[0] = 7.0
    for rows, want in cases:
        packed = flib.quant_matrix_q8(_planted(vocab, hidden, rows), vocab, hidden)
        qs, sc = flib.split_q8(packed, vocab, hidden)
        head = shard.ShardedHead.create(dev, qs, sc, vocab, hidden, n)
        tok, logits = head.run(x)
        assert logits[rows[0]] == logits[rows[1]]
        assert tok == want
        assert shard.reduce_shard_argmax(head.argmax_buffers()) == want


def test_sharded_head_full_vocab(dev, oracle):
    # kernels/test_shard_head.ts: all 151936 logits bit-identical to unsharded
    vocab, hidden = 151936, 1024
    packed = synth.q8_tensor(23, "head", vocab, hidden)
    qs, sc = flib.split_q8(packed, vocab, hidden)
    x = synth.normal(23, "x", hidden)
    full = ops.matvec(dev, flib.GpuTensor.from_split(dev, qs, sc, vocab, hidden), x)
    for n in (2, 4, 8):
        head = shard.ShardedHead.create(dev, qs, sc, vocab, hidden, n)
        tok, logits = head.run(x)
        assert np.array_equal(logits, full)
        assert tok == oracle.argmax(full)
