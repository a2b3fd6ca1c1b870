"""GGUF loading on the host (flock_gguf_*): the directory parse
(gguf-dir.mjs readDirectory), metadata, the byte planner (gguf.mjs
byteRanges) and the incremental Q8_0 / Q4_0 split (gguf-stream.mjs
SplitStreamer), which must equal the whole-tensor split (lib.ts splitQ8 /
splitQ4) byte for byte at every read size, including sizes that cut blocks.
Malformed files are refused with an error, never read past their end."""
import os

import numpy as np
import pytest

import gguf_writer as gw
from flock_b200 import lib as flib
from flock_b200 import synth
from flock_b200._abi import FlockError
from flock_b200.gguf import GGML_F32, GGML_Q4_0, GGML_Q8_0, GGUFFile


@pytest.fixture(scope="module")
def small():
    return synth.model(31, n_layers=2, vocab=512)


@pytest.fixture(scope="module")
def path(tmp_path_factory, small):
    p = str(tmp_path_factory.mktemp("gguf") / "m.gguf")
    q4 = synth.q4_tensor(5, "q4", 48, 96)
    extra = [("general.name", gw.STR, "tiny"), ("x.flag", gw.BOOL, True),
             ("x.i64", gw.I64, -7), ("x.f64", gw.F64, 2.5), ("x.u8s", gw.ARR, (gw.U8, [1, 2, 3]))]
    tensors = _tensors_of(small) + [("extra.q4", [96, 48], 2, q4.tobytes())]
    meta = _meta_of(small, 64) + extra
    gw.write(p, meta, tensors, alignment=64)
    return p


def _meta_of(m, alignment):
    s = m.shape
    return [("general.architecture", gw.STR, "qwen3"), ("general.alignment", gw.U32, alignment),
            ("qwen3.block_count", gw.U32, len(m.layers)),
            ("qwen3.embedding_length", gw.U32, s.hidden),
            ("qwen3.attention.head_count", gw.U32, s.n_heads),
            ("qwen3.attention.head_count_kv", gw.U32, s.n_kv_heads),
            ("qwen3.attention.key_length", gw.U32, s.head_dim),
            ("qwen3.feed_forward_length", gw.U32, s.ffn),
            ("qwen3.attention.layer_norm_rms_epsilon", gw.F32, 1e-6),
            ("qwen3.rope.freq_base", gw.F32, 1e6),
            ("tokenizer.ggml.tokens", gw.ARR, (gw.STR, [f"t{i}" for i in range(8)]))]


def _tensors_of(m):
    ts = [("token_embd.weight", [m.embd["cols"], m.embd["rows"]], 8, m.embd["packed"].tobytes())]
    for i, w in enumerate(m.layers):
        for name, t in w.items():
            if isinstance(t, dict):
                ts.append((f"blk.{i}.{name}", [t["cols"], t["rows"]], 8, t["packed"].tobytes()))
            else:
                ts.append((f"blk.{i}.{name}", [len(t)], 0, np.asarray(t, np.float32).tobytes()))
    ts.append(("output_norm.weight", [m.hidden], 0, np.asarray(m.output_norm, np.float32).tobytes()))
    return ts


def test_directory(path, small):
    g = GGUFFile(path)
    assert g.version == 3 and g.n_layers == 2
    assert g.data_start % 64 == 0
    q = g.by_name["blk.1.attn_q.weight"]
    assert (q.dtype, q.rows, q.cols) == (GGML_Q8_0, 2048, 1024)
    assert q.bytes == 2048 * 1024 // 32 * 34
    n = g.by_name["blk.0.attn_norm.weight"]
    assert (n.dtype, n.rows, n.cols, n.bytes) == (GGML_F32, 1, 1024, 4096)
    e = g.by_name["extra.q4"]
    assert (e.dtype, e.rows, e.cols, e.bytes) == (GGML_Q4_0, 48, 96, 48 * 3 * 18)
    assert all(t.offset % 64 == 0 for t in g.tensors)
    assert len(g.tensors) == 1 + 2 * 11 + 1 + 1
    assert g.vocab == 512


def test_metadata(path):
    g = GGUFFile(path)
    assert g.meta_str("general.architecture") == "qwen3"
    assert g.meta_str("general.name") == "tiny"
    assert g.meta_int("x.flag") == 1 and g.meta_int("x.i64") == -7
    assert g.meta_float("x.f64") == 2.5
    assert g.meta_int("x.u8s") == 3 and g.meta_int("tokenizer.ggml.tokens") == 8
    assert abs(g.meta_float("qwen3.attention.layer_norm_rms_epsilon") - 1e-6) < 1e-12
    with pytest.raises(FlockError, match="no metadata key"):
        g.meta_int("nope")
    c = g.config()
    assert (c.hidden, c.n_heads, c.n_kv_heads, c.head_dim, c.ffn) == (1024, 16, 8, 128, 3072)
    assert c.rope_base == 1e6


def test_layer_ranges_match_byte_ranges(path):
    g = GGUFFile(path)

    def byte_ranges(first, last, gap):  # server/gguf.mjs:78, restated
        ts = sorted((g.data_start + t.offset, g.data_start + t.offset + t.bytes)
                    for t in g.tensors
                    if any(t.name.startswith(f"blk.{l}.") for l in range(first, last + 1)))
        out = []
        for s, e in ts:
            if out and s - out[-1][1] <= gap:
                out[-1][1] = max(out[-1][1], e)
            else:
                out.append([s, e])
        return [tuple(r) for r in out]

    for first, last, gap in [(0, 0, 1 << 20), (0, 1, 1 << 20), (1, 1, 0), (0, 1, 0)]:
        assert g.layer_ranges(first, last, gap) == byte_ranges(first, last, gap)
    assert len(g.layer_ranges(0, 1, 1 << 20)) == 1  # layers are contiguous


@pytest.mark.parametrize("chunk", [7, 34, 35, 1000, 4 << 20])
def test_incremental_split_equals_whole_split(path, small, chunk):
    g = GGUFFile(path)
    t = small.layers[1]["ffn_down.weight"]
    qs, sc = g.split_host("blk.1.ffn_down.weight", chunk)
    wq, ws = flib.split_q8(t["packed"], t["rows"], t["cols"])
    assert np.array_equal(qs, wq) and np.array_equal(sc, ws)
    q4 = synth.q4_tensor(5, "q4", 48, 96)
    qs, sc = g.split_host("extra.q4", chunk)
    wq, ws = flib.split_q4(q4, 48, 96)
    assert np.array_equal(qs, wq) and np.array_equal(sc, ws)


def test_split_refuses_unquantised_and_missing(path):
    g = GGUFFile(path)
    with pytest.raises(FlockError, match="neither Q8_0 nor Q4_0"):
        g.split_host("output_norm.weight")
    with pytest.raises(KeyError):
        g.split_host("blk.9.attn_q.weight")


def test_malformed_files_are_refused(path, tmp_path):
    raw = open(path, "rb").read()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + raw[4:])
    with pytest.raises(FlockError, match="not a GGUF file"):
        GGUFFile(str(bad))
    bad.write_bytes(raw[:200])  # cut inside the metadata
    with pytest.raises(FlockError):
        GGUFFile(str(bad))
    bad.write_bytes(raw[:len(raw) - 100])  # the last tensor runs past the end
    with pytest.raises(FlockError, match="past the end"):
        GGUFFile(str(bad))
    v = bytearray(raw)
    v[4:8] = (9).to_bytes(4, "little")
    bad.write_bytes(bytes(v))
    with pytest.raises(FlockError, match="version"):
        GGUFFile(str(bad))
    with pytest.raises(FlockError, match="cannot open"):
        GGUFFile(os.path.join(str(tmp_path), "missing.gguf"))
