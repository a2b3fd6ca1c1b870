"""A small GGUF (version 3) writer for the loader tests: typed metadata,
tensor records with dims fastest-first ([cols, rows]), each tensor's data at
an offset aligned to general.alignment inside the data section."""
from __future__ import annotations

import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
        BOOL: "<?", U64: "<Q", I64: "<q", F64: "<d"}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(t: int, v) -> bytes:
    if t == STR:
        return _str(v)
    if t == ARR:
        et, items = v
        out = struct.pack("<IQ", et, len(items))
        return out + b"".join(_value(et, x) for x in items)
    return struct.pack(_FMT[t], v)


def write(path: str, meta: list[tuple[str, int, object]], tensors: list[tuple[str, list[int], int,
                                                                          bytes]],
          alignment: int = 32, version: int = 3) -> None:
    """meta: (key, type, value); tensors: (name, dims fastest-first, ggml type, data)."""
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(meta))
    for k, t, v in meta:
        head += _str(k) + struct.pack("<I", t) + _value(t, v)
    offs, at = [], 0
    for _, _, _, data in tensors:
        at = (at + alignment - 1) // alignment * alignment
        offs.append(at)
        at += len(data)
    for (name, dims, t, _), off in zip(tensors, offs):
        head += _str(name) + struct.pack("<I", len(dims))
        head += b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", t, off)
    start = (len(head) + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(head + b"\0" * (start - len(head)))
        pos = 0
        for (_, _, _, data), off in zip(tensors, offs):
            f.write(b"\0" * (off - pos))
            f.write(data)
            pos = off + len(data)


def write_model(path: str, m, alignment: int = 32, f16_norms: bool = False,
                extra: list | None = None) -> None:
    """A synthetic Qwen3 model (flock_b200.synth) as a GGUF file."""
    s = m.shape
    meta = [("general.architecture", STR, "qwen3"), ("general.alignment", U32, alignment),
            ("qwen3.block_count", U32, len(m.layers)),
            ("qwen3.embedding_length", U32, s.hidden),
            ("qwen3.attention.head_count", U32, s.n_heads),
            ("qwen3.attention.head_count_kv", U32, s.n_kv_heads),
            ("qwen3.attention.key_length", U32, s.head_dim),
            ("qwen3.feed_forward_length", U32, s.ffn),
            ("qwen3.attention.layer_norm_rms_epsilon", F32, 1e-6),
            ("qwen3.rope.freq_base", F32, 1e6),
            ("tokenizer.ggml.tokens", ARR, (STR, [f"t{i}" for i in range(8)]))]
    meta += extra or []

    def norm(name, g):
        g = np.asarray(g, np.float32)
        if f16_norms:
            return (name, [g.size], 1, g.astype(np.float16).tobytes())
        return (name, [g.size], 0, g.tobytes())

    ts = [("token_embd.weight", [m.embd["cols"], m.embd["rows"]], 8, m.embd["packed"].tobytes())]
    for i, w in enumerate(m.layers):
        for name, t in w.items():
            if isinstance(t, dict):
                ts.append((f"blk.{i}.{name}", [t["cols"], t["rows"]], 8, t["packed"].tobytes()))
            else:
                ts.append(norm(f"blk.{i}.{name}", t))
    ts.append(norm("output_norm.weight", m.output_norm))
    if m.output is not None:
        ts.append(("output.weight", [m.output["cols"], m.output["rows"]], 8,
                   m.output["packed"].tobytes()))
    write(path, meta, ts, alignment)
