"""Seeded synthetic weights in GGUF Q8_0 / Q4_0 layout.

The reference benchmarks and tests real Qwen3 GGUF tensors fetched over HTTP
(kernels/real_weights.ts:37-154).  There is no network here, so every tensor
is generated from a seed with the shapes and value distributions of the
workload configurations:

* Q8_0 block: f16 scale = f16(|N(0, 0.02)| / 127), then 32 int8 uniform in
  [-127, 127] -- the 34-byte on-disk block (kernels/lib.ts:25-26).
* Q4_0 block: the same f16 scale, then 16 bytes of uniform nibbles; byte i
  holds weight i (low) and weight i+16 (high), value = scale * (q - 8)
  (kernels/lib.ts:57-63).
* norm gains 1 + N(0, 0.05) as f32; activations and KV entries N(0, 1) f32.

Each tensor draws from its own ``numpy.random.Generator(PCG64(seed, key))`` so
a tensor is reproducible on its own, independent of generation order.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import numpy as np

Q8_BLOCK, Q8_BYTES = 32, 34
Q4_BLOCK, Q4_BYTES = 32, 18


def _rng(seed: int, key: str) -> np.random.Generator:
    h = int.from_bytes(hashlib.sha256(key.encode()).digest()[:8], "little")
    return np.random.Generator(np.random.PCG64([int(seed) & 0xFFFFFFFFFFFFFFFF, h]))


def _scales_f16(rng: np.random.Generator, n_blocks: int) -> np.ndarray:
    d = np.abs(rng.standard_normal(n_blocks, dtype=np.float64) * 0.02) / 127.0
    # f32to16 (web/js/wire.mjs:309) rounds to f32 first, then RNE to f16.
    return d.astype(np.float32).astype(np.float16)


def q8_tensor(seed: int, key: str, rows: int, cols: int) -> np.ndarray:
    """rows x cols Q8_0 in the packed 34-byte layout, as flat uint8."""
    if cols % Q8_BLOCK:
        raise ValueError(f"cols {cols} must be a multiple of {Q8_BLOCK}")
    rng = _rng(seed, key)
    nb = rows * (cols // Q8_BLOCK)
    out = np.empty((nb, Q8_BYTES), np.uint8)
    out[:, 0:2] = _scales_f16(rng, nb).view(np.uint8).reshape(nb, 2)
    out[:, 2:] = rng.integers(-127, 128, size=(nb, 32), dtype=np.int8).view(np.uint8)
    return out.reshape(-1)


def q4_tensor(seed: int, key: str, rows: int, cols: int) -> np.ndarray:
    """rows x cols Q4_0 in the packed 18-byte layout, as flat uint8."""
    if cols % Q4_BLOCK:
        raise ValueError(f"cols {cols} must be a multiple of {Q4_BLOCK}")
    rng = _rng(seed, key)
    nb = rows * (cols // Q4_BLOCK)
    out = np.empty((nb, Q4_BYTES), np.uint8)
    out[:, 0:2] = _scales_f16(rng, nb).view(np.uint8).reshape(nb, 2)
    out[:, 2:] = rng.integers(0, 256, size=(nb, 16), dtype=np.uint8)
    return out.reshape(-1)


def gain(seed: int, key: str, n: int) -> np.ndarray:
    return (1.0 + _rng(seed, key).standard_normal(n) * 0.05).astype(np.float32)


def normal(seed: int, key: str, n: int) -> np.ndarray:
    return _rng(seed, key).standard_normal(n, dtype=np.float32)


def uniform_ids(seed: int, key: str, n: int, vocab: int) -> np.ndarray:
    return _rng(seed, key).integers(0, vocab, size=n, dtype=np.int32)


@dataclass(frozen=True)
class Shape:
    """A Qwen3-family decoder shape (kernels/layer.ts:87 LayerConfig + vocab)."""
    hidden: int = 1024
    n_heads: int = 16
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 3072
    vocab: int = 151936
    n_layers: int = 28
    eps: float = 9.999999974752427e-7
    rope_base: float = 1e6
    tied: bool = True


QWEN3_06B = Shape()
QWEN3_8B = Shape(hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128, ffn=12288,
                 vocab=151936, n_layers=36, tied=False)

Q8_TENSORS = ("attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
              "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight")
F32_TENSORS = ("attn_norm.weight", "attn_q_norm.weight", "attn_k_norm.weight", "ffn_norm.weight")


def tensor_shapes(s: Shape) -> dict:
    """(rows, cols) of each Q8_0 tensor of one layer; GGUF lists [cols, rows]."""
    q = s.n_heads * s.head_dim
    kv = s.n_kv_heads * s.head_dim
    return {
        "attn_q.weight": (q, s.hidden),
        "attn_k.weight": (kv, s.hidden),
        "attn_v.weight": (kv, s.hidden),
        "attn_output.weight": (s.hidden, q),
        "ffn_gate.weight": (s.ffn, s.hidden),
        "ffn_up.weight": (s.ffn, s.hidden),
        "ffn_down.weight": (s.hidden, s.ffn),
    }


def layer_weights(seed: int, layer: int, s: Shape = QWEN3_06B) -> dict:
    """One layer's tensors keyed by GGUF suffix (kernels/layer.ts:59 LayerWeights).

    Q8_0 tensors are ``{"rows", "cols", "packed"}``; norm gains are f32 arrays.
    """
    out: dict = {}
    for name, (rows, cols) in tensor_shapes(s).items():
        out[name] = {"rows": rows, "cols": cols,
                     "packed": q8_tensor(seed, f"blk.{layer}.{name}", rows, cols)}
    out["attn_norm.weight"] = gain(seed, f"blk.{layer}.attn_norm.weight", s.hidden)
    out["attn_q_norm.weight"] = gain(seed, f"blk.{layer}.attn_q_norm.weight", s.head_dim)
    out["attn_k_norm.weight"] = gain(seed, f"blk.{layer}.attn_k_norm.weight", s.head_dim)
    out["ffn_norm.weight"] = gain(seed, f"blk.{layer}.ffn_norm.weight", s.hidden)
    return out


@dataclass
class SynthModel:
    """kernels/real_weights.ts:154 RealModel, synthetic: layers + embd + output_norm."""
    shape: Shape
    layers: list
    embd: dict
    output_norm: np.ndarray
    output: dict | None = None  # untied lm-head (8B shape); None = tied to embd
    seed: int = 0
    meta: dict = field(default_factory=dict)

    @property
    def hidden(self) -> int:
        return self.shape.hidden

    @property
    def vocab(self) -> int:
        return int(self.embd["rows"])

    @property
    def n_layers(self) -> int:
        return len(self.layers)


class LazyLayers:
    """The layers of a synthetic model, each generated when it is indexed (the
    same bytes as layer_weights), so a loader that uploads or slices one layer
    at a time never holds the whole model in host memory."""

    def __init__(self, seed: int, s: Shape, n: int):
        self.seed, self.s, self.n = seed, s, n

    def __len__(self) -> int:
        return self.n

    def __getitem__(self, i: int) -> dict:
        if not -self.n <= i < self.n:
            raise IndexError(i)
        return layer_weights(self.seed, i % self.n, self.s)

    def __iter__(self):
        return (self[i] for i in range(self.n))


def model(seed: int, s: Shape = QWEN3_06B, n_layers: int | None = None,
          vocab: int | None = None, lazy: bool = False) -> SynthModel:
    """A whole synthetic model.  ``n_layers``/``vocab`` shrink it for tests;
    ``lazy`` generates each layer when it is read."""
    nl = s.n_layers if n_layers is None else n_layers
    V = s.vocab if vocab is None else vocab
    layers = LazyLayers(seed, s, nl) if lazy else [layer_weights(seed, i, s) for i in range(nl)]
    embd = {"rows": V, "cols": s.hidden, "packed": q8_tensor(seed, "token_embd.weight", V, s.hidden)}
    out = None
    if not s.tied:
        out = {"rows": V, "cols": s.hidden, "packed": q8_tensor(seed, "output.weight", V, s.hidden)}
    return SynthModel(shape=s, layers=layers, embd=embd,
                      output_norm=gain(seed, "output_norm.weight", s.hidden), output=out,
                      seed=seed)
