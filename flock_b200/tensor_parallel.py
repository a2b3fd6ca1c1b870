"""Tensor-parallel slicing of one Qwen3 model over the GPUs of a box.

The reference shards one Q8_0 matrix in two directions (kernels/shard.ts:214
ShardedMatvec.create): "row" shards split the output rows and concatenate,
"col" shards split the input columns (32-aligned) and sum the partial
products serially in shard order (shard_ref.ts:327 shardReduceRef).  A
tensor-parallel layer applies them the Megatron way:

* attn_q / attn_k / attn_v by output rows, whole heads per rank (the rank's
  KV heads and the query heads of their GQA groups), so q/k norm, RoPE, the
  KV cache and attention stay local;
* attn_output by the input columns of those heads ("col", partial sums);
* ffn_gate / ffn_up by output rows and ffn_down by the same input columns,
  cut by shardRanges(ffn, n, 32) (shard_ref.ts:97);
* the lm-head by vocab rows, shardRanges(vocab, n, 1), each rank's
  (value, index) maximum reduced by reduceShardArgmax (shard_ref.ts:437).

Norm gains and the embedding are whole on every rank.  The C side
(flock_model_create_tp) all-gathers the two partials per layer and sums them
in rank order, so a rank's o_proj / down results equal shardedColMatvecRef.
"""
from __future__ import annotations

import numpy as np

from .layer import LayerConfig

Q8_BLOCK = 34  # GGUF Q8_0 block: f16 scale + 32 int8


def shard_ranges(total: int, n: int, align: int = 1) -> list[tuple[int, int]]:
    """shard_ref.ts:97 shardRanges: n (start, count) pieces of `total`, each a
    multiple of `align`, the first total/align % n pieces one unit larger."""
    if n < 1:
        raise ValueError(f"n shards must be >= 1, got {n}")
    if total < 0 or align < 1 or total % align:
        raise ValueError(f"total {total} is not a non-negative multiple of align {align}")
    units = total // align
    if units < n:
        raise ValueError(f"cannot cut {total} into {n} shards aligned to {align}")
    base, extra = divmod(units, n)
    out, at = [], 0
    for i in range(n):
        c = (base + (1 if i < extra else 0)) * align
        out.append((at, c))
        at += c
    return out


def check_world(cfg: LayerConfig, world: int) -> None:
    if world < 1:
        raise ValueError(f"world {world} < 1")
    if cfg.n_heads % cfg.n_kv_heads:
        raise ValueError(f"n_heads {cfg.n_heads} is not a multiple of n_kv_heads {cfg.n_kv_heads}")
    if cfg.n_kv_heads % world:
        raise ValueError(f"{cfg.n_kv_heads} KV heads do not split evenly over {world} ranks")
    shard_ranges(cfg.ffn, world, 32)


def head_ranges(cfg: LayerConfig, world: int) -> list[tuple[int, int]]:
    """(first KV head, KV head count) per rank."""
    check_world(cfg, world)
    return shard_ranges(cfg.n_kv_heads, world, 1)


def local_config(cfg: LayerConfig, world: int) -> list[LayerConfig]:
    """Each rank's layer shape: its KV heads with their query groups, its
    share of ffn."""
    g = cfg.n_heads // cfg.n_kv_heads
    ffn = shard_ranges(cfg.ffn, world, 32)
    return [cfg.with_(n_heads=kc * g, n_kv_heads=kc, ffn=ffn[r][1])
            for r, (_, kc) in enumerate(head_ranges(cfg, world))]


def slice_rows(t: dict, start: int, count: int) -> dict:
    """Output rows [start, start+count) of a packed Q8_0 tensor."""
    rb = (t["cols"] // 32) * Q8_BLOCK
    p = np.asarray(t["packed"], np.uint8).reshape(t["rows"], rb)
    return {"rows": count, "cols": t["cols"],
            "packed": np.ascontiguousarray(p[start:start + count]).reshape(-1)}


def slice_cols(t: dict, start: int, count: int) -> dict:
    """Input columns [start, start+count) (multiples of 32) of a packed Q8_0
    tensor: whole blocks, so scales and quants are copied unchanged."""
    if start % 32 or count % 32:
        raise ValueError(f"column slice {start}+{count} is not 32-aligned")
    p = np.asarray(t["packed"], np.uint8).reshape(t["rows"], t["cols"] // 32, Q8_BLOCK)
    blk = p[:, start // 32:(start + count) // 32, :]
    return {"rows": t["rows"], "cols": count, "packed": np.ascontiguousarray(blk).reshape(-1)}


def slice_layer(w: dict, cfg: LayerConfig, rank: int, world: int) -> dict:
    """This rank's tensors of one layer (packed LayerWeights, layer.ts:59)."""
    k0, kc = head_ranges(cfg, world)[rank]
    g, hd = cfg.n_heads // cfg.n_kv_heads, cfg.head_dim
    f0, fc = shard_ranges(cfg.ffn, world, 32)[rank]
    out = dict(w)
    out["attn_q.weight"] = slice_rows(w["attn_q.weight"], k0 * g * hd, kc * g * hd)
    out["attn_k.weight"] = slice_rows(w["attn_k.weight"], k0 * hd, kc * hd)
    out["attn_v.weight"] = slice_rows(w["attn_v.weight"], k0 * hd, kc * hd)
    out["attn_output.weight"] = slice_cols(w["attn_output.weight"], k0 * g * hd, kc * g * hd)
    out["ffn_gate.weight"] = slice_rows(w["ffn_gate.weight"], f0, fc)
    out["ffn_up.weight"] = slice_rows(w["ffn_up.weight"], f0, fc)
    out["ffn_down.weight"] = slice_cols(w["ffn_down.weight"], f0, fc)
    return out


def slice_head(head: dict, rank: int, world: int) -> dict:
    """This rank's vocab rows of the lm-head (shardRanges(vocab, n, 1))."""
    s, c = shard_ranges(head["rows"], world, 1)[rank]
    return slice_rows(head, s, c)
