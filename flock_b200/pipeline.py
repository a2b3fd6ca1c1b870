"""Layer-range pipeline across the GPUs of one box (kernels/model.ts:109
Model.create({cut}) + the bird layer ranges of web/bird.html:544-620 and
server/gguf.mjs:102 splitLayers), with the hidden state passed between
stages by NCCL send/recv (flock_pipeline_step) instead of the WebRTC hop.

stage_ranges() is the partition benchmark config 2 names: the first stage
(which also holds the embedding, output norm and head, as the reference's
coordinator does) takes `first` layers, the rest are split evenly with the
remainder going to the earlier stages.
"""
from __future__ import annotations


def stage_ranges(n_layers: int, world: int, first: int = 4) -> list[tuple[int, int]]:
    """[(start, end)) layer range per rank."""
    if n_layers < 1 or world < 1:
        raise ValueError("n_layers and world must be >= 1")
    if world > n_layers:
        raise ValueError(f"{world} stages for {n_layers} layers: every stage needs a layer")
    if world == 1:
        return [(0, n_layers)]
    first = max(1, min(first, n_layers - (world - 1)))
    rest = n_layers - first
    base, extra = divmod(rest, world - 1)
    out, at = [(0, first)], first
    for r in range(world - 1):
        c = base + (1 if r < extra else 0)
        out.append((at, at + c))
        at += c
    return out


def token_route(world: int) -> list[tuple[int, int]]:
    """The (sender, receiver) hops one token's hidden state takes: stage 0
    -> 1 -> ... -> last -> back to stage 0 for the head.  Every rank posts
    its receive before its send in this order, so the ring never deadlocks."""
    if world == 1:
        return []
    return [(r, r + 1) for r in range(world - 1)] + [(world - 1, 0)]
