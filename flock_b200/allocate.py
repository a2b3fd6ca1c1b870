"""Which layers each GPU holds -- server/allocate.js on one box.

A pipeline runs at the pace of its slowest stage, so the layer ranges are
chosen to minimise the makespan: max over devices of (bytes held / measured
bytes per ms + time the device already owes per token), with every device's
layers contiguous and in chain order.  Layers are weighed in bytes, not in
count, and two limits are checked before any weight moves: the largest
single tensor a device can bind and its total weight budget.

* ``allocate`` (allocate.js:113): the exact contiguous partition by dynamic
  programming over (device, first layer), with the reference's feasibility
  checks and their failure kinds (empty, too-many-devices, tensor, budget,
  contiguity) raised as ``Infeasible``.
* ``adjust`` (allocate.js:341): a membership change as the smallest edit --
  a departed device's run goes to its neighbours, a newcomer takes a prefix
  or suffix of one incumbent -- ranking candidates by their sorted stage
  times; falls back to ``allocate`` when no local edit fits.
* ``layer_plan`` (allocate.js:38) reads layer sizes from a GGUF directory or
  a synthetic model; ``measure_rate`` gives a GPU's bytes per ms from a timed
  Q8_0 matvec, the measurement the pipeline feeds in.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

# allocate.js:56 -- a device with no measurement yet starts at the slower
# measured rate (4 Qwen3-0.6B layers, 16.8 MB, in 15.4 ms).
DEFAULT_RATE = 16.8e6 / 15.4
INF = math.inf


@dataclass
class LayerInfo:
    layer: int
    bytes: int
    max_tensor: int
    biggest: str = ""


@dataclass
class Device:
    """allocate.js:73 device(): bind = largest tensor it can hold, budget =
    weight bytes it will hold, rate = bytes per ms, reserved_ms = per-token
    time it already owes (rank 0's embedding and head)."""
    id: str
    label: str = "?"
    bind: float = INF
    budget: float = INF
    rate: float = DEFAULT_RATE
    reserved_ms: float = 0.0

    def __post_init__(self):
        self.bind = self.bind or INF
        self.budget = self.budget or INF
        self.rate = self.rate if self.rate and self.rate > 0 else DEFAULT_RATE
        self.reserved_ms = self.reserved_ms if self.reserved_ms > 0 else 0.0


class Infeasible(ValueError):
    def __init__(self, message: str, detail: dict):
        super().__init__(message)
        self.detail = detail


def _mb(n: float) -> str:
    return "unlimited" if n == INF else f"{n / 1e6:.1f}MB"


@dataclass
class Assignment:
    id: str
    label: str
    start: int
    end: int
    layers: int
    bytes: int
    rate: float
    ms: float
    share: float


@dataclass
class Allocation:
    assign: list[Assignment]
    makespan_ms: float
    total_bytes: int
    even_ms: float
    sticky: bool | None = None
    extra: dict = field(default_factory=dict)

    def ranges(self) -> list[tuple[int, int]]:
        """[(first, last + 1)) per device, in chain order."""
        return [(a.start, a.end + 1) for a in self.assign]


def layer_plan(source, first: int = 0, last: int | None = None) -> list[LayerInfo]:
    """Each layer's total bytes and its largest tensor: from a GGUFFile's
    directory or a synthetic model (packed Q8_0 sizes; norm gains 4 B/f32)."""
    out = []
    if hasattr(source, "tensors") and hasattr(source, "by_name"):  # GGUFFile
        n = source.n_layers if last is None else last + 1
        for i in range(first, n):
            ts = [t for t in source.tensors if t.name.startswith(f"blk.{i}.")]
            if not ts:
                raise ValueError(f"model has no tensors for layer {i}")
            big = max(ts, key=lambda t: t.bytes)
            out.append(LayerInfo(i, sum(t.bytes for t in ts), big.bytes, big.name))
        return out
    n = len(source.layers) if last is None else last + 1
    for i in range(first, n):
        w = source.layers[i]
        sizes = {k: (len(v["packed"]) if isinstance(v, dict) else 4 * len(v)) for k, v in w.items()}
        big = max(sizes, key=sizes.get)
        out.append(LayerInfo(i, sum(sizes.values()), sizes[big], f"blk.{i}.{big}"))
    return out


def _even_ms(layers: list[LayerInfo], devices: list[Device]) -> float:
    D, L = len(devices), len(layers)
    prefix = [0]
    for l in layers:
        prefix.append(prefix[-1] + l.bytes)
    per, extra = divmod(L, D)
    worst, at = 0.0, 0
    for d in range(D):
        k = per + (1 if d < extra else 0)
        worst = max(worst, (prefix[at + k] - prefix[at]) / devices[d].rate)
        at += k
    return round(worst, 2)


def _check_counts(layers, devices):
    D, L = len(devices), len(layers)
    if not D:
        raise Infeasible("no devices in the flock", {"kind": "empty"})
    if L < D:
        raise Infeasible(
            f"{D} devices but only {L} layer(s) to give out: {D - L} device(s) would hold "
            f"nothing. Give the stages more layers or use fewer devices.",
            {"kind": "too-many-devices", "devices": D, "layers": L})


def allocate(layers: list[LayerInfo], devices: list[Device]) -> Allocation:
    """allocate.js:113 -- exact minimum-makespan contiguous partition."""
    _check_counts(layers, devices)
    D, L = len(devices), len(layers)
    for l in layers:
        if any(l.max_tensor <= d.bind for d in devices):
            continue
        best = max(devices, key=lambda d: d.bind)
        raise Infeasible(
            f"no device can hold layer {l.layer}: its largest tensor {l.biggest} is "
            f"{_mb(l.max_tensor)}, and the roomiest device ({best.label}) allows "
            f"{_mb(best.bind)} per tensor. One tensor cannot be split across devices, so "
            f"adding more devices will not help.",
            {"kind": "tensor", "layer": l.layer, "tensor": l.biggest, "needs": l.max_tensor,
             "has": best.bind, "device": best.id})
    total = sum(l.bytes for l in layers)
    budget = sum(d.budget for d in devices)
    if total > budget:
        raise Infeasible(
            f"the flock is {_mb(total - budget)} short: layers {layers[0].layer}-"
            f"{layers[-1].layer} are {_mb(total)} of weights but the {D} device(s) together "
            f"budget only {_mb(budget)}.",
            {"kind": "budget", "needs": total, "has": budget})

    # best[d][i]: smallest makespan for layers i.. on devices d..; cut[d][i]:
    # the last layer index device d takes in that optimum.
    best = [[INF] * (L + 1) for _ in range(D + 1)]
    cut = [[-1] * (L + 1) for _ in range(D + 1)]
    best[D][L] = 0.0
    for d in range(D - 1, -1, -1):
        dev = devices[d]
        room = D - 1 - d  # layers left for the devices after d
        for i in range(0, L - room):
            held = 0
            for j in range(i, L - room):
                layer = layers[j]
                if layer.max_tensor > dev.bind:
                    break
                held += layer.bytes
                if held > dev.budget:
                    break
                tail = best[d + 1][j + 1]
                if tail == INF:
                    continue
                span = max(held / dev.rate + dev.reserved_ms, tail)
                if span < best[d][i]:
                    best[d][i] = span
                    cut[d][i] = j
    if best[0][0] == INF:
        tight = min(devices, key=lambda d: d.bind)
        blocked = [l.layer for l in layers if l.max_tensor > tight.bind]
        what = f"layer(s) {', '.join(map(str, blocked))}" if blocked else "enough layers"
        raise Infeasible(
            f"no contiguous assignment fits: each device's layers must stay in order, and "
            f"{tight.label} ({_mb(tight.bind)} per tensor"
            f"{'' if tight.budget == INF else ', ' + _mb(tight.budget) + ' budget'}) cannot take "
            f"{what} from the position it holds in the chain.",
            {"kind": "contiguity", "device": tight.id, "blocked": blocked})
    assign, i = [], 0
    for d in range(D):
        end = cut[d][i]
        run = layers[i:end + 1]
        b = sum(l.bytes for l in run)
        dev = devices[d]
        assign.append(Assignment(dev.id, dev.label, run[0].layer, run[-1].layer, len(run), b,
                                 dev.rate, round(b / dev.rate, 2), round(b / total, 4)))
        i = end + 1
    return Allocation(assign, round(best[0][0], 2), total, _even_ms(layers, devices))


def _stage_ms(d: Device, b: float) -> float:
    return b / d.rate + d.reserved_ms


def _fits(d: Device, run: list[LayerInfo]) -> bool:
    b = 0
    for l in run:
        if l.max_tensor > d.bind:
            return False
        b += l.bytes
    return b <= d.budget


def _chain_cost(layers, by_id, chain) -> list[float]:
    out = []
    for c in chain:
        b = sum(l.bytes for l in layers if c["start"] <= l.layer <= c["end"])
        out.append(_stage_ms(by_id[c["id"]], b))
    return sorted(out, reverse=True)


def _describe(layers, devices, chain) -> Allocation:
    by_id = {d.id: d for d in devices}
    total = sum(l.bytes for l in layers)
    makespan, assign = 0.0, []
    for c in sorted(chain, key=lambda c: c["start"]):
        d = by_id[c["id"]]
        run = [l for l in layers if c["start"] <= l.layer <= c["end"]]
        b = sum(l.bytes for l in run)
        makespan = max(makespan, _stage_ms(d, b))
        assign.append(Assignment(d.id, d.label, c["start"], c["end"], len(run), b, d.rate,
                                 round(b / d.rate, 2), round(b / total, 4)))
    return Allocation(assign, round(makespan, 2), total,
                      _even_ms(layers, [by_id[a.id] for a in assign]))


def adjust(layers: list[LayerInfo], current: list[dict], devices: list[Device]) -> Allocation:
    """allocate.js:341 -- apply a membership change with the fewest moves.
    `current`: [{"id", "start", "end"}] as placed now (ids missing from
    `devices` have left); devices not in `current` are newcomers."""
    _check_counts(layers, devices)
    by_id = {d.id: d for d in devices}
    first, last = layers[0].layer, layers[-1].layer

    def run(s, e):
        return layers[s - first:e - first + 1]

    def exact():
        r = allocate(layers, devices)
        r.sticky = False
        return r

    chain = sorted(({"id": c["id"], "start": max(c["start"], first), "end": min(c["end"], last)}
                    for c in current if c["id"] in by_id and c.get("start") is not None),
                   key=lambda c: c["start"])
    chain = [c for c in chain if c["start"] <= c["end"]]
    if not chain:
        return exact()
    for c in chain:
        if not _fits(by_id[c["id"]], run(c["start"], c["end"])):
            return exact()

    # 1. free runs go to their neighbours, at the cheapest split point
    covered = {l for c in chain for l in range(c["start"], c["end"] + 1)}
    l = first
    while l <= last:
        if l in covered:
            l += 1
            continue
        e = l
        while e + 1 <= last and e + 1 not in covered:
            e += 1
        left = next((c for c in chain if c["end"] == l - 1), None)
        right = next((c for c in chain if c["start"] == e + 1), None)
        best = None
        for k in range(0, e - l + 2):  # left takes [l, l+k-1], right [l+k, e]
            if k > 0 and left is None:
                continue
            if k < e - l + 1 and right is None:
                continue
            trial = [dict(c) for c in chain]
            ok = True
            if k > 0:
                tl = next(c for c in trial if c["id"] == left["id"])
                tl["end"] = l + k - 1
                ok = _fits(by_id[tl["id"]], run(tl["start"], tl["end"]))
            if ok and k < e - l + 1:
                tr = next(c for c in trial if c["id"] == right["id"])
                tr["start"] = l + k
                ok = _fits(by_id[tr["id"]], run(tr["start"], tr["end"]))
            if not ok:
                continue
            cost = _chain_cost(layers, by_id, trial)
            if best is None or cost < best[0]:
                best = (cost, trial)
        if best is None:
            return exact()
        chain = best[1]
        covered.update(range(l, e + 1))
        l = e + 1

    # 2. newcomers in join order: a prefix or suffix of one incumbent
    for dev in devices:
        if any(c["id"] == dev.id for c in chain):
            continue
        best = None
        for donor in chain:
            n = donor["end"] - donor["start"] + 1
            for k in range(1, n):
                for side in ("suffix", "prefix"):
                    if side == "suffix":
                        mine = {"id": dev.id, "start": donor["end"] - k + 1, "end": donor["end"]}
                        kept = {"id": donor["id"], "start": donor["start"], "end": donor["end"] - k}
                    else:
                        mine = {"id": dev.id, "start": donor["start"], "end": donor["start"] + k - 1}
                        kept = {"id": donor["id"], "start": donor["start"] + k, "end": donor["end"]}
                    if not _fits(dev, run(mine["start"], mine["end"])):
                        continue
                    trial = [kept if c["id"] == donor["id"] else dict(c) for c in chain] + [mine]
                    cost = _chain_cost(layers, by_id, trial)
                    if best is None or cost < best[0]:
                        best = (cost, trial)
        if best is None:
            return exact()
        chain = sorted(best[1], key=lambda c: c["start"])
    r = _describe(layers, devices, chain)
    r.sticky = True
    return r


def explain(a: Assignment) -> str:
    """allocate.js:440 -- one line on why a device got its share."""
    return (f"{a.layers} layer{'' if a.layers == 1 else 's'} ({a.start}-{a.end}), {_mb(a.bytes)} = "
            f"{a.share * 100:.0f}% of the stage bytes, at {a.rate / 1e6:.2f}MB/ms -> {a.ms}ms")


def measure_rate(dev, rows: int = 8192, cols: int = 4096, iters: int = 20) -> float:
    """This GPU's streaming rate in bytes per ms: a timed Q8_0 matvec over a
    rows x cols synthetic matrix (larger than one layer of the 0.6B shape)."""
    from . import ops, synth
    from .lib import GpuTensor
    t = GpuTensor.from_packed(dev, synth.q8_tensor(1, "rate", rows, cols), rows, cols)
    ms = ops.matvec_timed(dev, t, 1, iters)
    t.free()
    return rows * cols * 1.0625 / ms
