"""The layer allocator (server/allocate.js restated in flock_b200.allocate):
byte-weighted minimum-makespan contiguous ranges, per-device tensor and
budget limits, precise infeasibility, sticky membership edits, and the
layer plan read from a GGUF directory."""
import itertools

import pytest

from flock_b200 import synth
from flock_b200.allocate import (DEFAULT_RATE, Device, Infeasible, LayerInfo, adjust, allocate,
                                 explain, layer_plan)

MB = 1e6


def run_of(first, n, size=20 * MB, max_tensor=6 * MB, sizes=None):
    return [LayerInfo(first + i, int(sizes[i] if sizes else size),
                      int(max_tensor[i] if isinstance(max_tensor, list) else max_tensor),
                      f"blk.{first + i}.ffn_down.weight") for i in range(n)]


def contiguous(alloc, layers):
    want = layers[0].layer
    for a in alloc.assign:
        if a.start != want or a.end < a.start:
            return False
        want = a.end + 1
    return want == layers[-1].layer + 1


def brute_makespan(layers, devices):
    """Every contiguous cut, for checking the DP's optimum."""
    L, D = len(layers), len(devices)
    best = float("inf")
    for cuts in itertools.combinations(range(1, L), D - 1):
        bounds = (0,) + cuts + (L,)
        span = 0.0
        ok = True
        for d in range(D):
            run = layers[bounds[d]:bounds[d + 1]]
            dev = devices[d]
            b = sum(l.bytes for l in run)
            if any(l.max_tensor > dev.bind for l in run) or b > dev.budget:
                ok = False
                break
            span = max(span, b / dev.rate + dev.reserved_ms)
        if ok:
            best = min(best, span)
    return best


@pytest.mark.parametrize("n", [1, 2, 3, 5, 8])
def test_any_device_count_covers_every_layer(n):
    ls = run_of(0, 28)
    r = allocate(ls, [Device(f"d{i}") for i in range(n)])
    assert contiguous(r, ls) and len(r.assign) == n
    assert all(a.layers >= 1 for a in r.assign)
    assert r.ranges()[0][0] == 0 and r.ranges()[-1][1] == 28


def test_weighted_by_bytes_not_count():
    ls = run_of(0, 6, sizes=[300 * MB] * 3 + [100 * MB] * 3)
    r = allocate(ls, [Device("a"), Device("b")])
    assert r.assign[0].layers < r.assign[1].layers
    assert r.even_ms > r.makespan_ms


def test_optimum_matches_exhaustive_search():
    sizes = [37, 12, 88, 5, 61, 23, 44, 19, 70, 8]
    ls = run_of(0, 10, sizes=[s * MB for s in sizes])
    devs = [Device("a", rate=3e3), Device("b", rate=1e3, reserved_ms=5), Device("c", rate=2e3)]
    r = allocate(ls, devs)
    assert abs(r.makespan_ms - round(brute_makespan(ls, devs), 2)) < 0.011


def test_binding_limit_keeps_big_tensors_off_small_devices():
    mt = [6 * MB] * 4 + [200 * MB] + [6 * MB] * 3
    ls = run_of(0, 8, max_tensor=mt)
    small = Device("phone", bind=128 * 1024 * 1024)
    big = Device("mac", bind=4 * 1024 ** 3)
    for order in ([small, big], [big, small]):
        r = allocate(ls, order)
        p = next(a for a in r.assign if a.id == "phone")
        assert not p.start <= 4 <= p.end and contiguous(r, ls)
    with pytest.raises(Infeasible) as e:
        allocate(run_of(0, 4, max_tensor=200 * MB), [small, big])
    assert e.value.detail["kind"] in ("contiguity", "tensor")


def test_budget_and_shortfall():
    ls = run_of(0, 8, size=50 * MB)
    r = allocate(ls, [Device("tiny", budget=120 * MB), Device("roomy", budget=2000 * MB)])
    assert next(a for a in r.assign if a.id == "tiny").bytes <= 120 * MB
    with pytest.raises(Infeasible, match="short") as e:
        allocate(ls, [Device("a", budget=100 * MB), Device("b", budget=100 * MB)])
    assert e.value.detail["kind"] == "budget"


def test_slow_device_gets_fewer_layers():
    ls = run_of(0, 12, size=4.2 * MB)
    phone = Device("phone", "iPhone", rate=16.8e6 / 15.4)
    mac = Device("mac", "Mac", rate=100.8e6 / 19.6)
    r = allocate(ls, [phone, mac])
    p, m = r.assign
    assert p.layers < m.layers and m.layers / p.layers > 3
    assert r.even_ms / r.makespan_ms > 1.5
    assert "layers" in explain(p) and "MB/ms" in explain(m)


def test_infeasible_kinds():
    with pytest.raises(Infeasible) as e:
        allocate([LayerInfo(40, int(700 * MB), int(638 * MB), "output.weight")],
                 [Device("phone", "iPhone", bind=128 * 1024 * 1024)])
    msg = str(e.value)
    assert "output.weight" in msg and "layer 40" in msg and "638.0MB" in msg
    assert "134.2MB" in msg and "adding more devices will not help" in msg
    assert e.value.detail["kind"] == "tensor" and e.value.detail["needs"] == int(638 * MB)
    with pytest.raises(Infeasible) as e:
        allocate(run_of(0, 2), [Device("a"), Device("b"), Device("c")])
    assert e.value.detail["kind"] == "too-many-devices"
    with pytest.raises(Infeasible) as e:
        allocate(run_of(0, 2), [])
    assert e.value.detail["kind"] == "empty"


def test_reserved_time_shrinks_the_coordinator_share():
    ls = run_of(0, 28, size=16.7 * MB)
    plain = allocate(ls, [Device(f"g{i}", rate=4e6) for i in range(4)])
    busy = allocate(ls, [Device("g0", rate=4e6, reserved_ms=10.0)] +
                    [Device(f"g{i}", rate=4e6) for i in range(1, 4)])
    assert busy.assign[0].layers < plain.assign[0].layers


def test_adjust_join_moves_only_the_donor():
    ls = run_of(0, 12)
    devs = [Device("a"), Device("b")]
    cur = [{"id": a.id, "start": a.start, "end": a.end} for a in allocate(ls, devs).assign]
    r = adjust(ls, cur, devs + [Device("c")])
    assert r.sticky and contiguous(r, ls) and len(r.assign) == 3
    moved = [c for c in cur if (c["start"], c["end"]) not in
             {(a.start, a.end) for a in r.assign if a.id == c["id"]}]
    assert len(moved) == 1  # one donor gave up a run; nobody else moved


def test_adjust_leave_goes_to_neighbours():
    ls = run_of(0, 12)
    devs = [Device("a"), Device("b"), Device("c")]
    cur = [{"id": a.id, "start": a.start, "end": a.end} for a in allocate(ls, devs).assign]
    r = adjust(ls, cur, [devs[0], devs[2]])
    assert r.sticky and contiguous(r, ls)
    a = next(x for x in r.assign if x.id == "a")
    assert a.start == cur[0]["start"]


def test_adjust_falls_back_when_limits_change():
    ls = run_of(0, 6, size=50 * MB)
    devs = [Device("a"), Device("b")]
    cur = [{"id": a.id, "start": a.start, "end": a.end} for a in allocate(ls, devs).assign]
    r = adjust(ls, cur, [Device("a", budget=60 * MB), Device("b")])
    assert r.sticky is False and contiguous(r, ls)


def test_layer_plan_from_model_and_gguf(tmp_path):
    import gguf_writer as gw
    from flock_b200.gguf import GGUFFile
    m = synth.model(3, n_layers=3, vocab=256)
    plan = layer_plan(m)
    assert [p.layer for p in plan] == [0, 1, 2]
    assert plan[0].biggest.endswith("ffn_down.weight") or plan[0].biggest.endswith("ffn_gate.weight")
    p = str(tmp_path / "m.gguf")
    gw.write_model(p, m)
    g = GGUFFile(p)
    gplan = layer_plan(g)
    assert [x.bytes for x in gplan] == [x.bytes for x in plan]
    assert [x.max_tensor for x in gplan] == [x.max_tensor for x in plan]
    r = allocate(gplan, [Device("g0", rate=DEFAULT_RATE), Device("g1")])
    assert contiguous(r, gplan)
