"""Small, fixed GPU workloads for profiling one kernel family at a time.

    python profile_cases.py layer [--time]   # one decode layer (config 0 shape, 256-key cache)
    python profile_cases.py head  [--time] [--fast]
                                                # the 151936 x 1024 Q8_0 head matvec (--fast:
                                                # and the int8 tensor-core matvec after it)
    python profile_cases.py gemv  [--time] [--8b]
                                                # the config 1 matvec sweep (M = 1), or the
                                                # 8B shapes (config 4)
    python profile_cases.py sweep [--time]   # config 1: Q8_0/Q4_0 x shapes x M in {1,16,128,512}
    python profile_cases.py gemm  [--time] [rows cols [M]]
                                                # one tensor-core GEMM (default 3072 x 1024, M 512)
    python profile_cases.py model [--time] [--kernels | --persistent] [--trace]
    python profile_cases.py model8b [--time] [--prompt P] [--decode N] [--persistent]
                                                # config 4 on one GPU: Qwen3-8B shape, 36
                                                # layers, untied head; 4096-token prompt
                                                # (tensor-core prefill, 512-token chunks), then
                                                # N (default 512) greedy decode tokens
    python profile_cases.py prefill [--time] [--exact]
                                                # config 3: 512-token prompt TTFT on the
                                                # 28-layer model, tensor-core (default) or
                                                # exact prefill, then 32 decode tokens
                                                # 28-layer 0.6B-shape decode: streaming
                                                # kernel (default), persistent kernel or
                                                # per-op kernel graph

Each case builds seeded synthetic weights, runs a few warm launches and, with
--time, prints CUDA-event timings.  They are small enough (< 1 GB on the
device) to run under ncu; the model case decodes 3 warm tokens after a
64-token prompt, then (with --time) 64 timed tokens.
"""
from __future__ import annotations

import sys

import os

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from flock_b200 import ops, synth  # noqa: E402
from flock_b200 import lib as flib  # noqa: E402
from flock_b200.layer import QWEN3_06B, Layer  # noqa: E402

SWEEP = [(2048, 1024), (1024, 1024), (1024, 2048), (3072, 1024), (1024, 3072), (151936, 1024)]
SWEEP_8B = [(4096, 4096), (1024, 4096), (12288, 4096), (4096, 12288), (151936, 4096)]


def layer_case(timed: bool, attention: str = "fast") -> None:
    dev = flib.get_device(0)
    L = Layer.create(dev, synth.layer_weights(100, 24), QWEN3_06B.with_(attention=attention))
    kvw = 1024
    L.write_cache(synth.normal(1, "k", 256 * kvw), synth.normal(1, "v", 256 * kvw))
    x = synth.normal(1, "x", 1024)
    for i in range(5):
        L.encode(x if i == 0 else None)
    dev.sync()
    if timed:
        # config 0: one layer's decode step from position 261 on, 1000 steps
        # (the cache grows to 1260 keys); bytes = weights + the K/V rows read
        n = 1000
        dev.timer_start()
        for _ in range(n):
            L.encode(None)
        ms = dev.timer_stop()
        keys = 261 + (n - 1) / 2.0 + 1
        b = 15728640 * 1.0625 + 2 * keys * 1024 * 4
        us = ms / n * 1000
        print(f"layer decode ({attention}): {us:.2f} us/step, {b / us / 1e3:.1f} GB/s "
              f"({b / 1e6:.2f} MB/step at {keys:.0f} keys on average)")


def head_case(timed: bool) -> None:
    """--fast: the exact matvec (2 launches untimed) and then the int8
    tensor-core matvec (FLOCK_MATVEC_FAST, 2 launches untimed)."""
    dev = flib.get_device(0)
    t = flib.GpuTensor.from_packed(dev, synth.q8_tensor(6, "head", 151936, 1024), 151936, 1024)
    fast = "--fast" in sys.argv
    ms = ops.matvec_timed(dev, t, 1, 50 if timed else (1 if fast else 3))
    b = 151936 * 1024 * 1.0625 + 4 * (1024 + 151936)
    if timed:
        print(f"head matvec: {ms * 1000:.2f} us, {b / ms / 1e6:.1f} GB/s")
    if fast:
        ms = ops.matvec_fast_timed(dev, t, 50 if timed else 1)
        if timed:
            print(f"head matvec (int8 tensor cores): {ms * 1000:.2f} us, {b / ms / 1e6:.1f} GB/s")


def gemv_case(timed: bool) -> None:
    dev = flib.get_device(0)
    shapes = SWEEP_8B if "--8b" in sys.argv else SWEEP
    for q8 in ((True,) if "--8b" in sys.argv else (True, False)):
        for rows, cols in shapes:
            make = synth.q8_tensor if q8 else synth.q4_tensor
            t = flib.GpuTensor.from_packed(dev, make(2, "t", rows, cols), rows, cols,
                                           flib.FLOCK_Q8_0 if q8 else flib.FLOCK_Q4_0)
            ms = ops.matvec_timed(dev, t, 1, 100 if timed else 2)
            if timed:
                b = rows * cols * (1.0625 if q8 else 0.5625) + 4 * (rows + cols)
                print(f"{'Q8_0' if q8 else 'Q4_0'} {rows}x{cols}: {ms * 1000:.2f} us "
                      f"{b / ms / 1e6:.1f} GB/s")


def sweep_case(timed: bool) -> None:
    """Config 1: M = 1 through the GEMV, M > 1 through the tensor-core GEMM
    (activation conversion included); the per-token GEMV at M = 16 beside it."""
    dev = flib.get_device(0)
    if timed:
        print("| wt | K x N | M | engine | us | GB/s | TFLOP/s |")
        print("|---|---|---|---|---|---|---|")
    for q8 in (True, False):
        for rows, cols in SWEEP:
            make = synth.q8_tensor if q8 else synth.q4_tensor
            t = flib.GpuTensor.from_packed(dev, make(2, "t", rows, cols), rows, cols,
                                           flib.FLOCK_Q8_0 if q8 else flib.FLOCK_Q4_0)
            bpw = 1.0625 if q8 else 0.5625
            runs = [(1, "gemv", lambda: (ops.matvec_timed(dev, t, 1, 50 if timed else 2), 0.0)),
                    (16, "gemv", lambda: (ops.matvec_timed(dev, t, 16, 10 if timed else 1), 0.0))]
            for m in (16, 128, 512):
                runs.append((m, "tcgen05", lambda m=m: ops.gemm_timed(dev, t, m, 20 if timed else 1)))
            for m, eng, f in runs:
                ms, img = f()
                if timed:
                    b = rows * cols * bpw + 4 * cols * m + 4 * rows * m
                    tf = 2.0 * m * rows * cols / (ms * 1e-3) / 1e12
                    extra = f" (+{img * 1000:.1f} us x->f16)" if img else ""
                    print(f"| {'Q8_0' if q8 else 'Q4_0'} | {cols} x {rows} | {m} | {eng} | "
                          f"{ms * 1000:.1f}{extra} | {b / ms / 1e6:.0f} | {tf:.1f} |")
            t.free()


def gemm_case(timed: bool) -> None:
    dev = flib.get_device(0)
    nums = [int(a) for a in sys.argv[2:] if a.isdigit()]
    rows, cols, m = (nums + [3072, 1024, 512][len(nums):])[:3]
    t = flib.GpuTensor.from_packed(dev, synth.q8_tensor(2, "t", rows, cols), rows, cols)
    ms, _ = ops.gemm_timed(dev, t, m, 20 if timed else 2)
    if timed:
        print(f"gemm M {m} x K {cols} x N {rows}: {ms * 1000:.1f} us, "
              f"{2 * m * rows * cols / (ms * 1e-3) / 1e12:.1f} TFLOP/s")


def prefill_case(timed: bool) -> None:
    from flock_b200.model import Model
    dev = flib.get_device(0)
    m = synth.model(300)
    exact = "--exact" in sys.argv
    cfg = QWEN3_06B.with_(attention="fast", max_keys=1024,
                          prefill="exact" if exact else "tensor")
    M = Model.create(dev, m, cfg)
    prompt = synth.uniform_ids(300, "p512", 512, synth.QWEN3_06B.vocab).tolist()
    M.step(prompt[:64])  # warm-up: kernels loaded, workspaces touched
    M.reset()
    dev.sync()
    dev.timer_start()
    first = M.step(prompt)
    ttft = dev.timer_stop()
    dev.timer_start()
    M.decode_device(32)
    dec = dev.timer_stop()
    if timed:
        print(f"prefill ({'exact' if exact else 'tensor cores'}): TTFT {ttft:.2f} ms for 512 "
              f"tokens ({512 / ttft * 1000:.0f} tok/s), first id {first}; 32 decode tokens "
              f"{dec / 32 * 1000:.1f} us/token")


def model8b_case(timed: bool) -> None:
    import time
    from flock_b200.layer import LayerConfig
    from flock_b200.model import Model
    s = synth.QWEN3_8B
    n_prompt = 4096
    n_dec = 512
    if "--decode" in sys.argv:
        n_dec = int(sys.argv[sys.argv.index("--decode") + 1])
    if "--prompt" in sys.argv:
        n_prompt = int(sys.argv[sys.argv.index("--prompt") + 1])
    dev = flib.get_device(0)
    t0 = time.perf_counter()
    m = synth.model(400, s)
    cfg = LayerConfig(hidden=s.hidden, n_heads=s.n_heads, n_kv_heads=s.n_kv_heads,
                      head_dim=s.head_dim, ffn=s.ffn, max_keys=n_prompt + n_dec + 64,
                      max_prefill=512, attention="fast", prefill="tensor")
    M = Model.create(dev, m, cfg)
    if "--persistent" in sys.argv:
        M.decode_mode = "persistent"
    t_load = time.perf_counter() - t0
    prompt = synth.uniform_ids(400, "p4096", n_prompt, s.vocab).tolist()
    M.step(prompt[:min(512, n_prompt)])  # warm-up
    M.reset()
    dev.sync()
    dev.timer_start()
    first = M.step(prompt)
    ttft = dev.timer_stop()
    M.decode_device(8)
    M.rewind(n_prompt)
    M.set_token(first)
    dev.sync()
    dev.timer_start()
    ids = M.decode_device(n_dec)
    ms = dev.timer_stop()
    if timed:
        q, kv = s.n_heads * s.head_dim, s.n_kv_heads * s.head_dim
        layer_w = (q * s.hidden + 2 * kv * s.hidden + s.hidden * q + 3 * s.ffn * s.hidden) * 1.0625
        keys = n_prompt + (n_dec + 1) / 2.0
        tok_bytes = s.n_layers * (layer_w + 2 * kv * 4 * keys) + s.vocab * s.hidden * 1.0625
        tok_s = n_dec / (ms * 1e-3)
        print(f"config 4 (8B shape, 1 GPU, {M.decode_mode}): synthetic weights + upload "
              f"{t_load:.1f} s; "
              f"TTFT {ttft:.1f} ms for {n_prompt} tokens; decode {n_dec} tokens "
              f"{ms / n_dec * 1000:.1f} us/token = {tok_s:.1f} tok/s = "
              f"{tok_bytes * tok_s / 1e9:.0f} GB/s ({tok_bytes / 1e9:.2f} GB/token); "
              f"first ids {first} {ids[:4].tolist()}")


PHASES = ("qkv", "attention", "o_proj", "gate/up", "down")


def trace_summary(tr, n_layers: int) -> str:
    """Per phase of the persistent kernel, averaged over layers: compute time
    (mean and slowest CTA) and time spent in the grid barrier after it."""
    import numpy as np
    t = (tr[:, :4 + 10 * n_layers].astype(np.int64) - int(tr[:, 0].min())) / 1000.0
    lines = [f"token: {t[:, 3 + 10 * n_layers].max():.1f} us; start skew {t[:, 0].max():.2f} us; "
             f"embed {np.mean(t[:, 1] - t[:, 0]):.2f} us"]
    for p, name in enumerate(PHASES):
        comp, slow, wait = [], [], []
        for l in range(n_layers):
            c = 2 + 10 * l + 2 * p
            d = t[:, c] - t[:, c - 1]
            comp.append(d.mean())
            slow.append(d.max())
            wait.append((t[:, c + 1] - t[:, c]).mean())
        lines.append(f"{name:>9}: compute {np.mean(comp):6.2f} us (slowest CTA {np.mean(slow):6.2f}), "
                     f"barrier {np.mean(wait):5.2f} us; x{n_layers} = "
                     f"{(np.mean(comp) + np.mean(wait)) * n_layers:7.1f} us")
    h = 2 + 10 * n_layers
    lines.append(f"     head: compute {np.mean(t[:, h] - t[:, h - 1]):6.2f} us "
                 f"(slowest {np.max(t[:, h] - t[:, h - 1]):.2f}), argmax "
                 f"{np.max(t[:, h + 1] - t[:, h]):.2f} us")
    return "\n".join(lines)


def stream_trace_summary(tr, n_layers: int) -> str:
    """The streaming decode kernel's trace: per step of a layer, the median
    and slowest CTA's time since the previous step (averaged over layers),
    the token time and the ring's wait totals."""
    import numpy as np
    t = (tr.astype(np.int64) - int(tr[:, 0].min())) / 1000.0
    names = ["h polled", "QKV rows", "q/k/v polled", "attention", "attn polled", "o_proj rows",
             "h polled", "gate/up rows", "act polled", "down rows"]
    L = n_layers
    # head stamps exist only when the head runs inside the kernel; otherwise
    # the slots hold whatever an earlier launch left (outside this token)
    t0 = int(tr[:, 0].min())
    hs = tr[:, 2 + 10 * L: 5 + 10 * L].astype(np.int64) - t0
    head_in = bool(((hs > 0) & (hs < 10**9)).all())
    end = t[:, 4 + 10 * L].max() if head_in else t[:, 1 + 10 * L].max()
    lines = [f"{'token' if head_in else 'layers (head launched after)'}: {end:.1f} us; "
             f"embed {np.median(t[:, 1]):.2f} us"]
    for k, name in enumerate(names):
        med, mx = [], []
        for l in range(1, L):
            c = 2 + 10 * l + k
            prev = c - 1 if k != 3 else c - 2   # attention: from the QKV rows
            if k == 2:
                sel = tr[:, c] > 0
                if not sel.any():
                    continue
                d = t[sel, c] - t[sel, c - 1]
            elif k == 4:
                d = t[:, c] - np.max(t[:, c - 1])   # after the slowest attention
            else:
                d = t[:, c] - t[:, prev]
            med.append(np.median(d))
            mx.append(np.max(d))
        if med:
            lines.append(f"{name:>14}: median {np.mean(med):6.2f} us, slowest CTA {np.mean(mx):6.2f} us")
    h = 2 + 10 * L
    if head_in:
        lines.append(f"head: input polled {np.median(t[:, h] - t[:, h - 1]):.2f} us, rows "
                     f"{np.median(t[:, h + 1] - t[:, h]):.2f} us (slowest "
                     f"{np.max(t[:, h + 1] - t[:, h]):.2f}), argmax "
                     f"{np.max(t[:, h + 2]) - np.max(t[:, h + 1]):.2f} us")
    det = tr[:, 8 + 10 * L: 20 + 10 * L].astype(np.int64)
    rows = det[:, 0] > 0
    if rows.any():
        steps = ["q/k/v polled", "q/k rotated", "key appended", "tile staged", "scores",
                 "softmax", "P.V", "published / weights", "combined"]
        d = (det[rows] - det[rows, :1]) / 1000.0
        parts = []
        for k in range(1, len(steps)):
            col = d[:, k][det[rows, k] > 0]
            if col.size:
                parts.append(f"{steps[k]} +{np.median(col):.2f}/{col.max():.2f}")
        lines.append("last layer's attention item (median/max us after its q/k/v poll): "
                     + ", ".join(parts))
    for off, name in ((0, "QKV"), (9, "gate/up"), (18, "down")):
        pd = tr[:, 20 + 10 * L + off: 29 + 10 * L + off].astype(np.int64)
        if (pd[:, 0] > 0).any():
            d = (pd - pd[:, :1]) / 1000.0
            parts = []
            for k in range(4):
                w, r = pd[:, 1 + 2 * k] > 0, pd[:, 2 + 2 * k] > 0
                if w.any():
                    parts.append(f"piece {k}: full +{np.median(d[w, 1 + 2 * k]):.2f}, rows "
                                 f"+{np.median(d[r, 2 + 2 * k]):.2f}")
            lines.append(f"last layer's {name} phase (median us after its start): "
                         + "; ".join(parts))
    lines.append(f"ring: consumers waited {np.median(tr[:, 5 + 10 * L]) / 1e3:.1f} us a token "
                 f"(median CTA), producer waited {np.median(tr[:, 6 + 10 * L]) / 1e3:.1f} us; "
                 f"{int(np.median(tr[:, 7 + 10 * L]))} pieces per CTA")
    return "\n".join(lines)


def model_case(timed: bool) -> None:
    from flock_b200.model import Model
    dev = flib.get_device(0)
    m = synth.model(300)
    M = Model.create(dev, m, QWEN3_06B.with_(attention="fast"))
    M.decode_mode = ("kernels" if "--kernels" in sys.argv else
                     "persistent" if "--persistent" in sys.argv else "stream")
    M.step(synth.uniform_ids(300, "prompt", 64, synth.QWEN3_06B.vocab).tolist())
    M.decode_device(3)
    dev.sync()
    if timed:
        dev.timer_start()
        M.decode_device(64)
        ms = dev.timer_stop()
        print(f"model decode ({M.decode_mode}): {ms / 64 * 1000:.1f} us/token, "
              f"{64 / ms * 1000:.1f} tok/s")
    if "--trace" in sys.argv:
        M.trace(True)
        M.decode_device(4)
        summary = stream_trace_summary if M.decode_mode == "stream" else trace_summary
        print(summary(M.read_trace(), M.held))
        M.trace(False)


if __name__ == "__main__":
    case = sys.argv[1] if len(sys.argv) > 1 else "layer"
    timed = "--time" in sys.argv
    {"layer": layer_case, "head": head_case, "gemv": gemv_case, "model": model_case,
     "sweep": sweep_case, "gemm": gemm_case, "prefill": prefill_case,
     "model8b": model8b_case}[case](timed)
    print("ok")
