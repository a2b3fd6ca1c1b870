#!/usr/bin/env python
"""Decode throughput of the Qwen3-0.6B-shaped Q8_0 model on B200.

Workload (benchmark config 2): the full 28-layer model with a tied
151936 x 1024 Q8_0 embedding/head and seeded synthetic Q8_0 weights, a
64-token prompt (ids uniform in [0, 151936)), then greedy batch-1 decode.  A
step is one decode token (embedding -> 28 layers -> output_norm -> head ->
argmax); K steps cover positions 64 .. 64+K-1 (K = 256 reproduces config 2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl flock|reference]

`value`: tokens/s with the token fed back on the device (one CUDA graph per
token, no host round trip), CUDA-event timed, max over ranks.
`e2e`:   the same decode through the public API, one Model.step([id]) per
token (4-byte H2D of the id, 4-byte D2H of the next id, host loop).
N > 1: layer-range pipeline (4 layers + head on rank 0, the rest split
evenly), hidden state passed with NCCL send/recv; per-token work is fixed,
so scaling is "strong".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "decode tok/s (bs1, Qwen3-0.6B-shape Q8_0)"
PROMPT = 64
SEED = 0


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ----------------------------------------------------------------- clocks
class Clocks:
    """nvidia-smi sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return int(vis.split(",")[local_rank])
        except (ValueError, IndexError):
            pass
    return local_rank


def peaks() -> dict:
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d.get("bf16_tflops", 1590.0),
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", 1400.0),
                "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "src": "fallback"}


def traffic_from_profile(name: str = "gemv_lm_head_traffic.txt") -> float | None:
    """dram bytes per launch from a committed ncu summary, if any."""
    p = os.path.join(HERE, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("dram_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


# ----------------------------------------------------------------- bytes
def bytes_per_token(shape, keys: float, kv_elem: int = 4) -> float:
    """Algorithmic HBM bytes of one decode token: every Q8_0 weight byte
    (1.0625 B/weight) and the K/V rows read (kv_elem bytes per element: 4 for
    the f32 cache, 2 for bf16)."""
    h, f, q, kv = shape.hidden, shape.ffn, shape.n_heads * shape.head_dim, \
        shape.n_kv_heads * shape.head_dim
    layer_w = (q * h + 2 * kv * h + h * q + 2 * f * h + h * f) * 1.0625
    head_w = shape.vocab * h * 1.0625
    kv_bytes = 2 * kv * kv_elem * keys
    return shape.n_layers * (layer_w + kv_bytes) + head_w


# ------------------------------------------------------------ cpu baseline
def cpu_baseline(m, shape, n_tokens: int = 2) -> dict:
    """The oracle (C restatement of layer_ref.ts / model.ts) decoding
    n_tokens at position 64 on all host cores."""
    import oracle
    cores = len(os.sched_getaffinity(0))
    oracle.set_threads(cores)
    cfg = dict(hidden=shape.hidden, n_heads=shape.n_heads, n_kv_heads=shape.n_kv_heads,
               head_dim=shape.head_dim, ffn=shape.ffn)
    kvw = shape.n_kv_heads * shape.head_dim
    layers = []
    for i, w in enumerate(m.layers):
        L = oracle.RefLayer(w, cfg, PROMPT + n_tokens + 1)
        L.fill_cache(np.random.default_rng(i).standard_normal(PROMPT * kvw).astype(np.float32),
                     np.random.default_rng(100 + i).standard_normal(PROMPT * kvw).astype(np.float32))
        layers.append(L)
    tok = 1
    t0 = time.perf_counter()
    for _ in range(n_tokens):
        h = oracle.embed(m.embd["packed"], [tok], shape.hidden)
        for L in layers:
            h = L.forward(h, 1)
        tok, _, _ = oracle.head(h, m.output_norm, m.embd["packed"], shape.vocab, shape.hidden)
    dt = time.perf_counter() - t0
    # the reference's JS engine runs one thread: the same path on one core
    oracle.set_threads(1)
    t1 = time.perf_counter()
    h = oracle.embed(m.embd["packed"], [tok], shape.hidden)
    for L in layers:
        h = L.forward(h, 1)
    oracle.head(h, m.output_norm, m.embd["packed"], shape.vocab, shape.hidden)
    single = 1.0 / (time.perf_counter() - t1)
    oracle.set_threads(cores)
    return {"value": n_tokens / dt, "unit": "tok/s", "cores": cores, "kind": "port",
            "single_thread_value": single,
            "sample": f"{n_tokens} decode tokens of the 28-layer model at position {PROMPT} "
                      f"(oracle/flock_oracle.c, OpenMP over rows, {cores} threads)"}


def oracle_ids(m, shape, prompt, n: int, kv: str = "f32") -> list:
    """The oracle's first n greedy ids for `prompt` (kernels/model.ts:387 step
    composed from layer_ref.ts / head_ref.ts): the checker for the timed run;
    kv: the cache rounding the run uses ("f32", "bf16", "fp8")."""
    import oracle
    oracle.set_threads(len(os.sched_getaffinity(0)))
    cfg = dict(hidden=shape.hidden, n_heads=shape.n_heads, n_kv_heads=shape.n_kv_heads,
               head_dim=shape.head_dim, ffn=shape.ffn)
    layers = [oracle.RefLayer(w, cfg, len(prompt) + n + 1, kv=kv) for w in m.layers]
    ids, cur = [], [int(t) for t in prompt]
    for _ in range(n):
        h = oracle.embed(m.embd["packed"], cur, shape.hidden)
        for L in layers:
            h = L.forward(h, len(cur))
        tok, _, _ = oracle.head(h[(len(cur) - 1) * shape.hidden:], m.output_norm,
                                m.embd["packed"], shape.vocab, shape.hidden)
        ids.append(int(tok))
        cur = [int(tok)]
    return ids


def config1_sweep(dev, pk) -> dict:
    """Benchmark config 1: the Q8_0 / Q4_0 matmul over the model's projection
    shapes.  M = 1 (and 16) through the decode GEMV (M = 1 also through the
    reassociated int8 tensor-core matvec, "gemv_fast"), M in {16, 128, 512}
    through the tcgen05 GEMM (f16 operands, f32 accumulation; the activation
    conversion is timed apart); every launch timed alone after a 256 MiB L2
    eviction, so the weights stream from HBM."""
    from flock_b200 import lib as flib
    from flock_b200 import ops, synth
    from flock_b200 import _abi
    import ctypes
    shapes = [(2048, 1024), (1024, 1024), (1024, 2048), (3072, 1024), (1024, 3072),
              (151936, 1024)]   # (rows N, cols K)
    rows_out = []
    for q8 in (True, False):
        for n, k in shapes:
            make = synth.q8_tensor if q8 else synth.q4_tensor
            t = flib.GpuTensor.from_packed(dev, make(2, "t", n, k), n, k,
                                           flib.FLOCK_Q8_0 if q8 else flib.FLOCK_Q4_0)
            bpw = 1.0625 if q8 else 0.5625
            for m_tok, eng in ((1, "gemv"), (1, "gemv_fast"), (16, "gemv"), (16, "tcgen05"),
                               (128, "tcgen05"), (512, "tcgen05")):
                ms = ctypes.c_float()
                img = ctypes.c_float()
                if eng == "gemv":
                    _abi.call("flock_op_matvec_timed_cold", dev.handle, t.handle, m_tok, 10,
                              ctypes.byref(ms))
                elif eng == "gemv_fast":
                    _abi.call("flock_op_matvec_fast_timed", dev.handle, t.handle, 10, 1,
                              ctypes.byref(ms))
                else:
                    _abi.call("flock_op_gemm_timed_cold", dev.handle, t.handle, m_tok, 10,
                              ctypes.byref(ms), ctypes.byref(img))
                b = n * k * bpw + 4 * k * m_tok + 4 * n * m_tok
                gbs = b / (ms.value * 1e-3) / 1e9
                tf = 2.0 * m_tok * n * k / (ms.value * 1e-3) / 1e12
                r = {"wt": "Q8_0" if q8 else "Q4_0", "KxN": f"{k}x{n}", "M": m_tok,
                     "engine": eng, "us": round(ms.value * 1000, 2), "GB_s": round(gbs, 1),
                     "frac_hbm": round(gbs / pk["hbm_gbs"], 3), "TFLOP_s": round(tf, 2)}
                if eng == "tcgen05":
                    r["frac_bf16_peak"] = round(tf / pk["bf16_tflops"], 3)
                    r["act_image_us"] = round(img.value * 1000, 2)
                rows_out.append(r)
            t.free()
    return {"workload": "config 1: Q8_0/Q4_0 matmul sweep, K x N over the 0.6B projections "
                        "and the 1024 x 151936 head, M in {1, 16} (GEMV; M = 1 also gemv_fast, "
                        "the int8 tensor-core matvec) and {16, 128, 512} (tcgen05)",
            "timing": "each launch alone after a 256 MiB L2 eviction, CUDA events, mean of 10",
            "peak_hbm_gbs": pk["hbm_gbs"], "peak_bf16_tflops": pk["bf16_tflops"],
            "rows": rows_out}


def run_reference(args, rank: int, world: int) -> None:
    """--impl reference: the reference's CPU path (its strict-f32 TS oracle,
    restated in C: Deno is absent) on this config, on the host cores."""
    if rank != 0:
        return
    from flock_b200 import synth
    import oracle
    shape = synth.QWEN3_06B
    m = synth.model(SEED, shape)
    cores = len(os.sched_getaffinity(0))
    oracle.set_threads(cores)
    cfg = dict(hidden=shape.hidden, n_heads=shape.n_heads, n_kv_heads=shape.n_kv_heads,
               head_dim=shape.head_dim, ffn=shape.ffn)
    kvw = shape.n_kv_heads * shape.head_dim
    n_layers = shape.n_layers
    # a step is one decoder layer of one decode token; every 28th also runs the
    # head, so 28 steps are one full token (bounded so K=256 stays ~minutes)
    total = args.warmup + args.steps
    layers = []
    for i, w in enumerate(m.layers):
        L = oracle.RefLayer(w, cfg, PROMPT + total // n_layers + 2)
        L.fill_cache(np.random.default_rng(i).standard_normal(PROMPT * kvw).astype(np.float32),
                     np.random.default_rng(100 + i).standard_normal(PROMPT * kvw).astype(np.float32))
        layers.append(L)
    h = oracle.embed(m.embd["packed"], [1], shape.hidden)

    def step(s):
        nonlocal h
        h = layers[s % n_layers].forward(h, 1)
        if s % n_layers == n_layers - 1:
            tok, _, _ = oracle.head(h, m.output_norm, m.embd["packed"], shape.vocab, shape.hidden)
            h = oracle.embed(m.embd["packed"], [tok], shape.hidden)

    for s in range(args.warmup):
        step(s)
    t0 = time.perf_counter()
    for s in range(args.warmup, total):
        step(s)
    dt = time.perf_counter() - t0
    tok_s = (args.steps / n_layers) / dt
    sample = (f"{args.steps} decoder-layer steps ({args.steps / n_layers:.2f} tokens) of the "
              f"28-layer model at position {PROMPT}, oracle/flock_oracle.c on {cores} threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1000 / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config 2: Qwen3-0.6B-shape Q8_0, 28 layers, tied 151936x1024 "
                               "head, prompt 64, greedy bs1 decode", "seed": SEED},
        "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference's own CPU path is TypeScript under Deno; Deno and every JS engine "
                "are absent here, so its C restatement (same operation order) is timed",
    }), flush=True)


# --------------------------------------------------------------- GPU arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="flock", choices=["flock", "reference"])
    ap.add_argument("--attention", default="fast", choices=["fast", "exact"])
    ap.add_argument("--decode", default="kernels", choices=["stream", "persistent", "kernels"],
                    help="kernels: the per-op kernel graph (default, the fastest measured); "
                         "stream: one cooperative kernel per token for the layers with the "
                         "weights streamed through shared-memory rings, then the head GEMV; "
                         "persistent: the kernel graph's kernels as phases of one cooperative "
                         "kernel")
    ap.add_argument("--also-stream", action=argparse.BooleanOptionalAction, default=True,
                    help="also time the streaming engine on the same workload (its own key)")
    ap.add_argument("--also-tp", action=argparse.BooleanOptionalAction, default=True,
                    help="N > 1 pipeline runs: also time the tensor-parallel path on the same "
                         "GPUs and report it as the line's tensor_parallel key")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the config 3 (512-token prefill) measurement")
    ap.add_argument("--parallel", default="pipeline", choices=["pipeline", "tensor"],
                    help="N > 1 (or --parallel tensor at N = 1): layer-range pipeline stages "
                         "(config 2 / 4a) or tensor-sharded layers and head (config 4b)")
    ap.add_argument("--shape", default="0.6b", choices=["0.6b", "8b"],
                    help="Qwen3-0.6B shape (configs 1-3) or Qwen3-8B shape (config 4)")
    ap.add_argument("--allocate", action="store_true",
                    help="pipeline stages from the makespan allocator fed by each GPU's measured "
                         "bytes/ms (rank 0 charged for its head), instead of config 2's 4 + even")
    ap.add_argument("--prompt", type=int, default=None,
                    help="prompt tokens before the timed decode (default 64; 4096 for 8b); "
                         "longer prompts prefill on the tensor cores")
    ap.add_argument("--min-timed-s", type=float, default=1.5,
                    help="repeat the K-step window (untimed rewind between) until the timed "
                         "windows add up to this many seconds")
    ap.add_argument("--no-oracle-ids", action="store_true",
                    help="skip checking the first decode ids against the CPU oracle")
    ap.add_argument("--sweep", action=argparse.BooleanOptionalAction, default=True,
                    help="config 1: the Q8_0/Q4_0 GEMV and tensor-core GEMM sweep (L2 flushed "
                         "before every timed launch)")
    ap.add_argument("--kv", default="f32", choices=["f32", "bf16", "fp8"],
                    help="KV cache element type (bf16 / fp8: a half / a quarter of the KV "
                         "bytes per token; the tensor-core prefill and split-K decode "
                         "attention)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    from flock_b200 import synth
    from flock_b200.layer import QWEN3_06B
    from flock_b200.lib import get_device
    from flock_b200.model import Model
    from flock_b200 import ops

    shape = synth.QWEN3_8B if args.shape == "8b" else synth.QWEN3_06B
    dev = get_device(local)
    pk = peaks()
    if args.parallel == "tensor":
        run_tensor(args, rank, world, local, dev, shape, pk)
        return
    if args.shape == "8b" and world == 1:
        raise SystemExit("--shape 8b runs as config 4: give --parallel tensor, or --gpus N > 1")
    t_gen = time.perf_counter()
    m = synth.model(SEED, shape, lazy=args.shape == "8b")
    log(f"[rank {rank}] synthetic model generated in {time.perf_counter() - t_gen:.1f}s")
    n_prompt = args.prompt if args.prompt is not None else PROMPT
    max_keys = n_prompt + args.warmup + args.steps + 8
    cfg = QWEN3_06B.with_(max_keys=max(max_keys, 512), attention=args.attention)
    if args.kv != "f32" or n_prompt > 512:
        cfg = cfg.with_(prefill="tensor", kv=args.kv)
    if args.shape == "8b":
        cfg = cfg.with_(hidden=shape.hidden, n_heads=shape.n_heads, n_kv_heads=shape.n_kv_heads,
                        ffn=shape.ffn)
    prompt = synth.uniform_ids(SEED, "prompt", n_prompt, shape.vocab)

    if world > 1:
        run_pipeline(args, rank, world, local, dev, m, shape, cfg, prompt, pk)
        return

    M = Model.create(dev, m, cfg)
    M.decode_mode = args.decode
    decode = M.decode_mode                # "kernels" when the shape rules the chosen engine out
    first = M.step(prompt)                # prefill (untimed)
    M.decode_device(args.warmup)          # warm-up steps
    M.rewind(n_prompt)
    M.set_token(first)
    dev.sync()

    # The timed region: windows of exactly K device-fed steps (positions
    # n_prompt .. n_prompt+K-1), each bracketed by CUDA events, repeated after
    # an untimed rewind until the windows add up to >= min_timed_s, so the
    # 200 ms clock sampler sees the GPU under load.
    clk = Clocks(gpu_index(local))
    clk.start()
    window_ms, ids_dev = [], None
    while True:
        dev.timer_start()
        ids_w = M.decode_device(args.steps)
        window_ms.append(dev.timer_stop())
        if ids_dev is None:
            ids_dev = ids_w
        windows_same = bool(np.array_equal(ids_w, ids_dev))
        if not windows_same or sum(window_ms) >= 1000.0 * args.min_timed_s:
            break
        M.rewind(n_prompt)
        M.set_token(first)
    clocks = clk.stop()
    ms = sum(window_ms) / len(window_ms)   # per K-step window
    tok_s = args.steps / (ms / 1000.0)
    log(f"decode: {len(window_ms)} windows of {args.steps} tokens, {ms:.3f} ms per window -> "
        f"{tok_s:.1f} tok/s; clocks {clocks}")
    stream_line = None
    if args.also_stream and decode != "stream":
        # the streaming engine on the same model and positions, its own windows
        M.decode_mode = "stream"
        if M.decode_mode == "stream":
            M.rewind(n_prompt)
            M.set_token(first)
            M.decode_device(args.warmup)
            sw = []
            ids_s = None
            while sum(sw) < 1000.0 * args.min_timed_s / 2:
                M.rewind(n_prompt)
                M.set_token(first)
                dev.timer_start()
                ids_w = M.decode_device(args.steps)
                sw.append(dev.timer_stop())
                ids_s = ids_w if ids_s is None else ids_s
            ms_s = sum(sw) / len(sw)
            stream_line = {"value": args.steps / (ms_s / 1000.0), "unit": "tok/s",
                           "ms_per_step": ms_s / args.steps, "windows": len(sw),
                           "ids_match_kernels": bool(np.array_equal(ids_s, ids_dev)),
                           "engine": "k_decode_stream (28 layers, one cooperative launch) + "
                                     "the head k_gemv launch"}
            log(f"stream engine: {stream_line}")
        M.decode_mode = decode
        M.rewind(n_prompt)
        M.set_token(first)
    ids_oracle = None
    if not args.no_oracle_ids:
        n_chk = min(4, args.steps)
        ids_oracle = oracle_ids(m, shape, prompt, n_chk + 1, kv=args.kv)
        ids_match = ids_oracle == [first] + ids_dev[:n_chk].tolist()
        log(f"oracle ids {ids_oracle}: match {ids_match}")

    # end to end through the public API, host loop
    e2e = None
    if not args.no_e2e:
        M.rewind(n_prompt)
        prev = first
        ids_api = []
        dev.timer_start()
        for _ in range(args.steps):
            prev = M.step([prev])
            ids_api.append(prev)
        ms_e2e = dev.timer_stop()
        e2e = {"value": args.steps / (ms_e2e / 1000.0), "unit": "tok/s",
               "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
               "ids_match_device_loop": ids_api == ids_dev.tolist()}
        log(f"e2e: {e2e}")

    # The Q8_0 GEMV at its largest launch (the tied 151936 x 1024 LM head),
    # timed alone with CUDA events: the dominant kernel of the per-op graph.
    embd_t = M._keep[1]
    head_ms = ops.matvec_timed(dev, embd_t, 1, 50)
    head_bytes = shape.vocab * shape.hidden * 1.0625 + 4 * shape.hidden + 4 * shape.vocab
    head_gbs = head_bytes / (head_ms / 1000.0) / 1e9
    avg_keys = n_prompt + (args.steps - 1) / 2.0 + 1
    kv_elem = {"bf16": 2, "fp8": 1}.get(args.kv, 4)
    tok_bytes = bytes_per_token(shape, avg_keys, kv_elem)
    token_gbs = tok_bytes * tok_s / 1e9
    # roofline: the whole decode token -- every weight byte and K/V row it
    # reads (bytes_per_token) over the measured time per token; for the
    # single-launch engines that is exactly one kernel launch
    if decode in ("stream", "persistent"):
        launches_per_token = 1
        kernel = ("k_decode_stream, one cooperative launch per token (weights streamed "
                  "through shared-memory rings)" if decode == "stream" else
                  "k_decode_mk, one cooperative launch per token")
        traffic = traffic_from_profile(f"decode_{decode}_traffic.txt")
    else:
        launches_per_token = 1 + shape.n_layers * (5 if args.attention == "fast" else 6) + 2
        kernel = (f"the kernel graph's {launches_per_token} launches per token (k_embed, "
                  "per layer 4 k_gemv + attention, head k_gemv + argmax, k_record)")
        traffic = None
    roofline = {"bound": "hbm", "achieved": token_gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": token_gbs / pk["hbm_gbs"], "traffic": traffic, "kernel": kernel,
                "bytes_per_launch": tok_bytes / launches_per_token if launches_per_token == 1
                else None,
                "bytes_per_token": tok_bytes, "ms_per_token": ms / args.steps,
                "peak_src": pk["src"], "peak_note": "measured copy bandwidth (burst)"}

    out = {
        "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": ("config 2: Qwen3-0.6B-shape Q8_0, 28 layers, tied 151936x1024 "
                                "head, prompt 64 then greedy bs1 decode at positions 64.."
                                if n_prompt == PROMPT and args.kv == "f32" else
                                f"long-context decode: Qwen3-0.6B-shape Q8_0, 28 layers, tied "
                                f"head, {args.kv} KV cache, prompt {n_prompt} then greedy bs1 "
                                f"decode at positions {n_prompt}.."),
                   "seed": SEED, "prompt": n_prompt, "attention": args.attention,
                   "kv": args.kv, "decode": decode,
                   "l2": "inputs larger than L2: 692 MB of weights streamed per token",
                   "timing": f"CUDA events around each window of K device-fed decode "
                             f"steps; {len(window_ms)} windows (untimed rewind between) so the "
                             f"timed region spans {sum(window_ms) / 1000:.2f} s",
                   "windows": len(window_ms), "windows_same_ids": windows_same},
        "roofline": roofline,
        "head_gemv": {"achieved": head_gbs, "unit": "GB/s", "ms_per_launch": head_ms,
                      "frac": head_gbs / pk["hbm_gbs"],
                      "traffic": traffic_from_profile(),
                      "kernel": "k_gemv<Q8,R2,ARGMAX> on the 151936x1024 head timed alone"},
        "token_roofline": {"achieved": token_gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                           "frac": token_gbs / pk["hbm_gbs"],
                           "bytes_per_token": tok_bytes, "avg_keys": avg_keys},
        "clocks": clocks,
        "gpu_launches": launches_per_token * args.steps * len(window_ms),
    }
    if stream_line:
        out["stream_engine"] = stream_line
    if ids_oracle is not None:
        out["ids_match_oracle"] = ids_match
        out["ids_checked"] = len(ids_oracle)
    if args.sweep:
        out["config1_sweep"] = config1_sweep(dev, pk)
    if e2e:
        out["e2e"] = e2e
    if not args.no_prefill:
        out["prefill"] = prefill_ttft(dev, m, shape, pk)
    if not args.no_cpu_baseline:
        try:
            out["cpu_baseline"] = cpu_baseline(m, shape)
        except Exception as e:  # reported, not fatal
            out["cpu_baseline"] = {"value": None, "error": str(e)}
    print(json.dumps(out), flush=True)


def prefill_ttft(dev, m, shape, pk, n_prompt: int = 512) -> dict:
    """benchmark config 3: time to first token of a 512-token prompt on the same
    28-layer model through the tensor-core prefill (tcgen05 f16 GEMMs and
    attention), device-timed; the weight GEMMs' FLOPs over the TTFT give a
    lower bound on tensor-pipe use."""
    from flock_b200.layer import QWEN3_06B
    from flock_b200.model import Model
    from flock_b200 import synth
    cfg = QWEN3_06B.with_(attention="fast", prefill="tensor", max_keys=n_prompt + 64,
                          max_prefill=n_prompt)
    M = Model.create(dev, m, cfg)
    prompt = synth.uniform_ids(SEED, "prompt512", n_prompt, shape.vocab).tolist()
    M.step(prompt[:64])  # kernels loaded, workspaces touched
    M.reset()
    dev.sync()
    best = None
    for _ in range(3):
        dev.timer_start()
        first = M.step(prompt)
        ms = dev.timer_stop()
        M.reset()
        best = ms if best is None else min(best, ms)
    h, f = shape.hidden, shape.ffn
    q, kv = shape.n_heads * shape.head_dim, shape.n_kv_heads * shape.head_dim
    gemm_flops = 2.0 * n_prompt * shape.n_layers * (h * (q + 2 * kv) + q * h + 2 * h * f + f * h)
    tf = gemm_flops / (best * 1e-3) / 1e12
    M.free()
    return {"workload": "config 3: 512-token prompt, 28 layers, tcgen05 f16 prefill "
                        "(GEMMs + causal attention), first token greedy",
            "ttft_ms": best, "prompt_tok_s": n_prompt / (best * 1e-3), "first_id": first,
            "gemm_tflops_over_ttft": tf, "peak_tflops": pk["bf16_tflops"],
            "frac_of_peak": tf / pk["bf16_tflops"],
            "timing": "CUDA events, best of 3 prefills"}


def _max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0])


def run_tensor(args, rank, world, local, dev, shape, pk, emit: bool = True,
               pg_ready: bool = False):
    """Config 4b (and the 0.6B shape likewise): every layer and the head
    sharded over the N GPUs (flock_model_create_tp) -- QKV / gate / up by
    output rows, o_proj / down by input columns with an NCCL all-gather and a
    rank-order sum per projection, the head by vocab rows with an 8-byte
    (value, index) all-gather per token.  Decode steps replay one captured
    graph per rank, NCCL inside.  emit=False returns rank 0's line instead
    of printing it (the pipeline line carries it as a key); pg_ready: the
    caller owns the gloo process group."""
    from datetime import timedelta
    import torch.distributed as dist
    from flock_b200 import synth
    from flock_b200.comm import Comm
    from flock_b200.layer import LayerConfig
    from flock_b200.model import Model

    n_prompt = args.prompt if args.prompt is not None else (4096 if args.shape == "8b" else PROMPT)
    if world > 1 and not pg_ready:
        dist.init_process_group("gloo", timeout=timedelta(seconds=600))
    uid = Comm.unique_id() if rank == 0 else None
    if world > 1:
        obj = [uid]
        dist.broadcast_object_list(obj, src=0)
        uid = obj[0]
    comm = Comm(dev, world, rank, uid, 120000)
    cfg = LayerConfig(hidden=shape.hidden, n_heads=shape.n_heads, n_kv_heads=shape.n_kv_heads,
                      head_dim=shape.head_dim, ffn=shape.ffn,
                      max_keys=n_prompt + args.warmup + args.steps + 8, max_prefill=512,
                      attention=args.attention, prefill="tensor", kv=args.kv)
    t0 = time.perf_counter()
    m = synth.model(SEED, shape, lazy=True)
    M = Model.create_tp(dev, m, cfg, comm, rank, world)
    t_load = time.perf_counter() - t0
    log(f"[rank {rank}] tensor-parallel rank built in {t_load:.1f}s")
    prompt = synth.uniform_ids(SEED, "prompt", n_prompt, shape.vocab)
    # warm-up prefill: NCCL connects its channels on the first collectives
    M.step(prompt[:min(64, n_prompt)])
    M.reset()
    if world > 1:
        dist.barrier()
    dev.timer_start()
    first = M.step(prompt)                 # prefill on the tensor cores (untimed for value)
    ttft = _max_over_ranks(dev.timer_stop(), world)
    M.decode_device(args.warmup)
    M.rewind(n_prompt)
    M.set_token(first)
    dev.sync()
    if world > 1:
        dist.barrier()
    clk = Clocks(gpu_index(local))
    clk.start()
    dev.timer_start()
    ids_dev = M.decode_device(args.steps)
    ms = _max_over_ranks(dev.timer_stop(), world)
    clocks = clk.stop()
    # e2e: the public API's host loop, the id read back on every rank each token
    M.rewind(n_prompt)
    M.set_token(first)
    if world > 1:
        dist.barrier()
    dev.timer_start()
    prev, ids_api = first, []
    for _ in range(args.steps):
        prev = M.step([prev])
        ids_api.append(prev)
    ms_e2e = _max_over_ranks(dev.timer_stop(), world)
    if rank == 0:
        tok_s = args.steps / (ms / 1000.0)
        avg_keys = n_prompt + (args.steps - 1) / 2.0 + 1
        tok_bytes = bytes_per_token(shape, avg_keys, 2 if args.kv == "bf16" else 4)
        per_gpu = tok_bytes / world * tok_s / 1e9
        out = {
            "metric": METRIC.replace("0.6B", "8B") if args.shape == "8b" else METRIC,
            "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"config 4b: Qwen3-{'8B' if args.shape == '8b' else '0.6B'}"
                                   f"-shape Q8_0, {shape.n_layers} layers, tensor-sharded over "
                                   f"{world} GPU(s): QKV/gate/up by rows, o_proj/down by "
                                   "columns with an NCCL all-gather + rank-order sum, head by "
                                   "vocab rows with a (value, index) all-gather",
                       "seed": SEED, "prompt": n_prompt, "attention": args.attention,
                       "kv": args.kv, "parallelism": f"tp{world}",
                       "tp_exchange": M.tp_exchange,
                       "collectives_per_token": 2 * shape.n_layers + 1,
                       "l2": "inputs larger than L2: weights streamed per token",
                       "timing": "CUDA events around K device-fed decode steps, max over ranks"},
            "roofline": {"bound": "hbm", "achieved": per_gpu, "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": per_gpu / pk["hbm_gbs"], "traffic": None,
                         "kernel": "whole token per GPU: its 1/N of every weight and KV byte",
                         "bytes_per_launch": tok_bytes / world, "peak_src": pk["src"]},
            "clocks": clocks,
            "e2e": {"value": args.steps / (ms_e2e / 1000.0), "unit": "tok/s",
                    "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                    "ids_match_device_loop": ids_api == ids_dev.tolist()},
            "ids": ids_dev.tolist(),
            "prefill": {"ttft_ms": ttft, "prompt": n_prompt, "path": "tcgen05 f16, tensor-sharded"},
            "gpu_launches": (1 + shape.n_layers * ((5 if args.attention == "fast" else 6) + 2) + 4)
            * args.steps,
            "load_s": t_load,
        }
        if emit:
            print(json.dumps(out), flush=True)
    M.free()  # the captured graph holds NCCL calls: release it before the communicator
    comm.free()
    if world > 1:
        dist.barrier()
        if not pg_ready:
            dist.destroy_process_group()
    return out if rank == 0 else None


def run_pipeline(args, rank, world, local, dev, m, shape, cfg, prompt, pk):
    import ctypes
    import torch.distributed as dist
    from datetime import timedelta
    from flock_b200 import _abi
    from flock_b200.layer import upload_layer
    from flock_b200.pipeline import stage_ranges
    from flock_b200.lib import GpuTensor
    from flock_b200.model import Model

    n_prompt = len(prompt)
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    uid = np.zeros(128, np.uint8)
    if rank == 0:
        _abi.call("flock_comm_unique_id", _abi.ptr(uid, _abi._u8p))
    obj = [uid.tobytes()]
    dist.broadcast_object_list(obj, src=0)
    uid = np.frombuffer(obj[0], np.uint8).copy()
    comm = ctypes.c_void_p()
    _abi.call("flock_comm_init", dev.handle, world, rank, _abi.ptr(uid, _abi._u8p), 60000,
              ctypes.byref(comm))
    ranges = stage_ranges(shape.n_layers, world)
    if args.allocate:
        # server/allocate.js fed by measurement: every rank's streaming rate,
        # rank 0 charged the time of the head it also runs
        from flock_b200.allocate import Device, allocate, layer_plan, measure_rate
        from flock_b200 import ops
        rate = measure_rate(dev)
        reserved = 0.0
        if rank == 0:
            ht = GpuTensor.from_packed(dev, m.embd["packed"], m.embd["rows"], m.embd["cols"])
            reserved = ops.matvec_timed(dev, ht, 1, 20)
            ht.free()
        got = [None] * world
        dist.all_gather_object(got, (rate, reserved))
        devs = [Device(f"gpu{r}", rate=got[r][0], reserved_ms=got[r][1]) for r in range(world)]
        ranges = allocate(layer_plan(m), devs).ranges()
    a, b = ranges[rank]
    layer_ts = [upload_layer(dev, m.layers[i]) for i in range(a, b)]
    if rank == 0:
        embd = GpuTensor.from_packed(dev, m.embd["packed"], m.embd["rows"], m.embd["cols"])
        onorm = GpuTensor.from_f32(dev, m.output_norm)
        head = None
        if m.output is not None:
            head = GpuTensor.from_packed(dev, m.output["packed"], m.output["rows"],
                                         m.output["cols"])
        M = Model.from_tensors(dev, cfg, shape.vocab, b - a, layer_ts, embd, onorm, head)
    else:
        M = Model.from_tensors(dev, cfg, shape.vocab, b - a, layer_ts, None, None)
    nxt = ctypes.c_int32()

    def pstep(ids, n, sync):
        p = None
        if ids is not None:
            arr = np.ascontiguousarray(ids, np.int32)
            pstep.keep = arr
            p = _abi.ptr(arr, _abi._i32p)
        _abi.call("flock_pipeline_step", M.handle, comm, p, n, sync, ctypes.byref(nxt))

    pstep(prompt if rank == 0 else None, n_prompt, 1)
    first = nxt.value
    for _ in range(args.warmup):
        pstep(None, 1, 0)
    dev.sync()
    M.rewind(n_prompt)
    if rank == 0:
        M.set_token(first)
    dist.barrier()
    import torch
    # windows of exactly K device-fed steps (the chosen id stays on rank 0's
    # device; no rank waits on its host inside a window), repeated after an
    # untimed rewind until they add up to min_timed_s; each window's time is
    # the max over ranks, so every rank takes the same decision to go on
    clk = Clocks(gpu_index(local))
    clk.start()
    window_ms, ids_dev = [], None
    while True:
        dev.timer_start()
        for _ in range(args.steps):
            pstep(None, 1, 0)
        w_ms = dev.timer_stop()
        tt = torch.tensor([w_ms], dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        window_ms.append(float(tt[0]))
        if ids_dev is None and rank == 0:
            ids_dev = np.zeros(args.steps, np.int32)
            _abi.call("flock_model_history", M.handle, n_prompt, args.steps,
                      _abi.ptr(ids_dev, _abi._i32p))
        if sum(window_ms) >= 1000.0 * args.min_timed_s:
            break
        M.rewind(n_prompt)
        if rank == 0:
            M.set_token(first)
        dist.barrier()
    clocks = clk.stop()
    ms_max = sum(window_ms) / len(window_ms)

    # e2e: host loop through the API, id read back on rank 0 every token
    M.rewind(n_prompt)
    if rank == 0:
        M.set_token(first)
    dist.barrier()
    dev.timer_start()
    prev = first
    for _ in range(args.steps):
        pstep([prev] if rank == 0 else None, 1, 1)
        prev = nxt.value
    ms_e2e = dev.timer_stop()
    tt = torch.tensor([ms_e2e], dtype=torch.float64)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms_e2e = float(tt[0])
    ids_api = []
    if rank == 0:
        ids_api = np.zeros(args.steps, np.int32)
        _abi.call("flock_model_history", M.handle, n_prompt, args.steps,
                  _abi.ptr(ids_api, _abi._i32p))
    dist.barrier()
    _abi.lib().flock_comm_free(comm)
    M.free()
    for lt in layer_ts:
        for t in lt.values():
            t.free()

    # the same decode on one GPU (rank 0, the whole model, same positions):
    # the ids the pipeline must reproduce, and the per-token time the hops add to
    one_gpu = None
    if rank == 0:
        M1 = Model.create(dev, m, cfg)
        f1 = M1.step(prompt)
        M1.decode_device(args.warmup)
        M1.rewind(n_prompt)
        M1.set_token(f1)
        dev.sync()
        dev.timer_start()
        ids_1 = M1.decode_device(args.steps)
        ms_1 = dev.timer_stop()
        M1.free()
        hop_us = (ms_max - ms_1) / args.steps * 1000.0 / world
        one_gpu = {"ms_per_step": ms_1 / args.steps, "first_id": int(f1),
                   "ids_match": f1 == first and ids_1.tolist() == ids_dev.tolist(),
                   "hop_us_est": hop_us}
        log(f"one GPU: {one_gpu}")
    dist.barrier()

    # the tensor-parallel path on the same N GPUs (config 4b's form at this
    # shape), reported as a key of this line
    tp_line, tp_error = None, None
    if args.also_tp and shape.n_layers == 28:
        try:
            tp_line = run_tensor(args, rank, world, local, dev, shape, pk, emit=False,
                                 pg_ready=True)
        except Exception as e:  # the pipeline line stands on its own
            tp_error = f"{type(e).__name__}: {e}"[:300]
            log(f"[rank {rank}] tensor-parallel run failed: {tp_error}")
        dist.barrier()
    if rank == 0:
        ids_oracle, ids_match = None, None
        if not args.no_oracle_ids:
            n_chk = min(4, args.steps)
            ids_oracle = oracle_ids(m, shape, prompt, n_chk + 1)
            ids_match = ids_oracle == [first] + ids_dev[:n_chk].tolist()
            log(f"oracle ids {ids_oracle}: match {ids_match}")
        tok_s = args.steps / (ms_max / 1000.0)
        avg_keys = n_prompt + (args.steps - 1) / 2.0 + 1
        tok_bytes = bytes_per_token(shape, avg_keys, 2 if args.kv == "bf16" else 4)
        token_gbs = tok_bytes * tok_s / 1e9
        out = {
            "metric": METRIC.replace("0.6B", "8B") if shape.n_layers == 36 else METRIC,
            "value": tok_s, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": f"config {'4a (8B shape)' if shape.n_layers == 36 else '2'} "
                                   "pipelined: contiguous layer ranges "
                                   f"{ranges}{' (allocator)' if args.allocate else ''}, "
                                   "hidden state over "
                                   "NCCL send/recv", "seed": SEED, "prompt": n_prompt,
                       "attention": args.attention, "kv": args.kv,
                       "parallelism": f"pp{world}", "l2": "inputs larger than L2",
                       "timing": f"CUDA events around each window of K device-fed steps, max "
                                 f"over ranks; {len(window_ms)} windows (untimed rewind between)",
                       "windows": len(window_ms)},
            "limit": {"collective": "NCCL send/recv of one token's hidden state, one hop per "
                                    "stage boundary and one back to rank 0 (N hops per token); "
                                    "batch 1 keeps one stage busy at a time",
                      "hops_per_token": world,
                      "hop_us_est": one_gpu["hop_us_est"],
                      "hop_share": world * one_gpu["hop_us_est"] / 1000.0 / (ms_max / args.steps),
                      "how": "(pipeline ms/token - one GPU's ms/token on the same model and "
                             "positions, rank 0) / hops"},
            "one_gpu": one_gpu,
            # batch 1 keeps one stage busy at a time: the roofline is one GPU's
            "roofline": {"bound": "hbm", "achieved": token_gbs, "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": token_gbs / pk["hbm_gbs"], "traffic": None,
                         "kernel": "whole token across the pipeline stages",
                         "bytes_per_launch": tok_bytes, "peak_src": pk["src"]},
            "clocks": clocks,
            "e2e": {"value": args.steps / (ms_e2e / 1000.0), "unit": "tok/s",
                    "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                    "ids_match_device_loop": ids_api.tolist() == ids_dev.tolist()},
            "gpu_launches": (1 + shape.n_layers * (5 if args.attention == "fast" else 6) + 2)
            * args.steps * len(window_ms),
        }
        if ids_oracle is not None:
            out["ids_match_oracle"] = ids_match
            out["ids_checked"] = len(ids_oracle)
        if tp_error:
            out["tensor_parallel"] = {"error": tp_error}
        if tp_line:
            out["tensor_parallel"] = {k: tp_line[k] for k in
                                      ("value", "unit", "ms_per_step", "e2e", "roofline",
                                       "prefill") if k in tp_line}
            out["tensor_parallel"]["parallelism"] = tp_line["config"]["parallelism"]
            out["tensor_parallel"]["tp_exchange"] = tp_line["config"]["tp_exchange"]
            # tensor parallelism sums the o_proj / down partials in rank order
            # (shardReduceRef), so its bits differ from one GPU's fold: equal
            # greedy ids are expected, not guaranteed
            out["tensor_parallel"]["ids_match_pipeline"] = tp_line.get("ids") == ids_dev.tolist()
        print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
