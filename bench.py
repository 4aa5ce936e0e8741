"""Decode throughput benchmark: Llama-3-8B architecture, Q4_K_M layout, batch-1
greedy decode on 1/2/4/8 B200 (tensor parallel, one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...

A step is one decode token: one forward of the whole model for one token at the
next position plus the greedy argmax. Workload (the benchmark's configuration
for this metric): random-init Llama-3-8B (seed 2, Q4_K layer matrices, Q6_K
embedding and head), context 4096, a 512-token random prompt prefilled in
batches of 128 (untimed), then decode steps from position 512.

  value  tokens/s of the device-resident decode loop (wgd_decode: each step's
         argmax feeds the next on the device), CUDA events, max over ranks.
  e2e    tokens/s through the per-token C-ABI call (wgd_forward) with the token
         id copied in from pinned host memory and the greedy id read back every
         step, wall clock around the loop, max over ranks.
  roofline  the persistent decode kernel over whole steps: algorithmic bytes
         per step (weights + KV) / step time vs the measured HBM peak; the
         stand-alone gate|up Q4_K GEMV (28672 x 4096) as gemv_probe.
  prefill  the 512-token prompt prefilled again in batches of 128 (device
         time, max over ranks): every Q4_K projection runs on the tcgen05
         GEMM; projection TFLOP/s against the measured bf16 tensor peak.
  sampled  the same decode with the reference's default draw (temperature 0.7,
         topK 40, topP 0.9, seeded uniforms) on the device: wgd_decode_sample
         (device time) and wgd_forward_sample per token (wall clock).
  cpu_baseline  the CPU restatement of the reference decoder (oracle/, float64)
         on a bounded sample of the same model, rank 0 only.
  qwen2_5_0_5b  the benchmark's Qwen2.5-0.5B configuration (23-token prompt, then
         128 greedy tokens of the device decode loop) with its own roofline
         fraction, one GPU only; reported beside the headline metric.

--impl reference times that CPU path (the reference's own implementation is
TypeScript/WebGPU, which has neither a runtime nor a graphics stack here) on
all host cores and prints the same line with impl=reference.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "decode tok/s Llama-3-8B Q4_K_M"
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) from ncu captures of the same kernels:
# the stand-alone GEMV at 28672x4096 (one launch), and the persistent kernel on the 4-layer
# Llama-3-8B-width model (two decode steps: 1.879 GB against 2 x 0.938 GB algorithmic) scaled to
# one full 32-layer step by the algorithmic bytes (4.50 GB / 0.938 GB).
GEMV_TRAFFIC = 66_133_760
STEP_TRAFFIC = 4_500_000_000
CONTEXT, PREFILL_BATCH, PROMPT = 4096, 128, 512


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16 TFLOP/s (burst) of MEASURED_PEAKS.json, else the fallback figure."""
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def projection_flops(c, tokens: int, world: int) -> float:
    """2 * tokens * (elements of every layer projection) / world: the prefill GEMM work."""
    H, hd = c.hidden, c.head_dim
    q, kv = c.heads * hd, c.kv_heads * hd
    per_layer = H * (q + 2 * kv) + q * H + 2 * H * c.intermediate + c.intermediate * H
    return 2.0 * tokens * per_layer * c.layers / world


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) >= 9:
                    rows.append(f)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------------- model

def build_model(layers=None):
    from webgpu_b200 import synth
    t0 = time.time()
    spec = synth.baseline_spec(3, layers=layers)
    image = synth.build_gguf(spec)
    log(f"[bench] synthetic Llama-3-8B GGUF: {image.nbytes / 1e9:.2f} GB in {time.time() - t0:.1f}s")
    return spec, image


def weight_bytes(gguf, config):
    """Algorithmic weight bytes of one decode token (every matrix once, embedding one row)."""
    total = 0
    for t in gguf.tensors.values():
        if t.name == "token_embd.weight":
            total += t.row_bytes
        elif len(t.dims) == 2 or t.dims[0] > 1:
            total += t.bytes
    return total


def qwen_config(device: int, steps: int = 128) -> dict:
    """The benchmark's Qwen2.5-0.5B configuration (qwen2 blocks with Q/K/V bias, hidden 896, 24 layers,
    14/2 heads, tied Q6_K embedding, seed 1): a 23-token prompt prefilled in one batch of 32, then `steps`
    greedy tokens of the device decode loop (CUDA events), resident on one GPU. Reported beside the
    headline metric, not as it."""
    from webgpu_b200 import _native, synth
    from webgpu_b200.engine import PagedEngine
    from webgpu_b200.source import MemorySource
    spec = synth.baseline_spec(2)
    image = synth.build_gguf(spec)
    eng = PagedEngine()
    eng.load(MemorySource(image), {"contextLength": 512, "batchSize": 32, "performance": "fast", "device": device})
    L = _native.lib()
    try:
        prompt = list(spec.prompt)
        tok = eng.forward(prompt, 0, True)
        buf = (ctypes.c_int32 * steps)()
        _native.check(L.wgd_decode(eng.ctx, tok, len(prompt), steps, buf), "decode")  # warm-up (graph capture)
        _native.check(L.wgd_decode(eng.ctx, tok, len(prompt), steps, buf), "decode")
        st = _native.StatsC()
        L.wgd_stats_get(eng.ctx, ctypes.byref(st))
        why = ctypes.create_string_buffer(256)
        persistent = L.wgd_persistent_status(eng.ctx, why, 256) == 1
        c = eng.config
        step_ms = st.last_forward_ms / steps
        kv = 2 * c.kv_heads * c.head_dim * 4 * c.layers * (len(prompt) + steps / 2)
        step_bytes = weight_bytes(eng.gguf, c) + kv
        peak, kind = peaks()
        achieved = step_bytes / (step_ms / 1000) / 1e9
        return {"workload": "Qwen2.5-0.5B arch Q4_K_M (Q4_0 / Q8_0 where a row width is not a multiple of 256), 23-token prompt "
                            "in one batch of 32, then batch-1 greedy decode",
                "steps": steps, "tok_per_s": steps / (st.last_forward_ms / 1000.0), "ms_per_step": step_ms,
                "algorithmic_bytes": step_bytes, "achieved_gbs": achieved, "frac": achieved / peak,
                "peak_kind": kind, "path": "persistent kernel" if persistent else f"per-kernel CUDA graph ({why.value.decode()})"}
    finally:
        eng.dispose()


# ------------------------------------------------------------- roofline probe

def gemv_probe(device: int, rows=28672, cols=4096, launches=40):
    """Average duration of the dominant GEMV (Q4_K, gate|up fused shape) over
    weight copies that together exceed L2, CUDA events on the launching stream."""
    import torch
    from webgpu_b200 import _native, synth
    L = _native.lib()
    ttype = synth.Q4_K
    raw = synth.random_blocks(ttype, rows * cols // 256, seed=2, stream=99)
    nbytes = L.wgd_tiled_bytes(ttype, rows, cols)
    copies = max(2, int(np.ceil(300e6 / nbytes)))  # > 126 MB L2 in total
    raw_d = torch.from_numpy(raw).to(f"cuda:{device}")
    mats = []
    for _ in range(copies):
        m = torch.empty(nbytes + 16, dtype=torch.uint8, device=f"cuda:{device}")
        _native.check(L.wgd_op_repack_tiled(ttype, rows, cols, raw_d.data_ptr(), m.data_ptr(), None))
        mats.append(m)
    del raw_d
    x = torch.randn(cols, device=f"cuda:{device}")
    y = torch.empty(rows, device=f"cuda:{device}")
    stream = torch.cuda.current_stream(device)
    sp = ctypes.c_void_p(stream.cuda_stream)
    for i in range(3 * copies):
        _native.check(L.wgd_op_gemv_tiled(ttype, rows, cols, mats[i % copies].data_ptr(), x.data_ptr(), 1, y.data_ptr(), sp))
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(launches):
        _native.check(L.wgd_op_gemv_tiled(ttype, rows, cols, mats[i % copies].data_ptr(), x.data_ptr(), 1, y.data_ptr(), sp))
    e1.record(stream)
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / launches
    alg = rows * cols // 256 * 144 + (cols + rows) * 4
    return ms, alg


# ------------------------------------------------------------- CPU baseline

def cpu_baseline(image, threads: int, budget_s: float = 20.0):
    """The float64 CPU decoder (oracle restatement of the reference's CPU path) on a
    bounded sample: decode steps from position 0 of the same model, timed per token."""
    import oracle
    from webgpu_b200.gguf import model_config, parse_gguf_header
    g = parse_gguf_header(image, image.nbytes)
    c = model_config(g)
    dec = oracle.Decoder(image, g, c, context=64, threads=threads)
    t0 = time.perf_counter()
    dec.forward([1], 0)
    per = time.perf_counter() - t0
    n = 1
    while n < 8 and (time.perf_counter() - t0) + per < budget_s:
        dec.forward([2 + n], n)
        n += 1
    dt = time.perf_counter() - t0
    dec.close()
    return n / dt, n


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ------------------------------------------------------------------ main

def run_reference(args, rank, world):
    """--impl reference: the CPU restatement on all host threads, same metric."""
    if rank != 0:
        return
    _, image = build_model()
    threads = cpu_threads()
    steps, warm = max(1, min(args.steps, 4)), max(0, min(args.warmup, 1))
    import oracle
    from webgpu_b200.gguf import model_config, parse_gguf_header
    g = parse_gguf_header(image, image.nbytes)
    c = model_config(g)
    dec = oracle.Decoder(image, g, c, context=64, threads=threads)
    for i in range(warm):
        dec.forward([1 + i], i)
    t0 = time.perf_counter()
    for i in range(steps):
        dec.forward([5 + i], warm + i)
    dt = time.perf_counter() - t0
    dec.close()
    v = steps / dt
    sample = f"{steps} decode steps (after {warm} warm-up) of the full model at positions {warm}..{warm + steps - 1}, f64"
    line = {"metric": METRIC, "value": v, "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * dt / steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded random-init weights)",
            "config": {"workload": "Llama-3-8B arch Q4_K_M, batch-1 greedy decode (CPU sample)", "threads": threads},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=None, help="trim depth (debug only; not a valid bench number)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
        dist = tdist

    if args.impl == "reference":
        run_reference(args, rank, world)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return

    import torch
    from webgpu_b200 import _native
    from webgpu_b200.engine import PagedEngine
    from webgpu_b200.source import MemorySource
    torch.cuda.set_device(local)

    spec, image = build_model(args.layers)
    opts = {"contextLength": CONTEXT, "batchSize": PREFILL_BATCH, "performance": "fast", "gpuBudgetMiB": 40 * 1024,
            "tensorParallel": world, "rank": rank, "device": local}
    if dist:
        def exchange(b: bytes):
            out = [None] * world
            dist.all_gather_object(out, b)
            return out
        opts["exchange"] = exchange
    eng = PagedEngine()
    t0 = time.time()
    eng.load(MemorySource(image), opts)
    log(f"[bench] rank {rank}: loaded in {time.time() - t0:.1f}s; gpu bytes {eng.stats()['gpuBytes'] / 1e9:.2f} GB")
    L = _native.lib()
    c = eng.config

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if not dist:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # prefill the 512-token prompt in batches of 128 (untimed)
    prompt = spec.prompt[:PROMPT]
    t0 = time.perf_counter()
    tok = None
    for i in range(0, len(prompt), PREFILL_BATCH):
        chunk = prompt[i:i + PREFILL_BATCH]
        tok = eng.forward(chunk, i, i + len(chunk) == len(prompt))
    prefill_s = time.perf_counter() - t0
    pos = len(prompt)

    # ---- prefill again, device time (the tcgen05 GEMM carries every Q4_K projection of a
    # 128-row batch); the same tokens rewrite the same KV rows
    barrier()
    pf_ms = 0.0
    for i in range(0, len(prompt), PREFILL_BATCH):
        chunk = prompt[i:i + PREFILL_BATCH]
        eng.forward(chunk, i, i + len(chunk) == len(prompt))
        stp = _native.StatsC()
        L.wgd_stats_get(eng.ctx, ctypes.byref(stp))
        pf_ms += stp.last_forward_ms
    pf_ms = max_over_ranks(pf_ms)

    # warm-up of both paths
    buf = (ctypes.c_int32 * max(args.steps, args.warmup))()
    _native.check(L.wgd_decode(eng.ctx, tok, pos, args.warmup, buf), "decode")
    why = ctypes.create_string_buffer(256)
    persistent = L.wgd_persistent_status(eng.ctx, why, 256) == 1
    for i in range(args.warmup):
        eng.forward([int(buf[i])], pos + 1 + i, True)

    # ---- value: device-resident decode loop, K steps from position `start`
    start = pos
    barrier()
    with ClockSampler(local) as clk:
        st0 = _native.StatsC()
        L.wgd_stats_get(eng.ctx, ctypes.byref(st0))
        _native.check(L.wgd_decode(eng.ctx, tok, start, args.steps, buf), "decode")
        barrier()
        st = _native.StatsC()
        L.wgd_stats_get(eng.ctx, ctypes.byref(st))
        dev_ms = max_over_ranks(st.last_forward_ms)
        launches = int(st.kernel_launches - st0.kernel_launches)  # this library's kernels in the timed call
        # ---- e2e: per-token public C-ABI call with host buffers (same positions)
        barrier()
        t0 = time.perf_counter()
        cur = tok
        tokens_e2e = []
        for i in range(args.steps):
            cur = eng.forward([cur], start + i, True)
            tokens_e2e.append(cur)
        barrier()
        e2e_s = max_over_ranks(time.perf_counter() - t0)
    clocks = clk.summary()
    tokens_dev = [int(buf[i]) for i in range(args.steps)]

    # ---- sampled decode at the reference's default settings (temperature 0.7, topK 40, topP 0.9),
    # drawn on the device: the device loop (wgd_decode_sample) and the per-token public call
    # (wgd_forward_sample, token id in and out); the same seeded uniforms on every rank
    T, K, P = 0.7, 40, 0.9
    draws = np.random.default_rng(7).random(max(args.steps, args.warmup)).tolist()
    us = (ctypes.c_double * len(draws))(*draws)
    sbuf = (ctypes.c_int32 * len(draws))()
    _native.check(L.wgd_decode_sample(eng.ctx, tok, start, args.warmup, T, K, P, us, sbuf), "decode_sample")
    barrier()
    _native.check(L.wgd_decode_sample(eng.ctx, tok, start, args.steps, T, K, P, us, sbuf), "decode_sample")
    st = _native.StatsC()
    L.wgd_stats_get(eng.ctx, ctypes.byref(st))
    smp_ms = max_over_ranks(st.last_forward_ms)
    it = iter(draws)
    eng.random = lambda: next(it)
    barrier()
    t0 = time.perf_counter()
    cur = tok
    tokens_smp = []
    for i in range(args.steps):
        cur = eng.forward_sample([cur], start + i, T, K, P)
        tokens_smp.append(cur)
    barrier()
    smp_e2e_s = max_over_ranks(time.perf_counter() - t0)
    sampled = {"settings": {"temperature": T, "topK": K, "topP": P}, "tok_per_s": args.steps / (smp_ms / 1000.0),
               "ms_per_step": smp_ms / args.steps, "e2e_tok_per_s": args.steps / smp_e2e_s,
               "kernel": "sample_kernel (top-k by bitonic sort in shared memory, nucleus cut and draw in double) after "
                         "each decode step; no logits readback",
               "tokens_match_e2e": [int(sbuf[i]) for i in range(args.steps)] == tokens_smp}

    value = args.steps / (dev_ms / 1000.0)
    e2e = args.steps / e2e_s
    wbytes = weight_bytes(eng.gguf, c)
    kv_read = 2 * c.kv_heads * c.head_dim * 4 * c.layers * (start + args.steps / 2)  # average position
    step_bytes = (wbytes + kv_read) / world
    step_ms = dev_ms / args.steps
    peak, peak_kind = peaks()

    roof = None
    if rank == 0:
        ms, alg = gemv_probe(local)
        g_achieved = alg / (ms / 1000.0) / 1e9
        probe = {"kernel": "gemv2 Q4_K 28672x4096 batch 1 (stand-alone tiled GEMV)", "achieved": g_achieved,
                 "frac": g_achieved / peak, "launch_ms": ms, "algorithmic_bytes": alg, "traffic": GEMV_TRAFFIC}
        achieved = step_bytes / (step_ms / 1000) / 1e9
        roof = {"bound": "hbm", "unit": "GB/s", "peak": peak, "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                "kernel": ("persist_kernel: whole decode steps (all layers, LM head, argmax) in one launch" if persistent
                           else "per-kernel decode step (CUDA graph)"),
                "achieved": achieved, "frac": achieved / peak,
                "per": "decode step (one launch runs all timed steps)", "algorithmic_bytes": step_bytes, "ms": step_ms,
                "traffic": STEP_TRAFFIC if persistent else None, "launch_ms": dev_ms, "steps_per_launch": args.steps,
                "gemv_probe": probe}

    prefill = None
    if rank == 0:
        tpk, tpk_kind = tensor_peak()
        pf_flops = projection_flops(c, len(prompt), world)
        pf_tflops = pf_flops / (pf_ms / 1000.0) / 1e12
        prefill = {"tokens": len(prompt), "batch": PREFILL_BATCH, "ms": pf_ms, "tok_per_s": len(prompt) / (pf_ms / 1000.0),
                   "kernel": "gemm_tc_kernel (tcgen05.mma kind::f16 M128 N128, TMEM accumulators) for every Q4_K and Q6_K projection",
                   "projection_tflops": pf_tflops, "tensor_peak": tpk, "tensor_peak_kind": f"{tpk_kind} (bf16_tflops)",
                   "frac": pf_tflops / tpk,
                   "tensor_work_frac": 2 * pf_tflops / tpk,
                   "note": "whole forward (projections, attention, rope, norms) timed; FLOPs count the projections only; "
                           "tensor work is twice the algorithmic FLOPs (activation hi/lo split); ncu tensor-pipe "
                           "utilisation of the GEMM kernel: profiles/gemm_tc_q4k_28672x4096_b128.md"}

    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = cpu_threads()
        v, n = cpu_baseline(image, threads)
        base = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                "sample": f"{n} decode steps of the full model from position 0 (float64 oracle decoder, {threads} threads)"}

    if dist:
        dist.barrier()  # no rank frees its exchange buffers while a peer may still use them
    eng.dispose()
    qwen = None
    if rank == 0 and world == 1:
        try:
            qwen = qwen_config(local)
        except Exception as ex:  # reported in the line; the headline numbers above stand
            qwen = {"error": f"{type(ex).__name__}: {ex}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": step_ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights, GGUF Q4_K/Q6_K blocks)",
            "config": {"workload": "Llama-3-8B arch Q4_K_M, batch-1 greedy decode after a 512-token prompt",
                       "model": "llama-3-8b-arch", "context": CONTEXT, "prompt": PROMPT, "prefill_batch": PREFILL_BATCH,
                       "positions": [start, start + args.steps - 1], "parallelism": f"tp{world}",
                       "l2": "weights (4.36 GB) exceed L2 every step", "rope": "adjacent-pair (llama GGUF rule)",
                       "layers": c.layers, "prefill_s": prefill_s},
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4 + 4, "d2h_bytes_per_step": 4},
            "roofline": roof, "cpu_baseline": base, "clocks": clocks, "prefill": prefill, "sampled": sampled,
            "gpu_launches": launches,
            "tokens_match_e2e": tokens_dev == tokens_e2e,
            "qwen2_5_0_5b": qwen,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
