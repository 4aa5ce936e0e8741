"""Decode throughput benchmark: Llama-3-8B architecture, Q4_K_M layout, batch-1
greedy decode on 1/2/4/8 B200 (tensor parallel, one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...
    python bench.py --case NAME [ARGS...]      # one fixed profiling workload (see CASES)

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
  roofline  the decode kernel over whole steps: algorithmic bytes per step and
         rank (weights + KV) / step time vs the measured HBM peak; the
         stand-alone gate|up Q4_K GEMV (28672 x 4096) as gemv_probe.
  parity  the CPU oracle (float64 restatement of the reference decoder) and the
         GPU on the same token ids from position 0: a 4-token prompt, then 4
         greedy tokens; tokens, device-loop tokens and the max relative logit
         error (rank 0 of a tensor-parallel group).
  prefill  the 512-token prompt prefilled again in batches of 128 (device
         time, max over ranks): every Q4_K projection runs on the tcgen05
         GEMM; projection TFLOP/s against the measured bf16 tensor peak.
  sampled  the same decode with the reference's default draw (temperature 0.7,
         topK 40, topP 0.9, seeded uniforms) on the device: wgd_decode_sample
         (device time) and wgd_forward_sample per token (wall clock).
  cpu_baseline  the oracle's decode of the parity leg, timed (all host threads,
         and one forward on one thread), rank 0 of a one-GPU run.
  c2     the quantised GEMV / GEMM microbench of the benchmark's configuration list:
         Q4_K and Q6_K at 4096x4096, 14336x4096, 4096x14336, batch 1/8/32/128
         (one GPU only).
  qwen2_5_0_5b  the benchmark's Qwen2.5-0.5B configuration (23-token prompt, then
         128 greedy tokens of the device decode loop) with its own roofline
         fraction, one GPU only; reported beside the headline metric.

--impl reference times that CPU path (the reference's own implementation is
TypeScript/WebGPU, which has neither a runtime nor a graphics stack here) on
all host cores at the GPU arm's decode positions and prints the same line with
impl=reference; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "decode tok/s Llama-3-8B Q4_K_M"
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) from ncu captures of the same kernels:
# the stand-alone GEMV at 28672x4096 (one launch), and the persistent kernel on the 4-layer
# Llama-3-8B-width model (two decode steps: 1.878 GB read + 7.7 MB written against 2 x 0.938 GB
# algorithmic) scaled to one full 32-layer step by the algorithmic bytes (4.49 GB x 1.886 / 1.876).
GEMV_TRAFFIC = 66_133_760
STEP_TRAFFIC = 4_517_000_000
STEP_TRAFFIC_SOURCE = ("scaled: ncu dram__bytes_read.sum + dram__bytes_write.sum of persist_kernel on the 4-layer "
                       "model (2 steps, 1.886 GB vs 1.876 GB algorithmic), scaled to one 32-layer step by the "
                       "algorithmic bytes; the full model is too large to capture")
CONTEXT, PREFILL_BATCH, PROMPT = 4096, 128, 512
PARITY_PROMPT, PARITY_STEPS, LOGIT_TOL = 4, 4, 1e-3
Q4_K, Q6_K = 12, 14


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


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


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


def shared_model(layers, world, local, host_barrier):
    """The synthetic model, built once per node: local rank 0 generates it (every core) and writes it
    to a node-local file that the other ranks map read-only; one rank builds it in memory."""
    from webgpu_b200 import synth
    if world == 1:
        return build_model(layers)
    spec = synth.baseline_spec(3, layers=layers)
    tag = f"wgd_bench_llama3_8b_seed2_L{layers or 32}_{os.environ.get('MASTER_PORT', '0')}.gguf"
    base = "/dev/shm" if os.path.isdir("/dev/shm") and shutil.disk_usage("/dev/shm").free > 12e9 else tempfile.gettempdir()
    path = os.path.join(base, tag)
    image = None
    if local == 0:
        spec, image = build_model(layers)
        t0 = time.time()
        image.tofile(path + ".tmp")
        os.replace(path + ".tmp", path)
        log(f"[bench] model written to {path} in {time.time() - t0:.1f}s")
    host_barrier()
    if image is None:
        image = np.memmap(path, dtype=np.uint8, mode="r")
    return spec, image, path


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


def c2_table(device: int, launches: int = 24) -> dict:
    """The quantised GEMV/GEMM microbench: Q4_K and Q6_K blocks with the configuration's value
    distributions (fp16 scales |N(0, 1e-3)|, uniform quants; Q6_K int8 scales in [-32, 31]),
    out x in = 4096x4096, 14336x4096, 4096x14336, activations N(0, 1), batch 1/8/32/128. Each case
    is timed with CUDA events on the launching stream over weight copies that together exceed L2
    (every launch reads its weights from HBM). The kernel is the one the engine uses for that
    batch: the integer tensor-core GEMV below 16 rows, the tcgen05 GEMM from 16 rows on.
    Algorithmic bytes: out*in*bpw + batch*(in + out)*4; FLOPs 2*batch*out*in."""
    import torch
    from webgpu_b200 import _native, synth
    L = _native.lib()
    hbm, hbm_kind = peaks()
    tpk, tpk_kind = tensor_peak()
    dev = f"cuda:{device}"
    stream = torch.cuda.current_stream(device)
    sp = ctypes.c_void_p(stream.cuda_stream)
    bpw = {Q4_K: 144 / 256, Q6_K: 210 / 256}
    cases = []
    for ttype, tname in ((Q4_K, "Q4_K"), (Q6_K, "Q6_K")):
        for rows, cols in ((4096, 4096), (14336, 4096), (4096, 14336)):
            raw = synth.random_blocks(ttype, rows * cols // 256, seed=2, stream=ttype * 100 + rows // 1024)
            nb = int(L.wgd_tiled_bytes(ttype, rows, cols))
            stride = (nb + 16 + 255) // 256 * 256
            copies = max(2, int(np.ceil(320e6 / nb)))
            pool = torch.empty(copies * stride, dtype=torch.uint8, device=dev)
            raw_d = torch.from_numpy(raw).to(dev)
            _native.check(L.wgd_op_repack_tiled(ttype, rows, cols, raw_d.data_ptr(), pool.data_ptr(), sp))
            for i in range(1, copies):
                pool[i * stride:i * stride + nb].copy_(pool[:nb])
            del raw_d
            x = torch.randn(128 * cols, device=dev)
            y = torch.empty(128 * rows, device=dev)
            for batch in (1, 8, 32, 128):
                gemm = batch >= 16
                fn = L.wgd_op_gemm_tiled if gemm else L.wgd_op_gemv_tiled

                def launch(i):
                    _native.check(fn(ttype, rows, cols, ctypes.c_void_p(pool.data_ptr() + (i % copies) * stride),
                                     x.data_ptr(), batch, y.data_ptr(), sp))
                for i in range(3):
                    launch(i)
                torch.cuda.synchronize(device)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for i in range(launches):
                    launch(i)
                e1.record(stream)
                torch.cuda.synchronize(device)
                us = e0.elapsed_time(e1) / launches * 1000.0
                alg = rows * cols * bpw[ttype] + batch * (rows + cols) * 4
                flops = 2.0 * batch * rows * cols
                entry = {"type": tname, "rows": rows, "cols": cols, "batch": batch,
                         "kernel": "gemm_tc_kernel (tcgen05)" if gemm else "gemv2_kernel (integer mma.sync)",
                         "us": us, "achieved_gbs": alg / us / 1e3, "frac": alg / us / 1e3 / hbm,
                         "tflops": flops / us / 1e6}
                if gemm:
                    entry["tensor_frac"] = flops / us / 1e6 / tpk
                cases.append(entry)
            del pool, x, y
    st = ctypes.c_int(0)
    _native.check(L.wgd_op_gemm_tiled_status(ctypes.byref(st)))
    return {"cases": cases, "hbm_peak_gbs": hbm, "hbm_peak_kind": hbm_kind, "tensor_peak_tflops": tpk,
            "tensor_peak_kind": tpk_kind, "launches": launches,
            "l2": "weight copies > 320 MB rotate, so every launch reads its weights from HBM",
            "pipeline_timeouts": st.value}


# ------------------------------------------------------------- parity and CPU baseline

def parity_gpu(eng, prompt, steps):
    """GPU side of the parity leg (every rank; the forwards are collective under TP): the prompt as one
    batch at position 0, then `steps - 1` single-token forwards with the full logits read back, then
    the same continuation through the device decode loop."""
    from webgpu_b200 import _native
    L = _native.lib()
    out = eng.forward(list(prompt), 0, True, want_logits=True)
    toks, logits, pos = [], [], len(prompt)
    for s in range(steps):
        tok, lg = out
        toks.append(int(tok))
        logits.append(np.array(lg, dtype=np.float64))
        if s + 1 < steps:
            out = eng.forward([tok], pos, True, want_logits=True)
            pos += 1
    buf = (ctypes.c_int32 * (steps - 1))()
    _native.check(L.wgd_decode(eng.ctx, toks[0], len(prompt), steps - 1, buf), "decode")
    return toks, logits, [int(b) for b in buf]


def parity_oracle(image, prompt, steps, threads, single_thread: bool):
    """The float64 CPU oracle on the same ids and positions (timed: the CPU baseline sample), and
    optionally one more forward on one thread."""
    import oracle
    from webgpu_b200.gguf import model_config, parse_gguf_header
    g = parse_gguf_header(image, image.nbytes)
    c = model_config(g)
    dec = oracle.Decoder(image, g, c, context=64, threads=threads)
    t0 = time.perf_counter()
    toks, logits = dec.greedy_decode(list(prompt), steps)
    dt = time.perf_counter() - t0
    forwards = len(prompt) + steps - 1
    st = None
    if single_thread:
        oracle.lib().or_set_threads(1)
        t1 = time.perf_counter()
        dec.forward([toks[-1]], len(prompt) + steps - 1)
        st = time.perf_counter() - t1
    dec.close()
    return toks, logits, forwards / dt, forwards, (1.0 / st if st else None)


def parity_summary(gpu, ref_toks, ref_logits):
    toks, logits, loop = gpu
    errs = [float(np.max(np.abs(a - b)) / np.max(np.abs(b))) for a, b in zip(logits, ref_logits)]
    margins = [float(np.sort(l)[-1] - np.sort(l)[-2]) for l in ref_logits]
    return {"tokens_equal": toks == ref_toks and loop == ref_toks[1:], "gpu_tokens": toks, "oracle_tokens": ref_toks,
            "device_loop_tokens": loop, "max_rel_logit_err": max(errs), "rel_logit_err_per_step": errs,
            "tolerance": LOGIT_TOL, "within_tolerance": max(errs) < LOGIT_TOL, "top2_margins": margins,
            "prompt_tokens": PARITY_PROMPT, "steps": PARITY_STEPS,
            "schedule": "prompt as one batch at position 0 (per-kernel prompt path), then single-token forwards "
                        "with logits (the decode kernel of the headline), then the device loop from the first token",
            "error_measure": "max|gpu - oracle| / max|oracle| over the vocabulary row"}


# ------------------------------------------------------------------ reference arm

def run_reference(args, rank, world):
    """--impl reference: the CPU restatement on all host threads at the GPU arm's first decode
    positions (KV rows of the 512 prompt positions filled with seeded values: the attention work of a
    decode step depends on the position, not on the cached values)."""
    if rank != 0:
        return
    _, image = build_model()
    threads = cpu_threads()
    steps, warm = max(1, min(args.steps, 4)), max(0, min(args.warmup, 1))
    import oracle
    from webgpu_b200 import synth
    from webgpu_b200.gguf import model_config, parse_gguf_header
    g = parse_gguf_header(image, image.nbytes)
    c = model_config(g)
    dec = oracle.Decoder(image, g, c, context=CONTEXT, threads=threads)
    dec.fill_cache(PROMPT, seed=2)
    ids = synth.uniform_ids(steps + warm, c.vocab, seed=2, stream=77)
    for i in range(warm):
        dec.forward([ids[i]], PROMPT + i)
    t0 = time.perf_counter()
    for i in range(steps):
        dec.forward([ids[warm + i]], PROMPT + i)
    dt = time.perf_counter() - t0
    dec.close()
    v = steps / dt
    sample = (f"{steps} decode steps (after {warm} warm-up) of the full model at positions {PROMPT}..{PROMPT + steps - 1} "
              f"(the GPU arm's first decode positions; cached K/V of positions 0..{PROMPT - 1} seeded), f64, "
              f"{threads} threads on {cpu_model()}")
    line = {"metric": METRIC, "value": v, "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * dt / steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded random-init weights)",
            "config": {"workload": "Llama-3-8B arch Q4_K_M, batch-1 greedy decode after a 512-token prompt (CPU sample)",
                       "model": "llama-3-8b-arch", "context": CONTEXT, "prompt": PROMPT,
                       "positions": [PROMPT, PROMPT + steps - 1], "threads": threads, "cpu_model": cpu_model()},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm

def run_ours(args, rank, world, local, dist, host_group):
    import torch
    from webgpu_b200 import _native
    from webgpu_b200.engine import PagedEngine
    from webgpu_b200.source import MemorySource

    def host_barrier():
        if dist:
            dist.barrier(group=host_group)

    model_file = None
    if world > 1:
        spec, image, model_file = shared_model(args.layers, world, local, host_barrier)
    else:
        spec, image = build_model(args.layers)
    opts = {"contextLength": CONTEXT, "batchSize": PREFILL_BATCH, "performance": "fast", "gpuBudgetMiB": 40 * 1024,
            "tensorParallel": world, "rank": rank, "device": local}
    if dist:
        def exchange(b: bytes):
            out = [None] * world
            dist.all_gather_object(out, b, group=host_group)
            return out
        opts["exchange"] = exchange
    eng = PagedEngine()
    t0 = time.time()
    eng.load(MemorySource(image), opts)
    log(f"[bench] rank {rank}: loaded in {time.time() - t0:.1f}s; gpu bytes {eng.stats()['gpuBytes'] / 1e9:.2f} GB")
    host_barrier()
    if model_file and local == 0:
        os.unlink(model_file)  # every rank has uploaded its shard (rank 0 keeps its image in memory)
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
                 "frac": g_achieved / peak, "launch_ms": ms, "algorithmic_bytes": alg, "traffic": GEMV_TRAFFIC,
                 "traffic_source": "ncu capture of this shape (one launch)"}
        achieved = step_bytes / (step_ms / 1000) / 1e9
        roof = {"bound": "hbm", "unit": "GB/s", "peak": peak, "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                "kernel": ("persist_kernel: whole decode steps (all layers, LM head, argmax) in one launch" if persistent
                           else "per-kernel decode step (CUDA graph of the step's kernels, replayed once per step)"),
                "achieved": achieved, "frac": achieved / peak,
                "per": ("decode step and rank (one launch runs all timed steps)" if persistent
                        else "decode step and rank (one graph replay per step)"),
                "algorithmic_bytes": step_bytes, "ms": step_ms,
                "traffic": STEP_TRAFFIC / world if persistent and world == 1 else None,
                "traffic_source": STEP_TRAFFIC_SOURCE if persistent and world == 1 else None,
                "launch_ms": dev_ms, "steps_per_launch": args.steps if persistent else 1, "gemv_probe": probe}

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
                           "tensor work is twice the algorithmic FLOPs (activation hi/lo split)"}

    # ---- parity: the oracle and the GPU on the same ids from position 0 (the prompt's KV rows are
    # rewritten; nothing timed follows on the GPU)
    parity, base = None, None
    if not args.no_parity:
        pprompt = list(spec.prompt[:PARITY_PROMPT])
        gpu = parity_gpu(eng, pprompt, PARITY_STEPS)
        if rank == 0:
            threads = cpu_threads()
            rt, rl, tps, forwards, single = parity_oracle(image, pprompt, PARITY_STEPS, threads, world == 1)
            parity = parity_summary(gpu, rt, rl)
            if world == 1 and not args.no_cpu_baseline:
                base = {"value": tps, "unit": "tok/s", "cores": threads, "kind": "port", "cpu_model": cpu_model(),
                        "single_thread_tok_per_s": single,
                        "sample": f"the parity leg's {forwards} forwards of the full model (positions 0..{forwards - 1}, one "
                                  f"token each: a {PARITY_PROMPT}-token prompt then {PARITY_STEPS - 1} greedy steps), float64 "
                                  f"oracle decoder on {threads} threads; single_thread_tok_per_s: one more forward on 1 thread"}
        host_barrier()

    c2 = None
    if rank == 0 and world == 1 and not args.no_c2:
        c2 = c2_table(local)

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
            "roofline": roof, "cpu_baseline": base, "parity": parity, "clocks": clocks, "prefill": prefill,
            "sampled": sampled, "gpu_launches": launches,
            "tokens_match_e2e": tokens_dev == tokens_e2e,
            "c2": c2, "qwen2_5_0_5b": qwen,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()


# ------------------------------------------------------------------ profiling cases

def case_gemv(rows: int, cols: int, ttype: int = Q4_K, launches: int = 5) -> None:
    """wgd_op_gemv_tiled on random blocks of TYPE (12 Q4_K, 14 Q6_K), repacked into the tile layout
    once, called LAUNCHES times (L2-resident after the first when the matrix fits)."""
    import torch
    from webgpu_b200 import _native, synth
    L = _native.lib()
    raw = synth.random_blocks(ttype, rows * cols // 256, 2, 99)
    nb = L.wgd_tiled_bytes(ttype, rows, cols)
    rd = torch.from_numpy(raw).cuda()
    m = torch.empty(nb + 16, dtype=torch.uint8, device="cuda")
    _native.check(L.wgd_op_repack_tiled(ttype, rows, cols, rd.data_ptr(), m.data_ptr(), None))
    x = torch.randn(cols, device="cuda")
    y = torch.empty(rows, device="cuda")
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(launches):
        _native.check(L.wgd_op_gemv_tiled(ttype, rows, cols, m.data_ptr(), x.data_ptr(), 1, y.data_ptr(), None))
    e1.record()
    torch.cuda.synchronize()
    print(f"gemv type {ttype} {rows}x{cols}: {e0.elapsed_time(e1) / launches * 1000:.2f} us/launch", flush=True)


def case_attention(heads: int = 32, kv: int = 8, hd: int = 128, cap: int = 4096, copies: int = 24) -> None:
    """wgd_op_attention (decode row) at L = 512 / 2048 / 4096 over 24 K/V caches of [8][4096][128]
    fp32 (more than L2), 24 graph-captured launches per length."""
    import torch
    from webgpu_b200 import _native
    L = _native.lib()
    ks = [torch.randn(kv, cap, hd, device="cuda") for _ in range(copies)]
    vs = [torch.randn(kv, cap, hd, device="cuda") for _ in range(copies)]
    q = torch.randn(heads, hd, device="cuda")
    out = torch.empty(heads, hd, device="cuda")
    for start in (511, 2047, 4095):
        def launch_all(stream):
            for i in range(copies):
                _native.check(L.wgd_op_attention(q.data_ptr(), ks[i].data_ptr(), vs[i].data_ptr(), out.data_ptr(), 1, heads, kv,
                                                 hd, start, 0.088, cap, cap, stream))
        launch_all(None)
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            launch_all(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / copies * 1000
        alg = (start + 1) * kv * hd * 4 * 2
        print(f"attention decode L={start + 1}: {us:7.2f} us  {alg / us / 1e3:7.1f} GB/s", flush=True)


def case_decode(layers: int, steps: int, persistent: int = 1) -> None:
    """The benchmark's Llama-3-8B architecture with LAYERS layers: 512-token prompt in batches of
    128, then wgd_decode of STEPS tokens three times (PERSISTENT 1: the persistent kernel, 0: the
    per-kernel path)."""
    from webgpu_b200 import _native, synth
    from webgpu_b200.engine import PagedEngine
    from webgpu_b200.source import MemorySource
    spec = synth.baseline_spec(3, layers=layers)
    img = synth.build_gguf(spec)
    e = PagedEngine()
    e.load(MemorySource(img), {"contextLength": 4096, "batchSize": 128, "performance": "fast", "gpuBudgetMiB": 100000})
    L = _native.lib()
    L.wgd_set_persistent(e.ctx, persistent)
    prompt = list(synth.uniform_ids(512, 128256, seed=2))
    tok = None
    for i in range(0, 512, 128):
        tok = e.forward(prompt[i:i + 128], i, i + 128 == 512)
    buf = (ctypes.c_int32 * steps)()
    _native.check(L.wgd_decode(e.ctx, tok, 512, steps, buf))
    st = _native.StatsC()
    for _ in range(3):
        _native.check(L.wgd_decode(e.ctx, tok, 512, steps, buf))
        _native.check(L.wgd_stats_get(e.ctx, ctypes.byref(st)))
        print(f"layers {layers} persistent {persistent}: {st.last_forward_ms / steps * 1000:.1f} us/token ({steps} steps)", flush=True)
    e.dispose()


def case_gemm(rows: int, cols: int, batch: int, launches: int = 20, ttype: int = Q4_K) -> None:
    """The tcgen05 GEMM and the tiled GEMV on one Q4_K / Q6_K matrix (CUDA events; up to 8 weight
    copies rotate so that every launch reads them from HBM when they exceed L2)."""
    import torch
    from webgpu_b200 import _native, synth
    L = _native.lib()
    nb = L.wgd_tiled_bytes(ttype, rows, cols)
    copies = max(1, min(8, (1 << 30) // nb))
    raw = synth.random_blocks(ttype, rows * cols // 256, 2, 99)
    rd = torch.from_numpy(raw).cuda()
    mats = []
    for _ in range(copies):
        m = torch.empty(nb + 16, dtype=torch.uint8, device="cuda")
        _native.check(L.wgd_op_repack_tiled(ttype, rows, cols, rd.data_ptr(), m.data_ptr(), None))
        mats.append(m)
    x = torch.randn(batch * cols, device="cuda")
    y = torch.empty(batch * rows, device="cuda")
    flops = 2.0 * rows * cols * batch
    for name, fn in (("gemm_tc", L.wgd_op_gemm_tiled), ("gemv_tiled", L.wgd_op_gemv_tiled)):
        for i in range(3):
            _native.check(fn(ttype, rows, cols, mats[i % copies].data_ptr(), x.data_ptr(), batch, y.data_ptr(), None))
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for i in range(launches):
            _native.check(fn(ttype, rows, cols, mats[i % copies].data_ptr(), x.data_ptr(), batch, y.data_ptr(), None))
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / launches * 1000
        print(f"{name} {'Q4_K' if ttype == Q4_K else 'Q6_K'} {rows}x{cols} batch {batch}: {us:8.2f} us/launch  "
              f"{flops / us / 1e6:8.1f} TFLOP/s  weights {nb / us / 1e3:7.1f} GB/s", flush=True)
    st = ctypes.c_int(0)
    _native.check(L.wgd_op_gemm_tiled_status(ctypes.byref(st)))
    assert st.value == 0


def case_prefill(layers: int, batch: int, min_batch: int = 16) -> None:
    """Prefill of 512 tokens in batches of BATCH through wgd_forward (Llama-3-8B widths)."""
    from webgpu_b200 import _native, synth
    from webgpu_b200.engine import PagedEngine
    from webgpu_b200.source import MemorySource
    spec = synth.baseline_spec(3, layers=layers)
    img = synth.build_gguf(spec)
    e = PagedEngine()
    e.load(MemorySource(img), {"contextLength": 4096, "batchSize": batch, "performance": "fast", "gpuBudgetMiB": 100000})
    L = _native.lib()
    _native.check(L.wgd_set_prefill_gemm(e.ctx, min_batch))
    prompt = list(synth.uniform_ids(512, 128256, seed=2))
    st = _native.StatsC()
    for _ in range(3):
        total = 0.0
        for i in range(0, 512, batch):
            e.forward(prompt[i:i + batch], i, i + batch == 512)
            _native.check(L.wgd_stats_get(e.ctx, ctypes.byref(st)))
            total += st.last_forward_ms
        print(f"prefill layers {layers} batch {batch} min_batch {min_batch}: {total:.2f} ms for 512 tokens "
              f"({512 / total * 1000:.0f} tok/s)", flush=True)
    e.dispose()


def case_qwen(steps: int, repeats: int = 3) -> None:
    """The Qwen2.5-0.5B configuration: 23-token prompt in one batch, then wgd_decode of STEPS tokens
    REPEATS times (the first call also captures the per-kernel step graph when that path runs)."""
    from webgpu_b200 import _native, synth
    from webgpu_b200.engine import PagedEngine
    from webgpu_b200.source import MemorySource
    spec = synth.baseline_spec(2)
    img = synth.build_gguf(spec)
    e = PagedEngine()
    e.load(MemorySource(img), {"contextLength": 512, "batchSize": 32, "performance": "fast"})
    L = _native.lib()
    prompt = list(spec.prompt)
    tok = e.forward(prompt, 0, True)
    buf = (ctypes.c_int32 * steps)()
    st = _native.StatsC()
    per = ctypes.c_int(0)
    for _ in range(repeats):
        _native.check(L.wgd_decode(e.ctx, tok, len(prompt), steps, buf))
        _native.check(L.wgd_stats_get(e.ctx, ctypes.byref(st)))
        _native.check(L.wgd_kernels_per_token(e.ctx, ctypes.byref(per)))
        print(f"qwen2.5-0.5b: {st.last_forward_ms / steps * 1000:.1f} us/token ({steps} steps); {per.value} kernels per token",
              flush=True)
    e.dispose()


def case_gemma_paged(layers: int, steps: int) -> None:
    """Gemma-3-27B widths (seed 3) with LAYERS layers under a 2 GiB engine budget and 16 MiB pages
    (low-memory): the matrices that do not fit stream from pinned host memory through two device page
    slots every forward. 1024-token prompt in batches of 128, then wgd_decode of STEPS tokens; reports
    the bytes streamed per token against a pinned host-to-device copy measured in the same process."""
    import torch
    from webgpu_b200 import _native, synth
    from webgpu_b200.engine import PagedEngine
    from webgpu_b200.source import MemorySource
    t0 = time.time()
    spec = synth.baseline_spec(4, layers=layers)
    img = synth.build_gguf(spec)
    print(f"gemma-3-27b widths, {layers} layers: {img.nbytes / 1e9:.2f} GB GGUF built in {time.time() - t0:.1f}s", flush=True)
    e = PagedEngine()
    t0 = time.time()
    e.load(MemorySource(img), {"contextLength": 2048, "batchSize": 128, "performance": "low-memory", "gpuBudgetMiB": 2048})
    st = _native.StatsC()
    L = _native.lib()
    _native.check(L.wgd_stats_get(e.ctx, ctypes.byref(st)))
    print(f"loaded in {time.time() - t0:.1f}s; device bytes {st.gpu_bytes / 1e9:.2f} GB", flush=True)
    prompt = list(synth.uniform_ids(1024, 262144, seed=3))
    tok, pf = None, 0.0
    for i in range(0, 1024, 128):
        tok = e.forward(prompt[i:i + 128], i, i + 128 == 1024)
        _native.check(L.wgd_stats_get(e.ctx, ctypes.byref(st)))
        pf += st.last_forward_ms
    print(f"prefill 1024 tokens in batches of 128: {pf:.0f} ms", flush=True)
    buf = (ctypes.c_int32 * steps)()
    _native.check(L.wgd_decode(e.ctx, tok, 1024, steps, buf))
    _native.check(L.wgd_stats_get(e.ctx, ctypes.byref(st)))
    per = st.last_forward_ms / steps
    streamed = st.streamed_bytes / steps
    print(f"decode: {per:.1f} ms/token ({1000 / per:.2f} tok/s); {streamed / 1e9:.2f} GB streamed per token = "
          f"{streamed / per / 1e6:.1f} GB/s", flush=True)
    e.dispose()
    h = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    d = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    for _ in range(2):
        d.copy_(h, non_blocking=True)
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(4):
        d.copy_(h, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    print(f"pinned host-to-device copy: {4 * (1 << 30) / (e0.elapsed_time(e1) / 1000) / 1e9:.1f} GB/s", flush=True)


def case_c2() -> None:
    """The c2 microbench table alone, one JSON object."""
    print(json.dumps(c2_table(0)), flush=True)


def case_gemma_tp(steps: int = 16) -> None:
    """The benchmark's Gemma-3-27B configuration resident and tensor-parallel over the ranks of a
    torchrun launch (one rank: one GPU): 62 gemma3 blocks (5 local : 1 global, Q/K norm, GeGLU),
    seed 3, the 1024-token prompt prefilled in batches of 128, then `steps` greedy tokens of the
    device decode loop (CUDA events, max over ranks). Parity: a 4-token prompt at position 0 and 3
    greedy tokens, the full logits gathered to rank 0 and compared with the float64 oracle there.
    Rank 0 prints one JSON object."""
    import datetime

    import torch
    from webgpu_b200 import _native, synth
    from webgpu_b200.engine import PagedEngine
    from webgpu_b200.source import MemorySource
    world, rank, local = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist, host_group = None, None
    if world > 1:
        import torch.distributed as tdist
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=torch.device("cuda", local))
        host_group = tdist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=900))
        dist = tdist

    def host_barrier():
        if dist:
            dist.barrier(group=host_group)
    try:
        t0 = time.time()
        spec = synth.baseline_spec(4)
        path = None
        if world > 1:
            base = "/dev/shm" if os.path.isdir("/dev/shm") and shutil.disk_usage("/dev/shm").free > 40e9 else tempfile.gettempdir()
            path = os.path.join(base, f"wgd_bench_gemma3_27b_seed3_{os.environ.get('MASTER_PORT', '0')}.gguf")
        image = None
        if local == 0:
            image = synth.build_gguf(spec)
            if path:
                image.tofile(path + ".tmp")
                os.replace(path + ".tmp", path)
        host_barrier()
        if image is None:
            image = np.memmap(path, dtype=np.uint8, mode="r")
        log(f"[gemma_tp] rank {rank}: model ready in {time.time() - t0:.1f}s ({image.nbytes / 1e9:.2f} GB)")
        opts = {"contextLength": 2048, "batchSize": 128, "performance": "fast", "gpuBudgetMiB": 60 * 1024,
                "tensorParallel": world, "rank": rank, "device": local}
        if dist:
            def exchange(b: bytes):
                out = [None] * world
                dist.all_gather_object(out, b, group=host_group)
                return out
            opts["exchange"] = exchange
        eng = PagedEngine()
        eng.load(MemorySource(image), opts)
        host_barrier()
        if path and local == 0:
            os.unlink(path)
        L = _native.lib()
        prompt = spec.prompt[:1024]
        st = _native.StatsC()
        pf_ms, tok = 0.0, None
        for i in range(0, len(prompt), 128):
            tok = eng.forward(prompt[i:i + 128], i, i + 128 == len(prompt))
            L.wgd_stats_get(eng.ctx, ctypes.byref(st))
            pf_ms += st.last_forward_ms
        buf = (ctypes.c_int32 * max(steps, 3))()
        _native.check(L.wgd_decode(eng.ctx, tok, len(prompt), 3, buf), "decode")  # warm-up (graph capture)
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        _native.check(L.wgd_decode(eng.ctx, tok, len(prompt), steps, buf), "decode")
        L.wgd_stats_get(eng.ctx, ctypes.byref(st))
        ms = st.last_forward_ms
        if dist:
            t = torch.tensor([ms, pf_ms], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms, pf_ms = float(t[0]), float(t[1])
        why = ctypes.create_string_buffer(256)
        persistent = L.wgd_persistent_status(eng.ctx, why, 256) == 1
        gpu = parity_gpu(eng, list(spec.prompt[:PARITY_PROMPT]), 3)
        par = None
        if rank == 0:
            rt, rl, _, _, _ = parity_oracle(image, list(spec.prompt[:PARITY_PROMPT]), 3, cpu_threads(), False)
            par = parity_summary(gpu, rt, rl)
        host_barrier()
        c = eng.config
        wbytes = weight_bytes(eng.gguf, c)
        eng.dispose()
        if rank == 0:
            peak, kind = peaks()
            step_ms = ms / steps
            achieved = wbytes / world / (step_ms / 1000) / 1e9
            print(json.dumps({"workload": "Gemma-3-27B arch Q4_K_M, 1024-token prompt in batches of 128, then batch-1 greedy decode",
                              "n_gpus": world, "steps": steps, "tok_per_s": steps / (ms / 1000.0), "ms_per_step": step_ms,
                              "prefill_ms": pf_ms, "prefill_tok_per_s": len(prompt) / (pf_ms / 1000.0),
                              "weight_bytes_per_rank": wbytes / world, "achieved_gbs_per_rank": achieved,
                              "frac": achieved / peak, "peak_kind": kind,
                              "path": "persistent kernel" if persistent else f"per-kernel CUDA graph ({why.value.decode()})",
                              "parity": par}), flush=True)
    finally:
        if dist:
            dist.destroy_process_group()


CASES = {"gemv": case_gemv, "attention": case_attention, "decode": case_decode, "gemm": case_gemm,
         "prefill": case_prefill, "qwen": case_qwen, "gemma_paged": case_gemma_paged, "c2": case_c2,
         "gemma_tp": case_gemma_tp}


# ------------------------------------------------------------------ main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=None, help="trim depth (debug only; not a valid bench number)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle comparison (debug only)")
    ap.add_argument("--no-c2", action="store_true", help="skip the GEMV/GEMM microbench table")
    ap.add_argument("--case", nargs="+", metavar=("NAME", "ARG"), help=f"one profiling workload: {', '.join(CASES)}")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.case:
        name, rest = args.case[0], [int(a) for a in args.case[1:]]
        if name not in CASES:
            ap.error(f"unknown case {name}; choose from {', '.join(CASES)}")
        CASES[name](*rest)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        # rank 0 alone runs the CPU path; no process group, so idle ranks hold no cores
        run_reference(args, rank, world)
        return

    dist, host_group = None, None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
        # host-side waits (model file, handle exchange, the oracle on rank 0) block in gloo instead
        # of spinning on a device synchronize
        host_group = tdist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=900))
        dist = tdist
    else:
        import torch
        torch.cuda.set_device(local)
    try:
        run_ours(args, rank, world, local, dist, host_group)
    finally:
        if dist:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
