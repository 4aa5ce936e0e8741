"""Small fixed workloads for profiling the library's kernels on one GPU (run them under
`ncu`, or alone to print CUDA-event timings):

    python -m webgpu_b200.probe gemv ROWS COLS TYPE [LAUNCHES]   # wgd_op_gemv_tiled on random blocks
    python -m webgpu_b200.probe attention                        # wgd_op_attention, decode, L = 512/2048/4096
    python -m webgpu_b200.probe decode LAYERS STEPS [PERSISTENT]  # Llama-3-8B-width model, wgd_decode
    python -m webgpu_b200.probe gemm ROWS COLS BATCH [LAUNCHES] [TYPE]  # wgd_op_gemm_tiled vs the GEMV (TYPE 12 Q4_K, 14 Q6_K)
    python -m webgpu_b200.probe prefill LAYERS BATCH [MIN_BATCH]  # Llama-3-8B-width prompt batches
    python -m webgpu_b200.probe qwen STEPS [REPEATS]              # Qwen2.5-0.5B architecture, wgd_decode
    python -m webgpu_b200.probe gemma_paged LAYERS STEPS          # Gemma-3-27B widths, 2 GiB budget, paged

`gemv` repacks random GGUF blocks of TYPE (12 = Q4_K, 14 = Q6_K) into the tile layout once and calls the
tiled GEMV LAUNCHES times (default 5). `attention` keeps 24 K/V caches of [8][4096][128] fp32 (more than
L2) and times 24 graph-captured launches per length. `decode` loads the synthetic Llama-3-8B
architecture (seed 2, Q4_K layers, Q6_K head) with LAYERS layers, prefills 512 tokens in batches of 128
and times `wgd_decode` of STEPS tokens three times (PERSISTENT 1: the persistent kernel, 0: the
per-kernel path).
"""
import ctypes
import sys

from . import _native, synth


def gemv(rows: int, cols: int, ttype: int, launches: int = 5) -> None:
    import torch
    L = _native.lib()
    raw = synth.random_blocks(ttype, rows * cols // synth.BLOCK[ttype][0], 2, 99)
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
    print(f"gemv type {ttype} {rows}x{cols}: {e0.elapsed_time(e1) / launches * 1000:.2f} us/launch (L2-resident after the first)")


def attention(heads: int = 32, kv: int = 8, hd: int = 128, cap: int = 4096, copies: int = 24) -> None:
    import torch
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


def decode(layers: int, steps: int, persistent: int = 1) -> None:
    from .engine import PagedEngine
    from .source import MemorySource
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


def gemm(rows: int, cols: int, batch: int, launches: int = 20, ttype: int = 12) -> None:
    """Times the tcgen05 GEMM and the tiled GEMV on one Q4_K / Q6_K matrix (CUDA events; the
    weights of 8 copies rotate so that every launch reads them from HBM when they exceed L2)."""
    import torch
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
        print(f"{name} {'Q4_K' if ttype == 12 else 'Q6_K'} {rows}x{cols} batch {batch}: {us:8.2f} us/launch  {flops / us / 1e6:8.1f} TFLOP/s "
              f"(f16 MMA work x2: {2 * flops / us / 1e6:8.1f})  weights {nb / us / 1e3:7.1f} GB/s", flush=True)
    st = ctypes.c_int(0)
    _native.check(L.wgd_op_gemm_tiled_status(ctypes.byref(st)))
    assert st.value == 0


def prefill(layers: int, batch: int, min_batch: int = 16) -> None:
    """Prefill of 512 tokens in batches of BATCH through wgd_forward (Llama-3-8B widths)."""
    from .engine import PagedEngine
    from .source import MemorySource
    spec = synth.baseline_spec(3, layers=layers)
    img = synth.build_gguf(spec)
    e = PagedEngine()
    e.load(MemorySource(img), {"contextLength": 4096, "batchSize": batch, "performance": "fast", "gpuBudgetMiB": 100000})
    L = _native.lib()
    _native.check(L.wgd_set_prefill_gemm(e.ctx, min_batch))
    prompt = list(synth.uniform_ids(512, 128256, seed=2))
    st = _native.StatsC()
    for rep in range(3):
        total = 0.0
        for i in range(0, 512, batch):
            e.forward(prompt[i:i + batch], i, i + batch == 512)
            _native.check(L.wgd_stats_get(e.ctx, ctypes.byref(st)))
            total += st.last_forward_ms
        print(f"prefill layers {layers} batch {batch} min_batch {min_batch}: {total:.2f} ms for 512 tokens "
              f"({512 / total * 1000:.0f} tok/s)", flush=True)
    e.dispose()


def qwen(steps: int, repeats: int = 3) -> None:
    """The Qwen2.5-0.5B benchmark configuration: 23-token prompt in one batch, then `wgd_decode` of
    STEPS tokens REPEATS times (the first call also captures the per-kernel step graph)."""
    from .engine import PagedEngine
    from .source import MemorySource
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


def gemma_paged(layers: int, steps: int) -> None:
    """Gemma-3-27B widths (seed 3) with LAYERS layers under a 2 GiB engine budget and 16 MiB pages
    (`low-memory`): the matrices that do not fit stream from pinned host memory through the two
    device page slots every forward. Prefills a 1024-token prompt in batches of 128, then times
    `wgd_decode` of STEPS tokens; reports the bytes streamed per token against a pinned
    host-to-device copy measured in the same process."""
    import time

    import torch

    from .engine import PagedEngine
    from .source import MemorySource
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


def main(argv):
    if not argv:
        print(__doc__)
        return 2
    cmd, args = argv[0], [int(a) for a in argv[1:]]
    if cmd == "gemv":
        gemv(*args)
    elif cmd == "attention":
        attention(*args)
    elif cmd == "decode":
        decode(*args)
    elif cmd == "gemm":
        gemm(*args)
    elif cmd == "prefill":
        prefill(*args)
    elif cmd == "qwen":
        qwen(*args)
    elif cmd == "gemma_paged":
        gemma_paged(*args)
    else:
        print(__doc__)
        return 2
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
