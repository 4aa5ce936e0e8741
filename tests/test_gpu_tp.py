"""Tensor parallelism on 2 GPUs of one box: one process per GPU, NCCL only for the start-up
handle exchange, and the library's own exchange over CUDA-IPC peer buffers after the row-split
O and down projections. The sharded decoder must give the oracle's greedy tokens and logits
(gathered on rank 0), for the llama, qwen2 and gemma blocks, and the device decode loop must give
the same tokens as one forward per token. For the models the persistent decode kernel covers, the
device loop runs it with the exchange fused in (partial rows pushed to the peer in the O/down
epilogues, one cross-rank barrier per exchange). A peer that never joins makes the waiting rank's
forward fail with WGD_ETIMEOUT after its wait limit, with no fault. Skipped with fewer than 2 GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest

from webgpu_b200 import synth

pytestmark = pytest.mark.gpu
WORLD = 2
STEPS = 4


def _need_gpus():
    import torch
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")


def _gemma_small():
    # 8 heads of 64: each rank's output-projection shard (4 heads, 256 columns) is one Q4_K block
    s = synth.gemma_spec(seed=12, layers=6, hidden=256, ffn=512, heads=8, kv_heads=4, head_dim=64, vocab=300, window=6,
                         wtype=synth.Q4_K, embd_type=synth.Q6_K, std=0.05)
    s.prompt = synth.uniform_ids(21, 300, seed=12)
    return s


def _llama8b_one_layer():
    s = synth.baseline_spec(3, layers=1)
    s.prompt = s.prompt[:12]
    return s


def _mid_llama(seed=41, layers=2):
    # 2048 wide, 16 heads of 128 / 4 KV heads, FFN 5632: at 2 ranks the O shard is 1024 columns (4
    # super-blocks) and the down shard 2816 (11): the persistent kernel's narrow-input epilogue and
    # tiles cut between CTAs
    s = synth.dense_spec("llama", seed=seed, layers=layers, hidden=2048, ffn=5632, heads=16, kv_heads=4, head_dim=128,
                         vocab=4096, eps=1e-5, theta=5e5, wtype=synth.Q4_K, out_type=synth.Q6_K, embd_type=synth.Q6_K,
                         std=0.05)
    s.prompt = synth.uniform_ids(20, 4096, seed=seed)
    return s


SPECS = {
    "tiny_llama_f32": lambda: synth.baseline_spec(0),
    "llama8b_one_layer_q4k": _llama8b_one_layer,
    "qwen05_two_layers": lambda: synth.baseline_spec(2, layers=2),
    "gemma_local_global": _gemma_small,
    "mid_llama_persistent": _mid_llama,
}
# models whose device decode loop must run the persistent kernel at 2 ranks
PERSISTENT = {"llama8b_one_layer_q4k", "mid_llama_persistent"}


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, port, name, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import ctypes

    import torch
    import torch.distributed as dist

    from webgpu_b200 import _native, tp
    from webgpu_b200.engine import PagedEngine
    from webgpu_b200.source import MemorySource
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    e = None
    try:
        spec = SPECS[name]()
        image = synth.build_gguf(spec)
        e = PagedEngine()
        batch = 8
        e.load(MemorySource(image), {"contextLength": 512, "batchSize": batch, "performance": "fast", "tensorParallel": WORLD,
                                     "rank": rank, "device": rank, "exchange": tp.torch_exchange()})
        prompt = list(spec.prompt)
        out = None
        for i in range(0, len(prompt), batch):
            chunk = prompt[i:i + batch]
            out = e.forward(chunk, i, i + len(chunk) == len(prompt), want_logits=True)
        pos, toks, logits = len(prompt), [], []
        for s in range(STEPS):
            tok, lg = out
            toks.append(int(tok))
            logits.append(np.array(lg, dtype=np.float32) if rank == 0 else None)
            if s + 1 < STEPS:
                out = e.forward([tok], pos, True, want_logits=True)
                pos += 1
        # the device loop from the same state: tokens 1.. follow from the first
        buf = (ctypes.c_int32 * (STEPS - 1))()
        _native.check(_native.lib().wgd_decode(e.ctx, toks[0], len(prompt), STEPS - 1, buf), "decode")
        why = ctypes.create_string_buffer(256)
        persistent = _native.lib().wgd_persistent_status(e.ctx, why, 256) == 1
        q.put((rank, toks, logits if rank == 0 else None, list(buf), None if persistent or name not in PERSISTENT
               else f"persistent kernel not used: {why.value.decode()}"))
    except BaseException as ex:  # reported to the parent; the peer fails its next collective by timeout
        q.put((rank, None, None, None, repr(ex)))
    finally:
        if e is not None:
            e.dispose()
        dist.destroy_process_group()


@pytest.mark.parametrize("name", list(SPECS))
def test_tensor_parallel_two_gpus_matches_oracle(cuda, name):
    _need_gpus()
    import torch.multiprocessing as mp

    import oracle
    from webgpu_b200.gguf import model_config, parse_gguf_header
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, name, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(WORLD):
            rank, toks, logits, dev, err = q.get(timeout=600)
            results[rank] = (toks, logits, dev, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    errs = {r: v[3] for r, v in results.items() if v[3]}
    assert not errs, errs
    # both ranks report the same greedy tokens
    assert results[0][0] == results[1][0]
    spec = SPECS[name]()
    image = synth.build_gguf(spec)
    g = parse_gguf_header(image, image.nbytes)
    dec = oracle.Decoder(image, g, model_config(g), 512, threads=8)
    ref_tokens, ref_logits = dec.greedy_decode(list(spec.prompt), STEPS)
    dec.close()
    toks, logits, dev, _ = results[0]
    assert toks == ref_tokens
    for got, exp in zip(logits, ref_logits):
        rel = float(np.max(np.abs(got.astype(np.float64) - exp)) / np.max(np.abs(exp)))
        assert rel < 1e-3, rel
    assert dev == toks[1:]


def _silent_peer_main(rank, port, q):
    """Rank 1 loads its shard and opens the exchange, then never runs a forward; rank 0's
    single-token forward (the persistent kernel) waits for rank 1's arrivals at the first
    cross-rank barrier, gives up after its limit (20 ms) and reports WGD_ETIMEOUT. Only host
    processes meet afterwards (gloo), so nothing waits on the GPU once rank 0 returns."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import ctypes

    import torch
    import torch.distributed as dist

    from webgpu_b200 import _native, tp
    from webgpu_b200.engine import PagedEngine
    from webgpu_b200.source import MemorySource
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120))
    e = None
    try:
        spec = _mid_llama(seed=43)
        image = synth.build_gguf(spec)
        e = PagedEngine()
        e.load(MemorySource(image), {"contextLength": 512, "batchSize": 8, "performance": "fast", "tensorParallel": WORLD,
                                     "rank": rank, "device": rank, "exchange": tp.torch_exchange()})
        L = _native.lib()
        result = None
        if rank == 0:
            assert L.wgd_persistent_status(e.ctx, None, 0) == 1
            _native.check(L.wgd_tp_set_timeout(e.ctx, 20000))  # 20 ms for a cross-rank wait
            ids = (ctypes.c_int32 * 1)(int(spec.prompt[0]))
            out = ctypes.c_int32(-1)
            rc = L.wgd_forward(e.ctx, ids, 1, 0, 1, ctypes.byref(out), None)
            msg = _native.last_error()
            rc2 = L.wgd_forward(e.ctx, ids, 1, 0, 1, ctypes.byref(out), None)  # the group stays broken
            result = (rc, msg, rc2)
        dist.barrier()  # rank 1 frees its exchange buffer only after rank 0's kernel has returned
        q.put((rank, result, None))
    except BaseException as ex:
        q.put((rank, None, repr(ex)))
    finally:
        if e is not None:
            e.dispose()
        dist.destroy_process_group()


def test_silent_peer_times_out_without_a_fault(cuda):
    _need_gpus()
    import torch.multiprocessing as mp

    from webgpu_b200 import _native
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_silent_peer_main, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(WORLD):
            rank, res, err = q.get(timeout=600)
            results[rank] = (res, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    assert not any(v[1] for v in results.values()), results
    rc, msg, rc2 = results[0][0]
    assert rc == _native.WGD_ETIMEOUT, (rc, msg)
    assert "limit" in msg
    assert rc2 == _native.WGD_ETIMEOUT
