"""The weight pager (WeightPager, pager.ts:7-47): with a GPU budget smaller than the model, the
matrices that do not fit stay in pinned host memory and stream through two device page slots
on a copy stream every forward; the embedding table, if it does not fit, is gathered from host
memory. A paged load must produce the float64 oracle's greedy tokens and logits (within 1e-3
relative), the resident load's tokens (the same kernels over row ranges), report streamed
bytes, and decode the same tokens through the device loop.
"""
import ctypes

import numpy as np
import pytest

import oracle
from webgpu_b200 import _native, synth
from webgpu_b200.gguf import model_config, parse_gguf_header
from webgpu_b200.engine import PagedEngine
from webgpu_b200.source import MemorySource

pytestmark = pytest.mark.gpu
STEPS = 4


def _llama_q4k():
    s = synth.baseline_spec(3, layers=2)  # Q4_K layers (tiled), Q6_K head and embedding (431 MB each)
    s.prompt = s.prompt[:24]
    return s


def _llama_q8():
    # row layout everywhere (Q8_0): pages are whole interleave blocks of the row-layout GEMV
    s = synth.dense_spec("llama", seed=31, layers=1, hidden=4096, ffn=14336, heads=32, kv_heads=8, head_dim=128, vocab=64000,
                         eps=1e-5, theta=5e5, wtype=synth.Q8_0, std=0.02)
    s.prompt = synth.uniform_ids(20, 64000, seed=31)
    return s


def _run(spec, image, budget):
    e = PagedEngine()
    e.load(MemorySource(image), {"contextLength": 512, "batchSize": 8, "performance": "low-memory", "gpuBudgetMiB": budget})
    prompt = list(spec.prompt)
    out = None
    for i in range(0, len(prompt), 8):
        chunk = prompt[i:i + 8]
        out = e.forward(chunk, i, i + len(chunk) == len(prompt), want_logits=True)
    pos, toks, logits, streamed = len(prompt), [], [], []
    for s in range(STEPS):
        tok, lg = out
        toks.append(int(tok))
        logits.append(np.array(lg, dtype=np.float64))
        streamed.append(e.stats()["streamedBytes"])
        if s + 1 < STEPS:
            out = e.forward([tok], pos, True, want_logits=True)
            pos += 1
    buf = (ctypes.c_int32 * (STEPS - 1))()
    _native.check(_native.lib().wgd_decode(e.ctx, toks[0], len(prompt), STEPS - 1, buf))
    st = e.stats()
    e.dispose()
    return toks, logits, streamed, list(buf), st


@pytest.mark.parametrize("make,budget", [(_llama_q4k, 768), (_llama_q8, 560)])
def test_paged_load_matches_resident(cuda, make, budget):
    spec = make()
    image = synth.build_gguf(spec)
    ref_toks, ref_logits, ref_streamed, ref_dev, ref_st = _run(spec, image, 16384)
    toks, logits, streamed, dev, st = _run(spec, image, budget)
    assert max(ref_streamed) == 0 and ref_st["gpuBytes"] > budget * 2 ** 20
    assert min(streamed) > 0, "nothing was paged"
    assert st["gpuBytes"] <= budget * 2 ** 20
    assert toks == ref_toks
    # the resident reference may decode with the persistent kernel (another summation order)
    for a, b in zip(logits, ref_logits):
        assert np.max(np.abs(a - b)) <= 1e-4 * np.max(np.abs(b))
    assert dev == toks[1:] == ref_dev
    # and both against the float64 CPU oracle on the same ids and positions
    g = parse_gguf_header(image, image.nbytes)
    dec = oracle.Decoder(image, g, model_config(g), 64, threads=8)
    try:
        o_toks, o_logits = dec.greedy_decode(list(spec.prompt), STEPS)
    finally:
        dec.close()
    assert toks == o_toks
    for a, b in zip(logits, o_logits):
        assert np.max(np.abs(a - b)) < 1e-3 * np.max(np.abs(b))


def test_pull_loading_through_the_page_reader(cuda):
    """wgd_set_page_reader + wgd_load_weights (the reference's ByteSource.read pull) load the same
    model as the push uploads, also when the weights are paged."""
    spec = _llama_q4k()
    image = synth.build_gguf(spec)
    outs = []
    for opts in ({}, {"pull": True}, {"pull": True, "gpuBudgetMiB": 768}):
        e = PagedEngine()
        o = {"contextLength": 512, "batchSize": 8, "performance": "low-memory", "gpuBudgetMiB": 16384}
        o.update(opts)
        e.load(MemorySource(image), o)
        tok = e.forward(list(spec.prompt)[:8], 0, True)
        outs.append((tok, e.stats()["readBytes"]))
        e.dispose()
    assert outs[0][0] == outs[1][0] == outs[2][0]
    assert outs[1][1] == outs[0][1] > 0
