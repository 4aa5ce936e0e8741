"""Greedy-token and logit parity at the FULL depth of the benchmark's model configurations,
against the float64 CPU oracle on identical GGUF bytes and token ids (the reference's end-to-end
check, scripts/verify-dense.mjs:165-211, compares whole-model greedy tokens the same way).

  * Llama-3-8B architecture, 32 layers, Q4_K layers + Q6_K head (the headline benchmark model):
    a 4-token prompt, then greedy tokens through single-row forwards, which run the persistent
    decode kernel, and the device decode loop from the first token.
  * Qwen2.5-0.5B architecture, 24 layers (the 23-token prompt in one batch of 32).
  * Gemma-3-27B architecture, 62 layers (5 local : 1 global, Q/K norm, GeGLU), resident and paged
    under a 2 GiB engine budget with 16 MiB pages (the matrices that do not fit stream from pinned
    host memory every forward).

Bars: greedy tokens identical; logits within 1e-3 max relative error (max|gpu - oracle| /
max|oracle| over the vocabulary row, fp32 accumulate paths)."""
import ctypes
import os

import numpy as np
import pytest

import oracle
from webgpu_b200 import _native, synth
from webgpu_b200.engine import PagedEngine
from webgpu_b200.gguf import model_config, parse_gguf_header
from webgpu_b200.source import MemorySource

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-3


def _threads():
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return os.cpu_count() or 1


def _oracle(image, prompt, steps, context=64):
    g = parse_gguf_header(image, image.nbytes)
    dec = oracle.Decoder(image, g, model_config(g), context, threads=_threads())
    try:
        return dec.greedy_decode(list(prompt), steps)
    finally:
        dec.close()


def _gpu(image, prompt, steps, *, batch, context=512, opts=None):
    """Prompt in batches of `batch`, then single-token forwards with the logits read back, then the
    device decode loop from the first greedy token. Returns tokens, logits, loop tokens, persistent."""
    e = PagedEngine()
    o = {"contextLength": context, "batchSize": batch, "performance": "fast", "gpuBudgetMiB": 40960}
    o.update(opts or {})
    e.load(MemorySource(image), o)
    try:
        why = ctypes.create_string_buffer(256)
        persistent = _native.lib().wgd_persistent_status(e.ctx, why, 256) == 1
        out = None
        for i in range(0, len(prompt), batch):
            chunk = list(prompt[i:i + batch])
            out = e.forward(chunk, i, i + len(chunk) == len(prompt), want_logits=True)
        toks, logits, pos = [], [], len(prompt)
        for s in range(steps):
            tok, lg = out
            toks.append(int(tok))
            logits.append(np.array(lg, dtype=np.float64))
            if s + 1 < steps:
                out = e.forward([tok], pos, True, want_logits=True)
                pos += 1
        buf = (ctypes.c_int32 * (steps - 1))()
        _native.check(_native.lib().wgd_decode(e.ctx, toks[0], len(prompt), steps - 1, buf))
        stats = e.stats()
        return toks, logits, list(buf), persistent, stats
    finally:
        e.dispose()


def _check(gpu, ref):
    toks, logits, loop, _, _ = gpu
    ref_toks, ref_logits = ref
    margins = [float(np.sort(l)[-1] - np.sort(l)[-2]) for l in ref_logits]
    errs = [float(np.max(np.abs(a - b)) / np.max(np.abs(b))) for a, b in zip(logits, ref_logits)]
    assert toks == ref_toks, (toks, ref_toks, margins)
    assert loop == ref_toks[1:], (loop, ref_toks)
    assert max(errs) < LOGIT_TOL, errs


def test_llama3_8b_full_depth_persistent(cuda):
    spec = synth.baseline_spec(3)  # 32 layers, 4.8 GB
    image = synth.build_gguf(spec)
    prompt, steps = spec.prompt[:4], 4
    gpu = _gpu(image, prompt, steps, batch=8)
    assert gpu[3], "the persistent decode kernel must carry this model"
    _check(gpu, _oracle(image, prompt, steps))


def test_qwen2_5_0_5b_full_depth(cuda):
    spec = synth.baseline_spec(2)  # 24 layers, the 23-token prompt of the configuration
    image = synth.build_gguf(spec)
    prompt, steps = spec.prompt, 4
    _check(_gpu(image, prompt, steps, batch=32), _oracle(image, prompt, steps))


def test_gemma3_27b_full_depth_resident_and_paged(cuda):
    spec = synth.baseline_spec(4)  # 62 layers, 15.6 GB
    image = synth.build_gguf(spec)
    prompt, steps = spec.prompt[:4], 3
    ref = _oracle(image, prompt, steps)
    _check(_gpu(image, prompt, steps, batch=8), ref)
    paged = _gpu(image, prompt, steps, batch=8, opts={"performance": "low-memory", "gpuBudgetMiB": 2048})
    assert paged[4]["gpuBytes"] <= 2048 * 2 ** 20
    assert paged[4]["streamedBytes"] > 10e9  # most of the weights cross the host link every forward
    _check(paged, ref)
