"""The persistent decode kernel (one cooperative launch per decode call) against the oracle
and against the per-kernel path.

The kernel covers dense llama/qwen2/qwen3 blocks whose projections are in the tiled layout
(Q4_K/Q6_K, input widths >= 2048). These mid-size models are the smallest that qualify; each
variant exercises one branch of the kernel: GQA groups of 4 and 8, head_dim 64 and 128,
Q/K norm, Q/K/V and output biases, a tied (embedding) LM head with a ragged last tile, an
ungated MLP, a sliding window whose ring wraps, attention split over many CTAs, and a head_dim that
is not a multiple of 32 (the attention item's four-warp form; eight warps otherwise).
"""
import ctypes

import numpy as np
import pytest

from webgpu_b200 import _native, synth
from test_gpu_decoder import LOGIT_TOL, compare, load

pytestmark = pytest.mark.gpu


def _mid(arch="llama", *, seed, heads=16, kv_heads=4, head_dim=128, ffn=5632, vocab=4096, prompt=24, **kw):
    s = synth.dense_spec(arch, seed=seed, layers=2, hidden=2048, ffn=ffn, heads=heads, kv_heads=kv_heads,
                         head_dim=head_dim, vocab=vocab, eps=1e-5, theta=5e5, wtype=synth.Q4_K, out_type=synth.Q6_K,
                         embd_type=synth.Q6_K, std=0.05, **kw)
    s.prompt = synth.uniform_ids(prompt, vocab, seed=seed)
    return s


def _ungated_obias():
    s = _mid("qwen2", seed=24, kv_heads=16, ffn=4096, bias=True, gate=False)
    for l in range(2):
        s.tensors.append(synth.TensorSpec(f"blk.{l}.attn_output.bias", (2048,), synth.F32, "normal", 0.05, 950 + l))
    return s


MODELS = {
    "llama_g4_hd128": lambda: _mid(seed=21),
    "llama_long_prompt_split_attention": lambda: _mid(seed=22, prompt=200),
    "llama_sliding_window_ring_wrap": lambda: _mid(seed=23, prompt=90,
                                                   extra=[("llama.attention.sliding_window", synth.T_U32, 40)]),
    "qwen2_g8_bias_tied_ragged_head": lambda: _mid("qwen2", seed=25, kv_heads=2, ffn=4864, vocab=3000, bias=True, tied=True),
    "qwen3_qknorm_hd64": lambda: _mid("qwen3", seed=26, heads=32, kv_heads=8, head_dim=64, qk_norm=True),
    # head_dim 80 (not a multiple of 32): the attention item's four-warp form
    "llama_hd80_four_warp_attention": lambda: _mid(seed=28, heads=16, kv_heads=4, head_dim=80, prompt=70),
    "qwen2_ungated_output_bias": _ungated_obias,
}


def _status(e):
    why = ctypes.create_string_buffer(256)
    ok = _native.lib().wgd_persistent_status(e.ctx, why, 256)
    return ok, why.value.decode()


@pytest.mark.parametrize("name", list(MODELS))
def test_persistent_decode_matches_oracle(cuda, name):
    spec = MODELS[name]()
    e, _ = load(spec, context=512, batch=32)
    ok, why = _status(e)
    e.dispose()
    assert ok == 1, why
    tokens, ref, errs, margins = compare(spec, 4, context=512, batch=32)
    assert tokens == ref, (tokens, ref, margins)
    assert max(errs) < LOGIT_TOL, errs


def _decode_stepwise(e, prompt, steps):
    out = e.forward(prompt, 0, True, want_logits=True)
    pos, toks, logits = len(prompt), [], []
    for _ in range(steps):
        tok, lg = out
        toks.append(tok)
        logits.append(lg)
        out = e.forward([tok], pos, True, want_logits=True)
        pos += 1
    return toks, logits


def test_persistent_equals_per_kernel_path(cuda):
    spec = MODELS["llama_g4_hd128"]()
    image = synth.build_gguf(spec)
    runs = []
    for persistent in (1, 0):
        e, _ = load(spec, context=512, batch=32, image=image)
        _native.lib().wgd_set_persistent(e.ctx, persistent)
        runs.append(_decode_stepwise(e, list(spec.prompt), 6))
        e.dispose()
    (ta, la), (tb, lb) = runs
    assert ta == tb
    for a, b in zip(la, lb):
        assert np.max(np.abs(a - b)) <= 1e-4 * np.max(np.abs(b)), np.max(np.abs(a - b))


def test_device_loop_equals_stepwise(cuda):
    """wgd_decode (all steps in one launch, tokens fed back on the device) == one forward per token."""
    spec = MODELS["llama_g4_hd128"]()
    e, _ = load(spec, context=512, batch=32)
    prompt = list(spec.prompt)
    steps = 8
    want, _ = _decode_stepwise(e, prompt, steps + 2)  # t0 .. t(steps+1)
    first = e.forward(prompt, 0, True)
    buf = (ctypes.c_int32 * steps)()
    _native.check(_native.lib().wgd_decode(e.ctx, first, len(prompt), steps, buf))
    assert [first] + list(buf) == want[:steps + 1]
    # a second call continues from where the first stopped
    _native.check(_native.lib().wgd_decode(e.ctx, buf[steps - 1], len(prompt) + steps, 1, buf))
    assert buf[0] == want[steps + 1]
    e.dispose()


def test_one_launch_per_call(cuda):
    spec = MODELS["llama_g4_hd128"]()
    e, _ = load(spec, context=512, batch=32)
    first = e.forward(list(spec.prompt), 0, True)
    L = _native.lib()
    before = _native.StatsC()
    _native.check(L.wgd_stats_get(e.ctx, ctypes.byref(before)))
    buf = (ctypes.c_int32 * 16)()
    _native.check(L.wgd_decode(e.ctx, first, len(spec.prompt), 16, buf))
    after = _native.StatsC()
    _native.check(L.wgd_stats_get(e.ctx, ctypes.byref(after)))
    assert after.kernel_launches - before.kernel_launches == 1
    assert after.tokens - before.tokens == 16
    e.dispose()


def test_models_outside_the_kernel_report_why(cuda):
    e, _ = load(synth.baseline_spec(0), batch=8)
    ok, why = _status(e)
    assert ok == 0 and "tiled" in why
    e.dispose()
