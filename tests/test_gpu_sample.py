"""Device-side temperature / top-k / top-p sampling (sample.cu) against the oracle's
restatement of the reference's sample() (engine.ts:305-324) with the same uniform draw.

The draw is the same double arithmetic in the same order on both sides; only exp()
may differ in the last ulp, so a token may differ only where the draw lies within
1e-12 of the retained mass from a boundary between two candidates (checked, never
seen in practice). Rows: vocabulary sizes of the benchmark models (128256, 151936,
262144) and odd ones (1, 5, 2049, 300001: several sort passes per CTA), ties, signed
zeros, non-finite values, fewer finite values than top_k, and a row built so that the
final merge keeps tens of thousands of keys. Through the engine: wgd_forward_sample
and wgd_decode_sample on the per-kernel path (F32 model) and on the persistent decode
kernel (Q4_K/Q6_K model) against host draws over the same device logits."""
import ctypes
import math

import numpy as np
import pytest

import oracle
from webgpu_b200 import _native, synth
from webgpu_b200.engine import PagedEngine
from webgpu_b200.source import MemorySource

pytestmark = pytest.mark.gpu


def near_boundary(x, t, k, p, u, tol=1e-12):
    """True if uniform * retained lies within tol * retained of a candidate boundary."""
    x = np.asarray(x, np.float32).astype(np.float64)
    fin = np.isfinite(x)
    idx = np.nonzero(fin)[0]
    vals = x[idx]
    order = np.lexsort((idx, -vals))[:k]
    best = vals[order[0]]
    probs = [math.exp((vals[j] - best) / t) for j in order]
    total, retained, cut = sum(probs), 0.0, 0
    while cut < len(probs):
        retained += probs[cut]
        cut += 1
        if retained / total >= p:
            break
    cum, draw = 0.0, u * retained
    for q in probs[:cut]:
        cum += q
        if abs(draw - cum) <= tol * retained:
            return True
    return False


def op_sample(torch, xd, n, t, k, p, u):
    tok = ctypes.c_int32(-7)
    st = _native.lib().wgd_op_sample(xd.data_ptr(), n, t, k, p, u, ctypes.byref(tok), None)
    return st, tok.value


def check_row(torch, x, cases):
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    for t, k, p, u in cases:
        st, got = op_sample(torch, xd, x.size, t, k, p, u)
        exp = oracle.sample(x, t, k, p, u)
        if exp < 0:
            assert st == _native.WGD_ENONFINITE
            continue
        assert st == 0, _native.last_error()
        if got != exp:
            assert near_boundary(x, t, k, p, u), (x.size, t, k, p, u, got, exp)


def settings(rng, m):
    out = []
    for _ in range(m):
        out.append((float(rng.choice([0.0, 0.1, 0.7, 1.0, 2.0])), int(rng.choice([1, 2, 40, 117, 200])),
                    float(rng.choice([0.05, 0.5, 0.9, 1.0])), float(rng.random())))
    return out


@pytest.mark.parametrize("n", [1, 5, 2049, 128256, 151936, 262144, 300001])
def test_sample_rows_match_oracle(cuda, n):
    rng = np.random.default_rng(n)
    x = rng.normal(0, 3, n).astype(np.float32)
    check_row(cuda, x, settings(rng, 30))


def test_sample_ties_zeros_and_nonfinite(cuda):
    rng = np.random.default_rng(5)
    n = 50000
    x = np.round(rng.normal(0, 2, n)).astype(np.float32)  # few distinct values: ties everywhere
    check_row(cuda, x, settings(rng, 20))
    x[rng.integers(0, n, 500)] = np.nan
    x[rng.integers(0, n, 500)] = np.inf
    x[rng.integers(0, n, 500)] = -np.inf
    check_row(cuda, x, settings(rng, 20))
    z = np.zeros(4096, np.float32)
    z[::3] = -0.0
    check_row(cuda, z, settings(rng, 10))
    few = np.full(9000, np.nan, np.float32)
    few[[17, 4000, 8999]] = [1.0, 3.0, 2.0]  # 3 finite values, top_k up to 200
    check_row(cuda, few, settings(rng, 10))
    none = np.full(1000, np.nan, np.float32)
    check_row(cuda, none, [(0.7, 40, 0.9, 0.5), (0.0, 40, 0.9, 0.5)])


def test_sample_large_final_merge(cuda):
    """Every CTA's share holds the same values, so the CTAs' top-200 lists all lie above the
    largest k-th key and the final merge keeps ~G*199 keys (many sort passes)."""
    n = 262144
    share = 1024
    x = -(np.arange(n) % share).astype(np.float32) * np.float32(0.01)
    rng = np.random.default_rng(9)
    check_row(cuda, x, [(2.0, 200, 1.0, float(rng.random())) for _ in range(6)] + [(0.5, 200, 0.9, 0.3)])


def test_sample_rejects_bad_settings(cuda):
    torch = cuda
    xd = torch.zeros(100, dtype=torch.float32, device="cuda")
    for t, k, p, u in [(-0.1, 40, 0.9, 0.5), (2.5, 40, 0.9, 0.5), (0.7, 0, 0.9, 0.5), (0.7, 201, 0.9, 0.5),
                       (0.7, 40, 0.0, 0.5), (0.7, 40, 1.5, 0.5), (0.7, 40, 0.9, 1.0), (0.7, 40, 0.9, -0.1),
                       (float("nan"), 40, 0.9, 0.5)]:
        st, _ = op_sample(torch, xd, 100, t, k, p, u)
        assert st == _native.WGD_EINVAL, (t, k, p, u)


def _engine(spec, context, batch):
    image = synth.build_gguf(spec)
    e = PagedEngine()
    e.load(MemorySource(image), {"contextLength": context, "batchSize": batch, "performance": "fast", "device": 0})
    return e


def _host_replay(e, prompt, t, k, p, uniforms):
    """Host draws over device logits: one wgd_forward(want=2) per token, then oracle.sample."""
    logits = e.forward(prompt, 0, True, want_logits=True)[1]
    tokens, rows, pos = [], [], len(prompt)
    for i, u in enumerate(uniforms):
        tok = oracle.sample(logits, t, k, p, u)
        tokens.append(tok)
        rows.append(logits)
        if i + 1 < len(uniforms):
            logits = e.forward([tok], pos, True, want_logits=True)[1]
            pos += 1
    return tokens, rows


def assert_same_draws(dev, host, rows, t, k, p, uniforms):
    for i, (a, b) in enumerate(zip(dev, host)):
        if a != b:  # only a draw on a boundary (exp's last ulp) may differ; later tokens then diverge
            assert near_boundary(rows[i], t, k, p, uniforms[i]), (i, dev, host)
            return


def _device_draws(e, prompt, t, k, p, uniforms):
    L = _native.lib()
    it = iter(uniforms)
    e.random = lambda: next(it)
    first = e.forward_sample(prompt, 0, t, k, p)
    n = len(uniforms) - 1
    buf = (ctypes.c_int32 * n)()
    us = (ctypes.c_double * n)(*uniforms[1:])
    _native.check(L.wgd_decode_sample(e.ctx, first, len(prompt), n, t, k, p, us, buf))
    return [first] + list(buf)


@pytest.mark.parametrize("persistent", [False, True])
def test_engine_device_draws_match_host_draws(cuda, persistent):
    if persistent:
        spec = synth.dense_spec("llama", seed=21, layers=1, hidden=2048, ffn=5632, heads=16, kv_heads=4, head_dim=128,
                                vocab=4096, eps=1e-5, theta=5e5, wtype=synth.Q4_K, out_type=synth.Q6_K,
                                embd_type=synth.Q6_K, std=0.05)
        prompt = synth.uniform_ids(24, 4096, seed=21)
    else:
        spec = synth.tiny_dense("llama")
        prompt = list(spec.prompt)
    e = _engine(spec, 256, 32)
    L = _native.lib()
    why = ctypes.create_string_buffer(256)
    assert L.wgd_persistent_status(e.ctx, why, 256) == int(persistent), why.value
    rng = np.random.default_rng(3)
    for t, k, p in [(0.7, 40, 0.9), (2.0, 200, 1.0), (0.3, 5, 0.5)]:
        uniforms = [float(v) for v in rng.random(8)]
        dev = _device_draws(e, prompt, t, k, p, uniforms)
        host, rows = _host_replay(e, prompt, t, k, p, uniforms)
        assert_same_draws(dev, host, rows, t, k, p, uniforms)
    e.dispose()


def test_generate_samples_on_device(cuda):
    """PagedEngine.generate with the default settings (temperature 0.7, topK 40, topP 0.9): the
    streamed tokens equal host draws over the device logits with the same uniforms."""
    spec = synth.tiny_dense("llama")
    e = _engine(spec, 256, 32)  # the whole prompt in one batch, as the replay runs it
    uniforms = [0.11, 0.93, 0.42, 0.67, 0.05, 0.5]
    it = iter(uniforms)
    e.random = lambda: next(it)
    got = [ev.token for ev in e.generate_ids(list(spec.prompt), {"maxTokens": 6})]
    assert got
    host, rows = _host_replay(e, list(spec.prompt), 0.7, 40, 0.9, uniforms)
    assert_same_draws(got, host, rows, 0.7, 40, 0.9, uniforms)
    e.dispose()


def test_public_sample_known_answers(cuda):
    """tests/quant.test.ts:46-49 through the package's sample() (drawn on the device)."""
    from webgpu_b200 import sample
    assert sample(np.array([np.nan, -2, 7, 3], np.float32), 0, 40, 0.9) == 2
    with pytest.raises(ValueError, match="non-finite"):
        sample(np.array([np.nan, -np.inf], np.float32), 0, 40, 0.9)
    x = np.array([0.5, 2.0, 1.0, -1.0], np.float32)
    for u in (0.0, 0.2, 0.6, 0.99):
        assert sample(x, 0.7, 40, 0.9, rng=lambda: u) == oracle.sample(x, 0.7, 40, 0.9, u)
