"""Single-kernel parity on the GPU through the C ABI (wgd_op_*), against the CPU
oracle. Mirrors the reference's per-kernel GPU checks (src/verify.ts:12-74 and
src/verify-context.ts:7-45 of ahpah-dev/WebGPU 0.9.0) with their fixtures and
their tolerance: |got - expected| <= 1e-3 * max(1, |expected|) (verify.ts:11),
abs 1e-3 for long-context attention (verify-context.ts:39). Dequantised
weights must be bit-exact with the WGSL-order fp32 oracle."""
import math

import numpy as np
import pytest

import oracle
from webgpu_b200 import _native, synth

pytestmark = pytest.mark.gpu

TYPES = [0, 1, 2, 8, 12, 13, 14]


def near(got, exp, rel=1e-3):
    got = np.asarray(got, np.float64)
    exp = np.asarray(exp, np.float64)
    assert np.all(np.isfinite(got))
    bad = np.abs(got - exp) > rel * np.maximum(1.0, np.abs(exp))
    assert not bad.any(), f"max err {np.max(np.abs(got - exp))} at {np.argwhere(bad)[:5].tolist()}"


def to_dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def packed_on_device(torch, ttype, raw, rows, cols):
    L = _native.lib()
    drb = L.wgd_dev_row_bytes(ttype, cols)
    raw_d = to_dev(torch, raw.reshape(-1))
    packed = torch.zeros(rows * drb + 16, dtype=torch.uint8, device="cuda")
    _native.check(L.wgd_op_repack(ttype, rows, cols, raw_d.data_ptr(), packed.data_ptr(), None))
    return packed


def verify_matrix(ttype, rows, cols):
    """verify.ts:17-25 — deterministic packed bytes (i*17+93)%256 with valid scales."""
    be, bb = synth.BLOCK[ttype]
    n = rows * cols // be * bb
    packed = np.array([(i * 17 + 93) % 256 for i in range(n)], np.uint8)
    if ttype == 0:
        f = np.sin(np.arange(n // 4)) * 0.5
        packed = f.astype(np.float32).view(np.uint8).copy()
    elif ttype == 1:
        for i in range(0, n, 2):
            packed[i] = i % 256
            packed[i + 1] = 0x30
    else:
        for off in range(0, n, bb):
            scale = off + 208 if ttype == 14 else off
            packed[scale], packed[scale + 1] = 0, 0x20
            if ttype in (12, 13):
                packed[off + 2], packed[off + 3] = 0, 0x1C
    return packed


@pytest.mark.parametrize("ttype", TYPES)
def test_dequant_bit_exact(cuda, ttype):
    torch = cuda
    rows, cols = 7, 1024
    be, _ = synth.BLOCK[ttype]
    raw = synth.random_blocks(ttype, rows * cols // be, seed=3, stream=ttype, scale_std=1e-2)
    if ttype in (0, 1):  # keep float payloads finite
        raw = synth.quantize(ttype, synth.normal(rows * cols, 3, ttype).reshape(rows, cols)).reshape(-1)
    packed = packed_on_device(torch, ttype, raw, rows, cols)
    out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    _native.check(_native.lib().wgd_op_dequant(ttype, rows, cols, packed.data_ptr(), out.data_ptr(), None))
    torch.cuda.synchronize()
    exp = oracle.decode_f32(raw, ttype, rows * cols)
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


def test_dequant_reference_fixtures(cuda):
    """The quant.test.ts byte fixtures decode bit-exactly on the device too."""
    import test_oracle_quant as q
    torch = cuda
    for ttype in (12, 13):
        data, expected = q.kquant_fixture(ttype)
        packed = packed_on_device(torch, ttype, data, 1, 256)
        out = torch.empty(256, dtype=torch.float32, device="cuda")
        _native.check(_native.lib().wgd_op_dequant(ttype, 1, 256, packed.data_ptr(), out.data_ptr(), None))
        assert out.cpu().numpy().tolist() == [float(e) for e in expected]
    data, expected = q.q6k_fixture()
    packed = packed_on_device(torch, 14, data, 1, 512)
    out = torch.empty(512, dtype=torch.float32, device="cuda")
    _native.check(_native.lib().wgd_op_dequant(14, 1, 512, packed.data_ptr(), out.data_ptr(), None))
    assert np.array_equal(out.cpu().numpy(), expected)


def run_gemv(torch, ttype, raw, rows, cols, x, batch):
    packed = packed_on_device(torch, ttype, raw, rows, cols)
    xd = to_dev(torch, x.astype(np.float32))
    y = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
    _native.check(_native.lib().wgd_op_gemv(ttype, rows, cols, packed.data_ptr(), xd.data_ptr(), batch, y.data_ptr(), None))
    torch.cuda.synchronize()
    return y.cpu().numpy().reshape(batch, rows)


@pytest.mark.parametrize("ttype", TYPES)
def test_gemv_verify_fixture_batch128(cuda, ttype):
    """verify.ts:16-36: 5 rows x 256 columns, batch 128, input offset 1."""
    rows, cols, batches = 5, 256, 128
    packed = verify_matrix(ttype, rows, cols)
    x = np.array([math.cos(i * 0.17) * 0.1 for i in range((batches + 1) * cols)], np.float32)
    xin = x[cols:]  # input offset 1 row
    y = run_gemv(cuda, ttype, packed, rows, cols, xin, batches)
    exp = oracle.matmul(packed, ttype, rows, cols, xin, batches)
    near(y, exp)


@pytest.mark.parametrize("ttype,rows,cols,batch", [
    (12, 4096, 4096, 1), (12, 14336, 4096, 1), (12, 4096, 14336, 1), (14, 4096, 4096, 1), (14, 4096, 14336, 1),
    (12, 4096, 4096, 8), (14, 4096, 4096, 8), (13, 1024, 4096, 2), (8, 1000, 896, 3), (2, 1000, 896, 1),
    (1, 512, 2048, 1), (0, 300, 640, 4), (14, 777, 5376, 1), (12, 513, 21504, 1),
])
def test_gemv_shapes(cuda, ttype, rows, cols, batch):
    be, _ = synth.BLOCK[ttype]
    if ttype in (0, 1):
        raw = synth.quantize(ttype, synth.normal(rows * cols, 4, 1, std=0.05).reshape(rows, cols)).reshape(-1)
    else:
        raw = synth.random_blocks(ttype, rows * cols // be, seed=4, stream=ttype)
    x = synth.normal(batch * cols, 4, 2)
    y = run_gemv(cuda, ttype, raw, rows, cols, x, batch)
    exp = oracle.matmul(raw, ttype, rows, cols, x, batch)
    near(y, exp)


def test_rmsnorm_and_qknorm_rope_verify_fixture(cuda):
    """verify.ts:39,55-66: RMS norm of q rows, then QK-norm + scaled RoPE (start 3, theta 1e4, scale .125)."""
    torch = cuda
    L = _native.lib()
    heads, hd, start, n = 4, 8, 3, 2
    q = np.array([math.sin(i) for i in range(n * heads * hd)], np.float32)
    w = np.array([1 + i * 0.1 for i in range(hd)], np.float32)
    qd, wd = to_dev(torch, q), to_dev(torch, w)
    out = torch.empty_like(qd)
    _native.check(L.wgd_op_rmsnorm(qd.data_ptr(), wd.data_ptr(), hd, n * heads, 1e-6, out.data_ptr(), None))
    normal = out.cpu().numpy()
    near(normal, oracle.rmsnorm(q.reshape(-1, hd), w, 1e-6).reshape(-1))
    _native.check(L.wgd_op_rope(qd.data_ptr(), wd.data_ptr(), n, heads, hd, start, 10000.0, 0.125, 1e-6, 0, 0, None))
    rot = qd.cpu().numpy()
    exp = oracle.rope(q, w, n, heads, hd, start, 10000.0, 0.125, 1e-6, hd, 0, True)
    near(rot, exp)


@pytest.mark.parametrize("mode,rot", [(0, 0), (1, 0), (0, 64), (1, 64)])
def test_rope_rotation_modes_and_partial_rotary(cuda, mode, rot):
    """ropeNeoxShader / ropeClassicShader, and 64-of-256 partial rotary with an unrotated tail."""
    torch = cuda
    n, heads, hd, start = 3, 5, 256 if rot else 128, 4093
    x = synth.normal(n * heads * hd, 7, mode * 10 + rot)
    xd = to_dev(torch, x)
    _native.check(_native.lib().wgd_op_rope(xd.data_ptr(), None, n, heads, hd, start, 500000.0, 1.0, 1e-5, rot, mode, None))
    exp = oracle.rope(x, None, n, heads, hd, start, 500000.0, 1.0, 1e-5, rot or hd, mode, False)
    near(xd.cpu().numpy(), exp)


def to_head_major(a, capacity, kv_heads, hd):
    return np.ascontiguousarray(a.reshape(capacity, kv_heads, hd).transpose(1, 0, 2))


@pytest.mark.parametrize("window", [2, 16])
def test_attention_verify_fixture(cuda, window):
    """verify.ts:39-54: causal GQA, start 3, batch 2, context 16."""
    torch = cuda
    heads, kvh, hd, start, n, ctx = 4, 2, 8, 3, 2, 16
    q = np.array([math.sin(i) for i in range(n * heads * hd)], np.float32)
    k = np.array([math.cos(i) for i in range(ctx * kvh * hd)], np.float32)
    v = np.array([math.sin(i / 3) for i in range(ctx * kvh * hd)], np.float32)
    out = torch.empty(n * heads * hd, dtype=torch.float32, device="cuda")
    qd, kd, vd = to_dev(torch, q), to_dev(torch, to_head_major(k, ctx, kvh, hd)), to_dev(torch, to_head_major(v, ctx, kvh, hd))
    _native.check(_native.lib().wgd_op_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr(), n, heads, kvh, hd,
                                                 start, 0.3, window, ctx, None))
    exp = oracle.attention(q, k, v, n, heads, kvh, hd, start, 0.3, window, ctx)
    near(out.cpu().numpy(), exp)


@pytest.mark.parametrize("context,start,batch,window,capacity,hd", [
    (4096, 2047, 3, 4096, 4096, 128), (32768, 32765, 3, 32768, 32768, 256), (32768, 32765, 3, 32768, 32768, 512),
    (32768, 32760, 8, 129, 136, 128)])
def test_attention_long_context_and_ring(cuda, context, start, batch, window, capacity, hd):
    """verify-context.ts:8-41 scenarios (heads 2, kv heads 1), abs tol 1e-3."""
    torch = cuda
    heads, kvh = 2, 1
    key = lambda t, d: np.sin(t * 0.013 + d * 0.37)
    val = lambda t, d: np.cos(t * 0.019 + d * 0.23)
    q = (np.sin(np.arange(batch * heads * hd) * 0.7) * 12).astype(np.float32)
    k = np.zeros(capacity * hd, np.float32)
    v = np.zeros_like(k)
    d = np.arange(hd)
    for t in range(max(0, start + batch - capacity), start + batch):
        k[(t % capacity) * hd:(t % capacity + 1) * hd] = key(t, d)
        v[(t % capacity) * hd:(t % capacity + 1) * hd] = val(t, d)
    out = torch.empty(batch * heads * hd, dtype=torch.float32, device="cuda")
    qd, kd, vd = to_dev(torch, q), to_dev(torch, k), to_dev(torch, v)
    _native.check(_native.lib().wgd_op_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr(), batch, heads, kvh,
                                                 hd, start, 0.125, window, capacity, None))
    exp = oracle.attention(q, k, v, batch, heads, kvh, hd, start, 0.125, window, capacity)
    got = out.cpu().numpy()
    assert np.max(np.abs(got - exp)) <= 1e-3


def test_argmax_semantics(cuda):
    """engine.ts:305-309 / quant.test.ts:46-49: NaN skipped, first max wins, none finite -> -1."""
    torch = cuda
    L = _native.lib()
    idx = torch.zeros(1, dtype=torch.int32, device="cuda")
    cases = [np.array([np.nan, -2, 7, 3], np.float32), np.array([np.nan, -np.inf], np.float32),
             np.array([1, 5, 5, -1], np.float32)]
    big = synth.normal(262144, 8, 1)
    big[200000] = 50.0
    big[12345] = 50.0
    big[5] = np.inf
    cases.append(big)
    for a in cases:
        xd = to_dev(torch, a)
        _native.check(L.wgd_op_argmax(xd.data_ptr(), a.size, idx.data_ptr(), None))
        assert int(idx.item()) == oracle.greedy(a)


def tiled_on_device(torch, ttype, raw, rows, cols):
    L = _native.lib()
    raw_d = to_dev(torch, raw.reshape(-1))
    nbytes = L.wgd_tiled_bytes(ttype, rows, cols)
    tiled = torch.zeros(nbytes + 16, dtype=torch.uint8, device="cuda")
    _native.check(L.wgd_op_repack_tiled(ttype, rows, cols, raw_d.data_ptr(), tiled.data_ptr(), None))
    return tiled


@pytest.mark.parametrize("ttype", [12, 14])
@pytest.mark.parametrize("rows", [16, 37])
def test_tiled_dequant_bit_exact(cuda, ttype, rows):
    """The tile-16 layout decodes to the same bits as the WGSL-order oracle (padded tail tile included)."""
    torch = cuda
    cols = 768
    raw = synth.random_blocks(ttype, rows * cols // 256, seed=13, stream=ttype, scale_std=1e-2)
    tiled = tiled_on_device(torch, ttype, raw, rows, cols)
    out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    _native.check(_native.lib().wgd_op_dequant_tiled(ttype, rows, cols, tiled.data_ptr(), out.data_ptr(), None))
    exp = oracle.decode_f32(raw, ttype, rows * cols)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), exp.view(np.uint32))


@pytest.mark.parametrize("ttype,rows,cols,batch", [
    (12, 4096, 4096, 1), (12, 28672, 4096, 1), (12, 4096, 14336, 1), (14, 4096, 4096, 1), (14, 128256 // 8, 4096, 1),
    (12, 4096, 4096, 2), (12, 1000, 4096, 3), (14, 777, 5376, 4), (12, 4096, 4096, 8), (12, 513, 21504, 1),
    (14, 37, 256, 1), (12, 16, 256, 5)])
def test_tiled_gemv_matches_oracle(cuda, ttype, rows, cols, batch):
    """Integer tensor-core GEMV (digit-plane activations) vs the f64 oracle: verify.ts tolerance."""
    torch = cuda
    raw = synth.random_blocks(ttype, rows * cols // 256, seed=14, stream=ttype)
    x = synth.normal(batch * cols, 14, 3)
    tiled = tiled_on_device(torch, ttype, raw, rows, cols)
    xd = to_dev(torch, x)
    y = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
    _native.check(_native.lib().wgd_op_gemv_tiled(ttype, rows, cols, tiled.data_ptr(), xd.data_ptr(), batch, y.data_ptr(), None))
    torch.cuda.synchronize()
    exp = oracle.matmul(raw, ttype, rows, cols, x, batch)
    got = y.cpu().numpy().reshape(batch, rows)
    near(got, exp)
    # and against the fp32 row-layout kernel: same sums to fp32 rounding
    y1 = run_gemv(torch, ttype, raw, rows, cols, x, batch)
    assert np.max(np.abs(got - y1)) <= 1e-4 * max(1.0, np.max(np.abs(y1)))
