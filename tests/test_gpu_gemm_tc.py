"""The prompt-batch tcgen05 GEMM (wgd_op_gemm_tiled) against the CPU oracle and
against the integer tensor-core GEMV on the same tiled Q4_K / Q6_K weights.

Shapes are the quantised-GEMM microbench ones (4096x4096, 14336x4096, 4096x14336
at batch 8/32/128) plus ragged cases: a last 16-row tile and a last 128-row
M-tile that are partly empty, one super-block of columns, batches that are not
multiples of 16, and M-tiles cut between several CTAs (split-K partials summed
by the last CTA). Tolerance: the reference's verify.ts bound against the f64
oracle, and fp32 rounding against the GEMV (both read the same weights
exactly)."""
import ctypes

import numpy as np
import pytest

import oracle
from webgpu_b200 import _native, synth
from test_gpu_ops import near, tiled_on_device, to_dev

pytestmark = pytest.mark.gpu
Q4K, Q6K = 12, 14


def _gemm(torch, tiled, rows, cols, xd, batch, ttype=Q4K):
    y = torch.full((batch * rows,), float("nan"), dtype=torch.float32, device="cuda")
    _native.check(_native.lib().wgd_op_gemm_tiled(ttype, rows, cols, tiled.data_ptr(), xd.data_ptr(), batch, y.data_ptr(), None))
    st = ctypes.c_int(-1)
    _native.check(_native.lib().wgd_op_gemm_tiled_status(ctypes.byref(st)))
    assert st.value == 0, "a pipeline wait ran out"
    return y.cpu().numpy().reshape(batch, rows)


def _gemv(torch, tiled, rows, cols, xd, batch, ttype=Q4K):
    y = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
    _native.check(_native.lib().wgd_op_gemv_tiled(ttype, rows, cols, tiled.data_ptr(), xd.data_ptr(), batch, y.data_ptr(), None))
    torch.cuda.synchronize()
    return y.cpu().numpy().reshape(batch, rows)


@pytest.mark.parametrize("rows,cols,batch,with_oracle", [
    (4096, 4096, 8, True), (4096, 4096, 32, True), (4096, 4096, 128, True),
    (14336, 4096, 32, True), (14336, 4096, 128, False), (4096, 14336, 32, True), (4096, 14336, 128, False),
    (1000, 4096, 17, True), (300, 512, 33, True), (16, 256, 1, True), (37, 256, 5, True), (6144, 4096, 128, False),
    (28672, 4096, 64, False), (1024, 14336, 100, True)])
def test_gemm_matches_oracle_and_gemv(cuda, rows, cols, batch, with_oracle):
    torch = cuda
    raw = synth.random_blocks(Q4K, rows * cols // 256, seed=21, stream=Q4K)
    x = synth.normal(batch * cols, 22, 3)
    tiled = tiled_on_device(torch, Q4K, raw, rows, cols)
    xd = to_dev(torch, x)
    got = _gemm(torch, tiled, rows, cols, xd, batch)
    assert np.all(np.isfinite(got))
    ref = _gemv(torch, tiled, rows, cols, xd, batch)
    scale = max(1.0, float(np.max(np.abs(ref))))
    assert np.max(np.abs(got - ref)) <= 1e-4 * scale, np.max(np.abs(got - ref)) / scale
    if with_oracle:
        near(got, oracle.matmul(raw, Q4K, rows, cols, x, batch))


def test_gemm_is_deterministic_and_scale_invariant(cuda):
    """Same inputs -> the same bits (split-K partials are summed in CTA order); activations
    scaled by a power of two -> results scaled exactly (the per-row power-of-two scaling)."""
    torch = cuda
    rows, cols, batch = 4096, 4096, 48
    raw = synth.random_blocks(Q4K, rows * cols // 256, seed=23, stream=Q4K)
    x = synth.normal(batch * cols, 24, 3)
    tiled = tiled_on_device(torch, Q4K, raw, rows, cols)
    a = _gemm(torch, tiled, rows, cols, to_dev(torch, x), batch)
    b = _gemm(torch, tiled, rows, cols, to_dev(torch, x), batch)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    for k in (-30, 40):  # far outside the f16 range before the row scaling
        c = _gemm(torch, tiled, rows, cols, to_dev(torch, x * np.float32(2.0 ** k)), batch)
        assert np.array_equal((a * np.float32(2.0 ** k)).view(np.uint32), c.view(np.uint32))


def test_gemm_zero_and_large_rows(cuda):
    """An all-zero activation row gives zeros; rows with |x| ~ 1e6 stay exact to fp32 rounding."""
    torch = cuda
    rows, cols, batch = 512, 1024, 20
    raw = synth.random_blocks(Q4K, rows * cols // 256, seed=25, stream=Q4K)
    x = synth.normal(batch * cols, 26, 3).reshape(batch, cols)
    x[3] = 0.0
    x[7] *= np.float32(1e6)
    tiled = tiled_on_device(torch, Q4K, raw, rows, cols)
    got = _gemm(torch, tiled, rows, cols, to_dev(torch, x.reshape(-1)), batch)
    assert np.all(got[3] == 0.0)
    exp = oracle.matmul(raw, Q4K, rows, cols, x.reshape(-1), batch)
    for r in range(batch):
        s = max(1.0, float(np.max(np.abs(exp[r]))))
        assert np.max(np.abs(got[r] - exp[r])) <= 1e-5 * s, (r, np.max(np.abs(got[r] - exp[r])) / s)


@pytest.mark.parametrize("rows,cols,batch,with_oracle", [
    (4096, 4096, 32, True), (4096, 4096, 128, False), (4096, 14336, 128, False), (1000, 4096, 17, True), (300, 512, 33, True),
    (37, 256, 5, True), (2048, 5376, 64, True)])
def test_gemm_q6k_matches_oracle_and_gemv(cuda, rows, cols, batch, with_oracle):
    """Q6_K: A = sc*(q-32) as two exact f16 terms (even part and last bit of the scale), four MMAs per K-step."""
    torch = cuda
    raw = synth.random_blocks(Q6K, rows * cols // 256, seed=27, stream=Q6K)
    x = synth.normal(batch * cols, 28, 3)
    tiled = tiled_on_device(torch, Q6K, raw, rows, cols)
    xd = to_dev(torch, x)
    got = _gemm(torch, tiled, rows, cols, xd, batch, Q6K)
    assert np.all(np.isfinite(got))
    ref = _gemv(torch, tiled, rows, cols, xd, batch, Q6K)
    scale = max(1.0, float(np.max(np.abs(ref))))
    assert np.max(np.abs(got - ref)) <= 1e-4 * scale, np.max(np.abs(got - ref)) / scale
    if with_oracle:
        exp = oracle.matmul(raw, Q6K, rows, cols, x, batch)
        near(got, exp)
        # exact weights: relative error at the level of the fp32 sums, not of f16
        assert np.max(np.abs(got - exp)) <= 1e-5 * max(1.0, float(np.max(np.abs(exp))))


def test_gemm_rejects_unsupported_shapes(cuda):
    L = _native.lib()
    for t, rows, cols, batch in [(13, 64, 256, 8), (Q4K, 64, 300, 8), (Q4K, 64, 256, 0), (Q4K, 64, 256, 129)]:
        assert L.wgd_op_gemm_tiled(t, rows, cols, 1, 1, batch, 1, None) != 0
