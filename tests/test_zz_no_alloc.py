"""wgd_op_gemv_tiled_noalloc: the tiled GEMV with fixed, non-allocated scratch.

Collected last on purpose (file name), so that it runs both after the rest of the GPU
suite and, when selected alone, in a fresh process. Each case compares two calls in a row
of the no-allocation entry point with wgd_op_gemv_tiled on the same inputs: the same
kernel with the same stream-K split, so the outputs must be bit-identical, and the second
call checks that the first left the shared tile counters zeroed.
"""
import numpy as np
import pytest

from webgpu_b200 import _native, synth

pytestmark = pytest.mark.gpu

Q4_K, Q6_K = 12, 14


def _tiled(torch, ttype, rows, cols, seed):
    L = _native.lib()
    raw = synth.random_blocks(ttype, rows * cols // 256, seed=seed, stream=ttype)
    raw_d = torch.from_numpy(np.ascontiguousarray(raw.reshape(-1))).cuda()
    tiled = torch.zeros(L.wgd_tiled_bytes(ttype, rows, cols) + 16, dtype=torch.uint8, device="cuda")
    _native.check(L.wgd_op_repack_tiled(ttype, rows, cols, raw_d.data_ptr(), tiled.data_ptr(), None))
    return tiled


@pytest.mark.parametrize("ttype,rows,cols,batch", [
    (Q4_K, 4096, 4096, 1), (Q4_K, 28672, 4096, 1), (Q4_K, 4096, 14336, 1), (Q6_K, 6144, 4096, 1),
    (Q4_K, 1000, 4096, 3), (Q6_K, 777, 5376, 4), (Q4_K, 16, 256, 5)])
def test_noalloc_matches_allocating_entry(cuda, ttype, rows, cols, batch):
    torch = cuda
    L = _native.lib()
    tiled = _tiled(torch, ttype, rows, cols, seed=rows + cols)
    x = torch.from_numpy(synth.normal(batch * cols, 21, 5)).cuda()
    ref = torch.full((batch * rows,), float("nan"), device="cuda")
    _native.check(L.wgd_op_gemv_tiled(ttype, rows, cols, tiled.data_ptr(), x.data_ptr(), batch, ref.data_ptr(), None))
    outs = []
    for _ in range(2):
        y = torch.full((batch * rows,), float("nan"), device="cuda")
        _native.check(L.wgd_op_gemv_tiled_noalloc(ttype, rows, cols, tiled.data_ptr(), x.data_ptr(), batch, y.data_ptr(), None))
        outs.append(y)
    torch.cuda.synchronize()
    assert torch.isfinite(ref).all()
    for y in outs:
        assert torch.equal(y.view(torch.int32), ref.view(torch.int32))


def test_noalloc_on_a_side_stream(cuda):
    """Same result when issued on a non-default stream, twice in a row."""
    torch = cuda
    L = _native.lib()
    rows, cols = 6144, 4096
    tiled = _tiled(torch, Q4_K, rows, cols, seed=5)
    x = torch.from_numpy(synth.normal(cols, 22, 5)).cuda()
    ref = torch.empty(rows, device="cuda")
    _native.check(L.wgd_op_gemv_tiled(Q4_K, rows, cols, tiled.data_ptr(), x.data_ptr(), 1, ref.data_ptr(), None))
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    ys = [torch.empty(rows, device="cuda") for _ in range(2)]
    with torch.cuda.stream(s):
        for y in ys:
            _native.check(L.wgd_op_gemv_tiled_noalloc(Q4_K, rows, cols, tiled.data_ptr(), x.data_ptr(), 1, y.data_ptr(),
                                                      s.cuda_stream))
    s.synchronize()
    for y in ys:
        assert torch.equal(y, ref)


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda):
    """A 128256-row output head needs ~5.9 MiB of partials: refused with a clear error and no kernel launch."""
    torch = cuda
    L = _native.lib()
    rows, cols = 128256, 4096
    x = torch.zeros(cols, device="cuda")
    y = torch.zeros(rows, device="cuda")
    w = torch.zeros(16, dtype=torch.uint8, device="cuda")  # never read: the shape check comes first
    with pytest.raises(_native.WgdError, match="fixed scratch"):
        _native.check(L.wgd_op_gemv_tiled_noalloc(Q6_K, rows, cols, w.data_ptr(), x.data_ptr(), 1, y.data_ptr(), None))
    with pytest.raises(_native.WgdError, match="bad type"):
        _native.check(L.wgd_op_gemv_tiled_noalloc(Q4_K, 16, 100, w.data_ptr(), x.data_ptr(), 1, y.data_ptr(), None))


def test_noalloc_calls_allocate_no_device_memory(cuda):
    """After the first call on the device, further calls leave the device's free memory and the
    torch allocator's bytes unchanged: the scratch is the fixed array, never an allocation."""
    torch = cuda
    L = _native.lib()
    rows, cols = 4096, 14336
    tiled = _tiled(torch, Q4_K, rows, cols, seed=9)
    x = torch.from_numpy(synth.normal(cols, 23, 5)).cuda()
    y = torch.empty(rows, device="cuda")
    _native.check(L.wgd_op_gemv_tiled_noalloc(Q4_K, rows, cols, tiled.data_ptr(), x.data_ptr(), 1, y.data_ptr(), None))
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    torch0 = torch.cuda.memory_allocated()
    for _ in range(5):
        _native.check(L.wgd_op_gemv_tiled_noalloc(Q4_K, rows, cols, tiled.data_ptr(), x.data_ptr(), 1, y.data_ptr(), None))
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.cuda.memory_allocated() == torch0
