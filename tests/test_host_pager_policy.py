"""The weight pager's residency policy without a GPU (the reference's tests/pager.test.ts uses a
fake Compute for the same purpose). wgd_plan_residency is the exact rule wgd_model_end applies:
a resident prefix of the matrices in execution order while the budget less a 16 MiB margin allows
(cacheBudget, pager.ts:22), everything else streamed through two page slots sized for whole page
units. Also the option checks that PagedEngine.load makes before touching a model."""
import ctypes

import pytest

from webgpu_b200 import _native
from webgpu_b200.engine import MAX_BUDGET_MIB, PagedEngine

MiB = 1 << 20


def plan(sizes, allocated, budget, page=16 * MiB, unit_max=0):
    L = _native.lib()
    n = len(sizes)
    arr = (ctypes.c_uint64 * max(n, 1))(*sizes)
    res = (ctypes.c_int32 * max(n, 1))()
    slot = ctypes.c_uint64(0)
    _native.check(L.wgd_plan_residency(arr, n, allocated, budget, page, unit_max, res, ctypes.byref(slot)), "plan")
    return [int(r) for r in res[:n]], slot.value


def device_bytes(sizes, resident, allocated, slot):
    slots = 2 * ((slot + 255) // 256 * 256) if slot else 0
    return allocated + slots + sum(s for s, r in zip(sizes, resident) if r)


def test_everything_resident_when_it_fits():
    sizes = [64 * MiB] * 10
    res, slot = plan(sizes, 100 * MiB, 740 * MiB)
    assert res == [1] * 10 and slot == 0


def test_resident_prefix_then_streaming_inside_the_budget():
    sizes = [64 * MiB] * 10
    allocated, budget = 100 * MiB, 512 * MiB
    res, slot = plan(sizes, allocated, budget)
    assert slot == 16 * MiB
    # 100 + 2x16 slots = 132 MiB; each 64 MiB matrix needs 64 + 16 MiB of headroom: five fit (452 MiB), not six
    assert res == [1] * 5 + [0] * 5
    assert device_bytes(sizes, res, allocated, slot) <= budget
    assert device_bytes(sizes, res, allocated, slot) + 64 * MiB + 16 * MiB > budget


def test_a_later_smaller_matrix_still_fits_after_a_large_one_streams():
    sizes = [200 * MiB, 300 * MiB, 8 * MiB, 400 * MiB, 4 * MiB]
    res, slot = plan(sizes, 0, 512 * MiB)
    assert res == [1, 0, 1, 0, 1]
    assert device_bytes(sizes, res, 0, slot) <= 512 * MiB


def test_slots_hold_the_largest_page_unit():
    # a page unit (a group of whole rows / tiles) larger than the page size widens both slots
    res, slot = plan([64 * MiB] * 4, 0, 100 * MiB, page=16 * MiB, unit_max=20 * MiB + 7)
    assert slot == 20 * MiB + 7
    assert device_bytes([64 * MiB] * 4, res, 0, slot) <= 100 * MiB
    _, slot64 = plan([64 * MiB] * 4, 0, 100 * MiB, page=64 * MiB, unit_max=1 * MiB)
    assert slot64 == 64 * MiB


def test_rejects_sizes_that_are_not_allocation_units():
    L = _native.lib()
    arr = (ctypes.c_uint64 * 1)(1000)
    res = (ctypes.c_int32 * 1)()
    slot = ctypes.c_uint64(0)
    assert L.wgd_plan_residency(arr, 1, 0, 1 << 30, 16 * MiB, 0, res, ctypes.byref(slot)) == _native.WGD_EINVAL


def test_options_are_rejected_before_the_model_is_read(tmp_path):
    p = tmp_path / "fixture.gguf"
    p.write_bytes(bytes(24))
    for opts, msg in (({"performance": "turbo"}, "Performance must"),
                      ({"performance": "fast", "batchSize": 256}, "Batch size"),
                      ({"performance": "fast", "gpuBudgetMiB": MAX_BUDGET_MIB + 1}, "GPU budget"),
                      ({"performance": "fast", "gpuBudgetMiB": 256}, "GPU budget"),
                      ({"contextLength": 100}, "Context must")):
        with pytest.raises(ValueError, match=msg):
            PagedEngine().load(str(p), opts)
