"""Host context policy, restating tests/context.test.ts:8-67 of the reference."""
import types

import pytest

from webgpu_b200.context import attention_memory, cache_copies, output_limit, suggest_budget, validate_context
from webgpu_b200.engine import PagedEngine


def test_context_limits_and_output_space():
    for n in (256, 4096, 12000, 32768):
        validate_context(n)
    for n in (255, 32769, 4096.5, float("nan")):
        with pytest.raises(ValueError, match="Context must"):
            validate_context(n)
    with pytest.raises(ValueError, match="model declares"):
        validate_context(32768, 8192)
    assert output_limit(32768, 100, 32768) == 32668
    assert output_limit(8192, 24000, 32768) == 8192
    assert output_limit(8192, 32767, 32768) == 1
    with pytest.raises(ValueError, match="prompt has"):
        output_limit(8192, 32768, 32768)
    with pytest.raises(ValueError, match="maxTokens"):
        output_limit(32769, 100, 32768)


def test_gemma_local_caches_keep_window_plus_batch_and_ring_wrap():
    c = types.SimpleNamespace(architecture="gemma3", family="gemma3", layers=6, period=6, window=1024, kv_heads=4, head_dim=128)
    m = attention_memory(c, 32768, 128)
    assert m["capacities"] == [1151, 1151, 1151, 1151, 1151, 32768]
    assert m["total_bytes"] == (5 * 1151 + 32768) * 4 * 128 * 8
    capacity, window, batch = 136, 129, 8
    for start in (128, 135, 136, 2047, 32760):
        ring = [-1] * capacity
        for t in range(max(0, start - capacity), start):
            ring[t % capacity] = t
        for copy in cache_copies(start, batch, capacity):
            for j in range(copy["count"]):
                ring[copy["target"] + j] = start + copy["source"] + j
        for b in range(batch):
            for t in range(max(0, start + b + 1 - window), start + b + 1):
                assert ring[t % capacity] == t


def test_llama_full_context_kv_no_sliding_window():
    c = types.SimpleNamespace(architecture="llama", family="llama", layers=3, period=0, window=0, kv_heads=2, head_dim=16,
                              sliding_window=0)
    m = attention_memory(c, 4096, 8)
    assert m["capacities"] == [4096, 4096, 4096]
    assert m["kv_bytes"] == 3 * 4096 * 2 * 16 * 8


def test_suggested_budgets():
    tiny, mid, huge = 400 * 1024 ** 2, 2 * 1024 ** 3, 16 * 1024 ** 3
    assert suggest_budget(tiny, "lite") == 1024
    assert suggest_budget(tiny, "low-memory") == 1024
    assert suggest_budget(mid, "low-memory") == 2048
    assert suggest_budget(huge, "low-memory") == 2048
    assert suggest_budget(huge, "fast") == 6144
    assert suggest_budget(tiny, "fast") == 2048
    for mode in ("lite", "low-memory", "fast"):
        for b in (0, tiny, mid, huge):
            v = suggest_budget(b, mode)
            assert 512 <= v <= 16384 and v % 256 == 0


def test_generation_runs_to_the_exact_context_boundary():
    """context.test.ts:55-67: a fake forward; 1000-token prompt, 4096 context -> 3096 tokens."""
    e = PagedEngine()
    positions = []
    e.context, e.batch, e.ctx = 4096, 128, object()
    e.config = types.SimpleNamespace(vocab=1)
    e.kv_capacities = [4096]
    e.tokenizer = types.SimpleNamespace(chat=lambda m: [0] * 1000, eos=set(), usable=True,
                                        decode=lambda ids: "a" * len(ids))
    e.stats = lambda: {}

    def fake_forward(ids, start, logits, want_logits=False):
        positions.append(start + len(ids) - 1)
        return 0
    e.forward = fake_forward
    count = 0
    for tok in e.generate([{"role": "user", "content": "x" * 20000}], {"maxTokens": 32768, "temperature": 0}):
        count += 1
        assert tok.promptTokens == 1000 and tok.contextLength == 4096
    assert count == 3096 and max(positions) == 4094
