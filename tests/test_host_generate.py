"""The generate loop's host rules (engine.ts:257-301 of the reference) with a fake forward, no GPU:
prefix reuse across turns (only the new suffix is forwarded, and at least the last prompt token),
no rewind on sliding-window rings, EOS, argument checks, and the cache cleared after an error."""
import types

import pytest

from webgpu_b200.engine import PagedEngine


def engine(capacities=(512,), context=512, batch=4, eos=(), fail_at=None):
    e = PagedEngine()
    e.context, e.batch, e.ctx = context, batch, object()
    e.kv_capacities = list(capacities)
    e.tokenizer = types.SimpleNamespace(eos=set(eos), usable=True, decode=lambda ids: "".join(chr(97 + i % 26) for i in ids),
                                        chat=lambda m: [1, 2, 3])
    e.stats = lambda: {}
    e.calls = []

    def fake_forward(ids, start, logits, want_logits=False):
        e.calls.append((start, list(ids)))
        if fail_at is not None and start >= fail_at:
            raise RuntimeError("device error")
        return 100 + start + len(ids)  # the "greedy token": a function of the position
    e.forward = fake_forward
    return e


def run(e, prompt, n):
    return [t.token for t in e.generate_ids(prompt, {"maxTokens": n, "temperature": 0})]


def test_prefix_reuse_forwards_only_the_new_suffix():
    e = engine()
    a = list(range(10))
    out = run(e, a, 3)
    assert e.calls[0] == (0, [0, 1, 2, 3]) and e.calls[2] == (8, [8, 9])  # prefill in batches of 4
    assert e.tokens_in_cache == a + out[:2]  # the last generated token is never forwarded
    e.calls.clear()
    b = a + out[:2] + [50, 51]
    run(e, b, 1)
    assert e.calls == [(12, [50, 51])]


def test_exact_retry_still_evaluates_the_last_prompt_token():
    e = engine()
    a = list(range(6))
    run(e, a, 1)
    e.calls.clear()
    run(e, a, 1)
    assert e.calls == [(5, [5])]


def test_full_caches_rewind_but_sliding_rings_refill():
    a = list(range(10))
    full = engine(capacities=(512, 512))
    out = run(full, a, 3)
    full.calls.clear()
    run(full, a[:5] + [77], 1)
    assert full.calls == [(5, [77])]  # an edited turn keeps the shared 5-token prefix
    ring = engine(capacities=(512, 64))
    run(ring, a, 3)
    ring.calls.clear()
    run(ring, a[:5] + [77], 1)
    assert ring.calls[0][0] == 0  # a sliding ring cannot rewind: the prompt is forwarded again
    assert out


def test_eos_stops_and_is_not_yielded():
    e = engine(eos={100 + 4})  # the token after a 4-token prompt
    assert run(e, [1, 2, 3, 4], 5) == []
    e = engine(eos={100 + 5})
    assert run(e, [1, 2, 3, 4], 5) == [104]


def test_an_error_clears_the_cache_and_releases_the_engine():
    e = engine(fail_at=6)
    with pytest.raises(RuntimeError, match="device error"):
        run(e, [1, 2, 3, 4], 10)
    assert e.tokens_in_cache == [] and not e.busy


def test_argument_checks():
    e = engine()
    with pytest.raises(ValueError, match="maxTokens"):
        run(e, [1], 0)
    with pytest.raises(ValueError, match="Invalid sampling settings"):
        list(e.generate_ids([1], {"temperature": 3}))
    with pytest.raises(ValueError, match="Invalid sampling settings"):
        list(e.generate_ids([1], {"topK": 201}))
    # Number.isFinite / Number.isInteger accept numbers only: strings and booleans fail the same check
    for bad in ({"temperature": "0.7"}, {"topP": None}, {"topK": True}, {"topK": 2.5}):
        with pytest.raises(ValueError, match="Invalid sampling settings"):
            list(e.generate_ids([1], bad))
    with pytest.raises(ValueError, match="maxTokens"):
        list(e.generate_ids([1], {"maxTokens": True}))
    with pytest.raises(ValueError, match="user/assistant"):
        list(e.generate([{"role": "system", "content": "x"}]))
    with pytest.raises(ValueError, match="no tokens"):
        list(e.generate_ids([]))
    e.ctx = None
    with pytest.raises(RuntimeError, match="Load a model first"):
        list(e.generate_ids([1]))
