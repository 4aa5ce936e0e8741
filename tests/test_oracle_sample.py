"""The oracle's temperature / top-k / top-p sampler (oracle.sample, engine.ts:305-324)
against a second, literal restatement of the reference function in Python: the
candidate list is pushed to, re-sorted with a stable sort by value (descending) and
popped exactly as the TypeScript does, with Math.random() replaced by a given draw.
Inputs include ties (coarsely rounded logits), non-finite values, fewer finite values
than top_k, and the reference's greedy known-answer cases (tests/quant.test.ts:46-49)."""
import math

import numpy as np
import pytest

import oracle


def js_sample(logits, temperature, top_k, top_p, uniform):
    best, best_id = -math.inf, -1
    for i, v in enumerate(logits):
        v = float(v)
        if math.isfinite(v) and v > best:
            best, best_id = v, i
    if best_id < 0:
        return -1
    if temperature == 0:
        return best_id
    cand = []
    for i, v in enumerate(logits):
        v = float(v)
        if not math.isfinite(v):
            continue
        if len(cand) < top_k or v > cand[-1][1]:
            cand.append((i, v, math.exp((v - best) / temperature)))
            cand.sort(key=lambda c: -c[1])  # Python's sort is stable, like Array.prototype.sort
            if len(cand) > top_k:
                cand.pop()
    total = 0.0
    for c in cand:
        total += c[2]
    retained, cutoff = 0.0, 0
    while cutoff < len(cand):
        retained += cand[cutoff][2]
        if retained / total >= top_p:
            cutoff += 1
            break
        cutoff += 1
    draw = uniform * retained
    for c in cand[:cutoff]:
        draw -= c[2]
        if draw <= 0:
            return c[0]
    return best_id


def test_greedy_known_answers():
    assert oracle.sample(np.array([np.nan, -2, 7, 3], np.float32), 0, 40, 0.9, 0.5) == 2
    assert oracle.sample(np.array([np.nan, -np.inf], np.float32), 0, 40, 0.9, 0.5) == -1
    assert oracle.sample(np.array([np.nan, -np.inf], np.float32), 0.7, 40, 0.9, 0.5) == -1


@pytest.mark.parametrize("seed", range(12))
def test_sample_matches_literal_restatement(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 700))
    x = rng.normal(0, float(rng.choice([0.5, 2.0, 8.0])), n).astype(np.float32)
    if seed % 3 == 0:
        x = np.round(x * 2) / 2  # many ties
    if seed % 4 == 1:
        x[rng.integers(0, n, max(1, n // 10))] = rng.choice([np.nan, np.inf, -np.inf])
    for _ in range(25):
        t = float(rng.choice([0.0, 0.05, 0.7, 1.3, 2.0]))
        k = int(rng.choice([1, 2, 5, 40, 200]))
        p = float(rng.choice([0.05, 0.5, 0.9, 1.0]))
        u = float(rng.random())
        assert oracle.sample(x, t, k, p, u) == js_sample(x, t, k, p, u), (t, k, p, u)


def test_sample_edges():
    x = np.array([1.0, 1.0, 1.0], np.float32)
    # equal logits: candidates in index order, each with probability 1
    assert [oracle.sample(x, 1.0, 3, 1.0, u) for u in (0.0, 0.3, 0.5, 0.9)] == [0, 0, 1, 2]
    # +0 and -0 are equal values (index order decides)
    z = np.array([-0.0, 0.0], np.float32)
    assert oracle.sample(z, 1.0, 1, 1.0, 0.99) == 0
    # draw at the very end of the retained mass falls back to the last candidate
    y = np.array([3.0, 2.0, 1.0], np.float32)
    assert oracle.sample(y, 1.0, 3, 1.0, 0.999999999) == js_sample(y, 1.0, 3, 1.0, 0.999999999)
