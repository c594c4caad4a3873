"""Invariants of the oracle's selection on random inputs (CPU, hypothesis).

The golden vectors pin the oracle to the reference on fixed cases; these
properties check the restated quota plan and selection everywhere else:
exactly `budget` sorted unique positions, protected windows kept, per-segment
keep counts equal to the V3 plan, quotas summing to the eviction count, and
every kept middle token scoring at least as high as every evicted one of its
segment (global: of the whole middle).
"""

from __future__ import annotations

import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import triattention_oracle as O


@st.composite
def selection_case(draw):
    t = draw(st.integers(1, 600))
    budget = draw(st.integers(1, t))
    prefix = draw(st.integers(0, budget))
    recent = draw(st.integers(0, budget - prefix))
    segments = draw(st.integers(1, 40))
    policy = draw(st.sampled_from(["global", "v3"]))
    seed = draw(st.integers(0, 2 ** 31 - 1))
    ties = draw(st.booleans())
    g = torch.Generator().manual_seed(seed)
    scores = torch.randint(0, 4, (t,), generator=g).float() if ties else torch.randn(t, generator=g)
    return scores, budget, prefix, recent, segments, policy


@settings(max_examples=300, deadline=None)
@given(selection_case())
def test_selection_invariants(case):
    scores, budget, prefix, recent, segments, policy = case
    t = scores.numel()
    p = min(prefix, t)
    r = min(recent, t - p)
    if policy == "v3" and t - budget > t - p - r:
        with pytest.raises(ValueError):
            O.select_keep_indices(scores, budget=budget, protected_prefix=prefix, protected_recent=recent,
                                  segments=segments, policy=policy)
        return
    keep = O.select_keep_indices(scores, budget=budget, protected_prefix=prefix, protected_recent=recent,
                                 segments=segments, policy=policy)
    assert keep.dtype == torch.int64 and keep.numel() == budget
    assert torch.equal(keep, torch.unique(keep))  # sorted ascending, unique
    assert int(keep.min()) >= 0 and int(keep.max()) < t
    kept = torch.zeros(t, dtype=torch.bool)
    kept[keep] = True
    assert bool(kept[:p].all()) and bool(kept[t - r:].all())
    if policy == "v3":
        plan = O.v3_segments(t, budget, p, r, segments)
        assert sum((b - a) - k for a, b, k in plan) == t - budget  # quotas sum to the evictions
        ranges = [(a, b, k) for a, b, k in plan]
    else:
        ranges = [(p, t - r, budget - p - r)]
    for a, b, k in ranges:
        seg_kept = kept[a:b]
        assert int(seg_kept.sum()) == k
        if 0 < k < b - a:
            assert float(scores[a:b][seg_kept].min()) >= float(scores[a:b][~seg_kept].max())


@settings(max_examples=200, deadline=None)
@given(st.integers(1, 100_000), st.integers(0, 100), st.integers(0, 100), st.integers(1, 64), st.data())
def test_v3_plan_partitions_the_middle(t, prefix, recent, segments, data):
    if prefix + recent > t:
        return
    budget = data.draw(st.integers(max(1, prefix + recent), t))
    m = t - prefix - recent
    if t - budget > m or m == 0:
        return
    plan = O.v3_segments(t, budget, prefix, recent, segments)
    assert plan[0][0] == prefix and plan[-1][1] == t - recent
    assert all(plan[i][1] == plan[i + 1][0] for i in range(len(plan) - 1))
    assert all(0 <= k <= b - a for a, b, k in plan)
    assert sum(k for _, _, k in plan) == budget - prefix - recent
