"""Pin the CPU oracle to the reference: golden vectors + the reference's known answers.

The golden vectors were produced by running the reference plugin itself
(tests/golden/make_golden.py).  Known-answer cases restate the literal values of
the reference's tests (tests/test_scoring.py, test_selection.py, test_cache.py).
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

import kvc_workloads as W
from cases import (  # noqa: I001
    cpu_caches,
    golden,
    golden_small_cases,
    oracle_options,
    oracle_request,
    oracle_stats,
)
from oracle import triattention_oracle as O


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def _workloads():
    return {"config0": W.config0(), **golden_small_cases()}


@pytest.mark.parametrize("name", ["config0", "partial", "global_max", "score_max"])
def test_oracle_matches_reference_golden(name):
    arrays, spec = golden()
    w = _workloads()[name]
    assert spec[name]["lengths"] == w.lengths
    assert spec[name]["compressed"] == w.compressed()
    caches = cpu_caches(w)
    stats = oracle_stats(w)
    opts = oracle_options(w)
    offs = O.geometric_offsets(w.options.max_model_len)
    for i in w.compressed():
        req = oracle_request(w, i)
        rows, extras = O.layer_rows([c[0] for c in caches], stats, req, opts, offs, keep_raw=True)
        agg = O.aggregate_rows(rows, opts.layer_aggregation)
        keep = O.select_keep_indices(
            agg, budget=opts.kv_budget, protected_prefix=opts.protected_prefix_window,
            protected_recent=opts.protected_recent_window, segments=opts.position_segments,
            policy=opts.position_policy)
        g_agg = torch.from_numpy(arrays[f"{name}/r{i}/agg"])
        torch.testing.assert_close(agg, g_agg, rtol=1e-5, atol=1e-5)
        assert torch.equal(keep, torch.from_numpy(arrays[f"{name}/r{i}/keep"]))
        raw, mean, var = extras[0]
        torch.testing.assert_close(raw[..., :256], torch.from_numpy(arrays[f"{name}/r{i}/raw_head"]),
                                   rtol=1e-5, atol=1e-4)
        torch.testing.assert_close(mean, torch.from_numpy(arrays[f"{name}/r{i}/mean"]), rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(var, torch.from_numpy(arrays[f"{name}/r{i}/var"]), rtol=1e-5, atol=1e-5)
        for kc, vc in caches:
            O.materialize(kc, vc, req.src_blocks, req.dst_blocks, keep)
        for li, (kc, vc) in enumerate(caches):
            assert _sha(kc[req.dst_blocks]) == spec[name]["dest_hashes"][f"r{i}/layer{li}/k"]
            assert _sha(vc[req.dst_blocks]) == spec[name]["dest_hashes"][f"r{i}/layer{li}/v"]


def test_oracle_tp2_max_sync_matches_reference_golden():
    arrays, spec = golden()
    w = golden_small_cases()["partial"]
    caches = cpu_caches(w)
    stats = oracle_stats(w)
    opts = oracle_options(w)
    offs = O.geometric_offsets(w.options.max_model_len)
    half = w.geometry.num_kv_heads // 2
    for i in w.compressed():
        req = oracle_request(w, i)
        rows = []
        for r in (0, 1):
            kc = [c[0][:, :, r * half:(r + 1) * half] for c in caches]
            rows.append(O.layer_rows(kc, [s.shard(r, 2) for s in stats], req, opts, offs))
            torch.testing.assert_close(rows[r], torch.from_numpy(arrays[f"partial/r{i}/rows_rank{r}"]),
                                       rtol=1e-5, atol=1e-5)
        agg, keep = O.select_request([c[0] for c in caches], stats, req, opts, offs, tp_size=2)
        assert torch.equal(keep, torch.from_numpy(arrays[f"partial/r{i}/keep_tp2"]))
        # TP=2 selection equals TP=1 selection (MAX commutes with head sharding)
        assert torch.equal(keep, torch.from_numpy(arrays[f"partial/r{i}/keep"]))
        torch.testing.assert_close(agg, torch.from_numpy(arrays[f"partial/r{i}/agg_tp2"]), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("case", ["calib_full", "calib_partial"])
def test_oracle_calibration_matches_reference_golden(case):
    arrays, spec = golden()
    inputs = {n: (h, d, r, q) for n, h, d, r, q in W.golden_calibration_inputs()}
    heads, hd, rot, calls = inputs[case]
    acc = O.CalibrationSums()
    for q in calls:
        acc.add(q, heads, hd, rot)
    assert acc.count == spec[case]["count"]
    for k in ("real_sum", "imag_sum", "abs_sum", "pass_sum"):
        key = f"{case}/{k}"
        if key in arrays:
            torch.testing.assert_close(getattr(acc, k), torch.from_numpy(arrays[key]), rtol=1e-6, atol=1e-4)


def test_oracle_selection_matches_reference_golden():
    arrays, spec = golden()
    cases = spec["selection"]
    scores = W.golden_selection_scores(cases)
    for n, (t, b, p, r, s, pol) in enumerate(cases):
        keep = O.select_keep_indices(scores[n], budget=b, protected_prefix=p, protected_recent=r,
                                     segments=s, policy=pol)
        assert keep.numel() == b
        assert np.array_equal(keep.numpy(), arrays[f"selection/{n}/keep"]), (t, b, p, r, s, pol)


# ---- known answers restated from the reference's own tests -----------------


def _kat_stats():
    return O.LayerStats(
        q_mean_real=torch.tensor([[[1.0, 0.5], [0.25, 0.75]]]),
        q_mean_imag=torch.tensor([[[0.0, 0.5], [0.5, 0.25]]]),
        q_abs_mean=torch.ones(1, 2, 2),
        freq_scale_sq=torch.ones(1, 2, 2),
        omega=torch.tensor([1.0, 0.1]),
    )


def test_kat_vectorized_mean_equals_per_offset_loop():
    """reference tests/test_scoring.py:53-70 (slow per-offset reference)."""
    keys = torch.tensor([[[1.0, 2.0, 3.0, 4.0]], [[0.5, 1.5, 2.5, 3.5]], [[2.0, 1.0, 4.0, 3.0]]])
    offsets = torch.tensor([1.0, 2.0, 4.0])
    st = _kat_stats()
    got = O.score_keys(keys, st, round_start=3, offsets=offsets)
    kr = keys[..., :2].permute(1, 0, 2).unsqueeze(1)
    ki = keys[..., 2:].permute(1, 0, 2).unsqueeze(1)
    qr, qi = st.q_mean_real.unsqueeze(2), st.q_mean_imag.unsqueeze(2)
    pr, pi = qr * kr + qi * ki, qi * kr - qr * ki
    per = [(pr * torch.cos((3.0 + o) * st.omega) - pi * torch.sin((3.0 + o) * st.omega)).sum(-1) for o in offsets]
    qabs = torch.sqrt(st.q_mean_real.square() + st.q_mean_imag.square() + 1e-8)
    expected = torch.stack(per).mean(0) + (torch.sqrt(kr.square() + ki.square()) * (st.q_abs_mean - qabs).unsqueeze(2)).sum(-1)
    torch.testing.assert_close(got, expected)


def test_kat_query_side_scale_gives_four():
    """reference tests/test_scoring.py:85-104."""
    st = O.LayerStats(torch.ones(1, 1, 1), torch.zeros(1, 1, 1), torch.ones(1, 1, 1),
                      torch.full((1, 1, 1), 4.0), torch.zeros(1))
    got = O.score_keys(torch.tensor([[[2.0, 0.0]]]), st, round_start=1, offsets=torch.tensor([1.0]))
    torch.testing.assert_close(got, torch.tensor([[[4.0]]]))


def test_kat_partial_rope_content_term():
    """reference tests/test_scoring.py:107-133 -> [2, -5]."""
    st = O.LayerStats(torch.zeros(1, 1, 1), torch.zeros(1, 1, 1), torch.zeros(1, 1, 1),
                      torch.ones(1, 1, 1), torch.zeros(1), rotary_dim=2,
                      q_pass_mean=torch.tensor([[[2.0, -1.0]]]))
    keys = torch.tensor([[[0.0, 0.0, 3.0, 4.0]], [[0.0, 0.0, -2.0, 1.0]]])
    got = O.score_keys(keys, st, round_start=1, offsets=torch.tensor([1.0]))
    torch.testing.assert_close(got, torch.tensor([[[2.0, -5.0]]]))


def test_kat_v3_evicts_one_per_segment():
    """reference tests/test_selection.py:60-75 -> evicted {2, 5, 8, 11}."""
    keep = O.select_keep_indices(torch.arange(16, dtype=torch.float32), budget=12, protected_prefix=2,
                                 protected_recent=2, segments=4, policy="v3")
    assert set(range(16)) - set(keep.tolist()) == {2, 5, 8, 11}


def test_kat_v3_uneven_segments_exact_budget():
    """reference tests/test_selection.py:78-91."""
    keep = O.select_keep_indices(torch.zeros(19), budget=13, protected_prefix=2, protected_recent=2,
                                 segments=8, policy="v3")
    assert keep.numel() == 13 and {0, 1, 17, 18} <= set(keep.tolist())


def test_kat_global_policy():
    """reference tests/test_selection.py:144-154 -> [0, 1, 4, 5]."""
    keep = O.select_keep_indices(torch.tensor([10.0, 9.0, 8.0, 7.0, -5.0, -6.0]), budget=4,
                                 protected_prefix=0, protected_recent=2, segments=8, policy="global")
    assert keep.tolist() == [0, 1, 4, 5]


def test_kat_gather_through_block_table():
    """reference tests/test_cache.py:39-47 -> [8, 11, 0, 3]."""
    cache = torch.arange(12, dtype=torch.float32).view(3, 4, 1, 1)
    got = O.gather_slots(cache, O.token_slots(torch.tensor([2, 0]), torch.tensor([0, 3, 4, 7]), 4))
    assert got.flatten().tolist() == [8.0, 11.0, 0.0, 3.0]


def test_kat_overlapping_destination_gathers_first():
    """reference tests/test_cache.py:15-36: destination block is also a source block."""
    k = torch.arange(16, dtype=torch.float32).view(4, 4, 1, 1)
    v = k.clone() + 100
    src, keep = torch.tensor([2, 0, 3]), torch.tensor([1, 4, 6, 9])
    ek = O.gather_slots(k, O.token_slots(src, keep, 4)).clone()
    ev = O.gather_slots(v, O.token_slots(src, keep, 4)).clone()
    O.materialize(k, v, src, torch.tensor([2]), keep, 4)
    torch.testing.assert_close(k[2], ek)
    torch.testing.assert_close(v[2], ev)


def test_kat_padded_interleaved_pages_keep_unused_bytes():
    """reference tests/test_cache.py:50-93: K and V share a padded raw buffer."""
    bs, nb, heads, dim = 4, 4, 1, 2
    page = bs * heads * dim
    stride = 2 * page + 4
    raw = torch.full((nb * stride,), -1, dtype=torch.float16)
    shape, strides = (nb, bs, heads, dim), (stride, heads * dim, dim, 1)
    k = torch.as_strided(raw, shape, strides)
    v = torch.as_strided(raw, shape, strides, storage_offset=page)
    k.copy_(torch.arange(nb * page).view(shape))
    v.copy_(torch.arange(nb * page).view(shape) + 100)
    src, keep = torch.tensor([2, 0, 3]), torch.tensor([1, 4, 6, 9])
    ek = O.gather_slots(k, O.token_slots(src, keep, bs)).clone()
    ev = O.gather_slots(v, O.token_slots(src, keep, bs)).clone()
    O.materialize(k, v, src, torch.tensor([2]), keep, bs)
    torch.testing.assert_close(k[2], ek)
    torch.testing.assert_close(v[2], ev)
    torch.testing.assert_close(raw.view(nb, stride)[:, -4:], torch.full((nb, 4), -1, dtype=torch.float16))


def test_kat_shift_positions():
    """reference tests/run_npu_kernel_smoke.py:31-40 -> [128, 20, 129]."""
    got = O.shift_positions(torch.tensor([300, 20, 301]), torch.tensor([0, 1, 0]), torch.tensor([172, 0]))
    assert got.tolist() == [128, 20, 129]
