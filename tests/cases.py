"""Shared builders for parity tests: seeded inputs, oracle stats, golden loader."""

from __future__ import annotations

import json
from functools import lru_cache
from pathlib import Path

import numpy as np
import torch

import kvc_workloads as W
from oracle import triattention_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


@lru_cache(maxsize=1)
def golden():
    z = np.load(GOLDEN / "golden.npz")
    return {k: z[k] for k in z.files}, json.loads((GOLDEN / "golden.json").read_text())


def golden_small_cases() -> dict[str, W.Workload]:
    """The small workloads of make_golden.small_cases(), rebuilt from their seeds."""
    partial = W.place_blocks(W.Workload(
        "partial", W.Geometry(4, 2, 16, 256, 64, 1e7, model_type="qwen3_5_moe_text"),
        W.Options(kv_budget=1024, recompute_window=128, protected_prefix_window=16,
                  protected_recent_window=128, score_layer_stride=2, score_chunk_size=512),
        [1400, 2000], seed=5, cache_blocks_per_page=2))
    glob = W.place_blocks(W.Workload(
        "global_max", W.Geometry(3, 2, 4, 64, 64, 1e4),
        W.Options(kv_budget=512, protected_prefix_window=0, protected_recent_window=128,
                  position_policy="global", layer_aggregation="max", score_chunk_size=256,
                  score_layer_stride=1),
        [700, 1000], seed=6))
    maxagg = W.place_blocks(W.Workload(
        "score_max", W.Geometry(2, 1, 4, 64, 64, 1e6),
        W.Options(kv_budget=256, protected_prefix_window=8, protected_recent_window=128,
                  score_aggregation="max", score_layer_stride=1, score_chunk_size=256),
        [600], seed=7))
    return {w.name: w for w in (partial, glob, maxagg)}


def group_rows(t: torch.Tensor, kvh: int, g: int) -> torch.Tensor:
    """[q_heads, F] -> [kvh, G, F] (query heads ordered kv-major, as GQA does)."""
    return t.reshape(kvh, g, -1).contiguous()


def oracle_stats(w: W.Workload, payload: dict | None = None) -> list[O.LayerStats]:
    """Per-layer LayerStats grouped by KV head from the workload's payload."""
    geo = w.geometry
    payload = payload or W.calibration_payload(geo, w.seed)
    out = []
    for li in range(geo.num_layers):
        e = payload["layer_stats"][str(li)]
        kvh, g = geo.num_kv_heads, geo.group
        out.append(O.LayerStats(
            q_mean_real=group_rows(e["q_mean_real"].float(), kvh, g),
            q_mean_imag=group_rows(e["q_mean_imag"].float(), kvh, g),
            q_abs_mean=group_rows(e["q_abs_mean"].float(), kvh, g),
            freq_scale_sq=group_rows(e["freq_scale_sq"].float(), kvh, g),
            omega=e["inv_freq"].float().contiguous(),
            rotary_dim=geo.rotary_dim,
            q_pass_mean=None if "q_pass_mean" not in e else group_rows(e["q_pass_mean"].float(), kvh, g),
        ))
    return out


def oracle_options(w: W.Workload) -> O.OracleOptions:
    o = w.options
    return O.OracleOptions(
        kv_budget=o.kv_budget, protected_prefix_window=o.protected_prefix_window,
        protected_recent_window=o.protected_recent_window, position_segments=o.position_segments,
        position_policy=o.position_policy, score_aggregation=o.score_aggregation,
        layer_aggregation=o.layer_aggregation, score_chunk_size=o.score_chunk_size,
        score_layer_stride=o.score_layer_stride,
    )


def oracle_request(w: W.Workload, i: int) -> O.OracleRequest:
    return O.OracleRequest(
        semantic_num_tokens=w.lengths[i], physical_num_tokens=w.lengths[i],
        src_blocks=torch.tensor(w.src_tables[i], dtype=torch.long),
        dst_blocks=torch.tensor(w.dst_tables[i], dtype=torch.long),
    )


def cpu_caches(w: W.Workload):
    return [W.kv_pages(w, layer) for layer in range(w.geometry.num_layers)]


def near_tie_mismatches(ref_scores: torch.Tensor, ref_keep: torch.Tensor, got_keep: torch.Tensor,
                        w: W.Workload, tol: float = 1e-3) -> tuple[int, int]:
    """(#differing indices, #of them NOT explained by a near tie).

    An index may differ only if its oracle score lies within ``tol`` (relative,
    floor 1) of the oracle's kept/evicted boundary of its segment.
    """
    a = set(ref_keep.tolist())
    b = set(got_keep.tolist())
    diff = sorted(a ^ b)
    if not diff:
        return 0, 0
    o = w.options
    bounds = O.selection_boundaries(
        ref_scores, ref_keep, budget=o.kv_budget, prefix=o.protected_prefix_window,
        recent=o.protected_recent_window, segments=o.position_segments, policy=o.position_policy)
    bad = 0
    for idx in diff:
        thr = None
        for lo, hi, th in bounds:
            if lo <= idx < hi:
                thr = th
        if thr is None or abs(float(ref_scores[idx]) - thr) > tol * max(abs(thr), 1.0):
            bad += 1
    return len(diff), bad
