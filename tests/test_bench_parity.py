"""The bench's in-run result check (bench.parity_check), exercised on the CPU.

The check compares one request's GPU scores, keep indices and compacted pages
with the oracle run on the same K/V.  Here the "GPU" side is the oracle's own
output, so the check must pass; mistakes planted in that output (a keep index
far from any near tie, one flipped byte in a compacted page, a perturbed score)
must each be caught.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

import bench
import kvc_workloads as W
from cases import oracle_options, oracle_request, oracle_stats
from oracle import triattention_oracle as O


def _sample(w: W.Workload, i: int, tp: int = 1) -> bench.Sample:
    k, v = W.kv_pages(w, 0)
    req = oracle_request(w, i)
    offs = O.geometric_offsets(w.options.max_model_len)
    agg, keep = O.select_request([k], oracle_stats(w), req, oracle_options(w), offs, tp)
    kd, vd = k.clone(), v.clone()
    O.materialize(kd, vd, req.src_blocks, req.dst_blocks, keep)
    n = -(-w.lengths[i] // 128)
    src, dst = req.src_blocks[:n], req.dst_blocks
    return bench.Sample(i, w.lengths[i], {0: k[src]}, {0: v[src]}, {0: kd[dst]}, {0: vd[dst]}, keep, agg,
                        None if tp == 1 else True)


@pytest.fixture(scope="module")
def w0():
    return W.config0()


def test_oracle_against_itself_passes(w0):
    s = _sample(w0, w0.compressed()[1])
    out = bench.parity_check(SimpleNamespace(world=1), w0, s)
    assert out["ok"] and out["keep_differing"] == 0 and out["bytes_equal"]
    assert out["scores_max_err_over_tol"] == 0.0


def test_tensor_parallel_check_uses_the_sharded_oracle(w0):
    s = _sample(w0, w0.compressed()[0], tp=2)
    out = bench.parity_check(SimpleNamespace(world=2), w0, s)
    assert out["ok"] and out["tp_size"] == 2 and out["ranks_identical"] is True


def test_planted_keep_mistake_is_caught(w0):
    s = _sample(w0, w0.compressed()[2])
    kept = set(s.keep.tolist())
    # replace the kept middle token with the highest score by the evicted one with the lowest
    mid = [t for t in range(4, s.tokens - 128)]
    worst_evicted = min((t for t in mid if t not in kept), key=lambda t: float(s.agg[t]))
    best_kept = max((t for t in mid if t in kept), key=lambda t: float(s.agg[t]))
    keep = sorted((kept - {best_kept}) | {worst_evicted})
    s.keep = torch.tensor(keep, dtype=torch.long)
    out = bench.parity_check(SimpleNamespace(world=1), w0, s)
    assert not out["keep_match"] and not out["ok"]


def test_planted_byte_and_score_mistakes_are_caught(w0):
    s = _sample(w0, w0.compressed()[0])
    s.k_dst[0].view(torch.int16).view(-1)[12345] ^= 1
    out = bench.parity_check(SimpleNamespace(world=1), w0, s)
    assert not out["bytes_equal"] and not out["ok"]
    s = _sample(w0, w0.compressed()[0])
    s.agg = s.agg.clone()
    s.agg[100] += 0.01 * max(1.0, abs(float(s.agg[100])))
    out = bench.parity_check(SimpleNamespace(world=1), w0, s)
    assert not out["scores_within_tol"] and not out["ok"]


def test_cpu_baseline_reports_the_sample(w0):
    s = _sample(w0, w0.compressed()[0])
    line = bench.cpu_baseline(w0, s, repeats=1)
    assert line["kind"] == "port" and line["cores"] >= 1 and line["value"] > 0
    assert str(s.tokens) in line["sample"]
