"""Helpers for the GPU parity tests (CUDA path through the C ABI vs the CPU oracle)."""

from __future__ import annotations

import torch

import kvc_workloads as W
from cases import near_tie_mismatches, oracle_options, oracle_request, oracle_stats
from oracle import triattention_oracle as O

SCORE_TOL = 1e-3  # |d| <= 1e-3 * max(|ref|, 1) on fp32 scores (the benchmark's 1e-3 relative bound)


def to_gpu(cpu_caches):
    return [(k.cuda(), v.cuda()) for k, v in cpu_caches]


def bind(w: W.Workload, gpu_caches, tmp_path, **kw):
    return W.b200_method(w, gpu_caches, W.write_stats_file(w, tmp_path), **kw)


def oracle_select(w: W.Workload, cpu_caches, indices=None, tp_size: int = 1):
    stats = oracle_stats(w)
    opts = oracle_options(w)
    offs = O.geometric_offsets(w.options.max_model_len)
    out = {}
    for i in (indices if indices is not None else w.compressed()):
        out[i] = O.select_request([c[0] for c in cpu_caches], stats, oracle_request(w, i), opts, offs, tp_size)
    return out


def assert_scores_close(got: torch.Tensor, ref: torch.Tensor, tol: float = SCORE_TOL) -> None:
    got, ref = got.float().cpu(), ref.float().cpu()
    finite = torch.isfinite(ref)
    assert torch.equal(finite, torch.isfinite(got)), "non-finite pattern differs"
    err = (got[finite] - ref[finite]).abs()
    bound = tol * ref[finite].abs().clamp_min(1.0)
    worst = (err / bound).max().item() if err.numel() else 0.0
    assert worst <= 1.0, f"score error {worst:.3g}x over the tolerance"


def assert_selection(w: W.Workload, ref_agg, ref_keep, got_keep) -> int:
    got_keep = got_keep.cpu()
    assert got_keep.numel() == w.options.kv_budget
    assert bool((got_keep[1:] > got_keep[:-1]).all()), "keep indices must be strictly increasing"
    n, bad = near_tie_mismatches(ref_agg, ref_keep, got_keep, w)
    assert bad == 0, f"{bad} of {n} differing indices are not near ties"
    return n


def page_offsets(w: W.Workload, indices) -> list[int]:
    """Token offset of each request inside the page-padded batch space."""
    out, pos = [], 0
    for i in indices:
        out.append(pos * 128)
        pos += -(-w.lengths[i] // 128)
    return out


def assert_compaction(w: W.Workload, cpu_caches, gpu_caches, keeps: dict[int, torch.Tensor]) -> None:
    """Apply the oracle compaction with the GPU's own keep sets; bytes must match."""
    for i, keep in keeps.items():
        req = oracle_request(w, i)
        for kc, vc in cpu_caches:
            O.materialize(kc, vc, req.src_blocks, req.dst_blocks, keep.cpu())
    for i in keeps:
        dst = torch.tensor(w.dst_tables[i])
        for (kc, vc), (kg, vg) in zip(cpu_caches, gpu_caches):
            assert torch.equal(kc[dst].view(torch.int16), kg[dst.cuda()].cpu().view(torch.int16))
            assert torch.equal(vc[dst].view(torch.int16), vg[dst.cuda()].cpu().view(torch.int16))
