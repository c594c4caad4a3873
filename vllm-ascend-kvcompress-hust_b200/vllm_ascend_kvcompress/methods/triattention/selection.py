"""Budget selection over one score row on CUDA (reference selection.py:108-196).

``select_keep_indices`` keeps the reference's argument checks and returns the
same sorted int64 positions, computed by the segmented radix-select kernel
(``kvc_select_keep``).  Equal scores are taken lowest position first; the
reference leaves their order to torch.topk.
"""

from __future__ import annotations

import torch

from ... import _native as N
from . import kernels as K

BLOCK = 128


def validate_selection(token_count: int, budget: int, protected_prefix: int, protected_recent: int,
                       segments: int, policy: str) -> None:
    if budget <= 0 or budget > token_count:
        raise ValueError("budget must be in [1, token_count]")
    if protected_prefix < 0 or protected_recent < 0:
        raise ValueError("protected windows must be non-negative")
    if protected_prefix + protected_recent > budget:
        raise ValueError("protected windows cannot exceed the selection budget")
    if segments <= 0:
        raise ValueError("segments must be positive")
    if policy not in ("global", "v3"):
        raise ValueError(f"unsupported position policy: {policy}")


def select_keep_indices(scores: torch.Tensor, *, budget: int, protected_prefix: int, protected_recent: int,
                        segments: int, policy: str, error_flag: torch.Tensor | None = None) -> torch.Tensor:
    """Sorted positions to keep from a 1-D fp32 CUDA score row."""
    if scores.ndim != 1:
        raise ValueError("scores must be one-dimensional")
    K.require_cuda(scores)
    t = int(scores.numel())
    validate_selection(t, budget, protected_prefix, protected_recent, segments, policy)
    scores = scores.to(torch.float32).contiguous()
    pages = -(-t // BLOCK)
    dev = scores.device
    meta = torch.tensor([t, 0, pages], dtype=torch.int32, device=dev)
    plan = K.BatchPlan(num_requests=1, total_pages=pages, tokens=meta[:1], page_off=meta[1:],
                       src_blocks=meta.new_zeros(0, dtype=torch.int64), src_off=meta.new_zeros(2, dtype=torch.int64),
                       dst_blocks=meta.new_zeros(0, dtype=torch.int64), dst_off=meta.new_zeros(2, dtype=torch.int64),
                       round_start=meta.new_zeros(1, dtype=torch.int64), semantic=meta.new_zeros(1, dtype=torch.int64),
                       tokens_host=(t,), max_dst_blocks=0)
    out = torch.empty(budget, dtype=torch.int64, device=dev)
    K.select_keep(scores, plan, budget, protected_prefix, protected_recent, segments,
                  N.POLICY_V3 if policy == "v3" else N.POLICY_GLOBAL, out, error_flag)
    return out
