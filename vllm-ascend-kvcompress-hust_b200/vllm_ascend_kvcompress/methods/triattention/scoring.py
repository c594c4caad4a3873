"""Scoring helpers shared by the method and the CUDA scorer.

The per-token trigonometric score itself runs in ``kvc_score_paged_keys``
(see kernels.py); this module keeps the reference's offset construction
(src/vllm_ascend_kvcompress/methods/triattention/scoring.py:11-20).
"""

from __future__ import annotations

import torch


def build_geometric_offsets(maximum: int, device: torch.device) -> torch.Tensor:
    """Future-query offsets 1, 2, 4, ... up to ``maximum`` (fp32, on ``device``)."""
    if maximum < 1:
        raise ValueError("maximum scoring offset must be positive")
    n = maximum.bit_length()  # 2**(n-1) <= maximum < 2**n
    return torch.tensor([float(1 << i) for i in range(n)], dtype=torch.float32, device=device)
