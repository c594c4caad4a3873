"""Calibration reduction on CUDA: running per-(head, frequency) query sums.

``LayerAccumulator.add`` has the contract of the reference's stats builder
(src/vllm_ascend_kvcompress/calibration.py:87-131, ``_LayerAccumulator``): it
takes one forward's pre-RoPE query projection, accepts the packed
query+gate layout and the [..., heads, head_dim] layout, and accumulates the
sums of the real part q[:F], the imaginary part q[F:rot], the modulus and the
unrotated dims q[rot:], plus the row count.  The sums run in
``kvc_calibration_accumulate`` and stay on the device in fp64 until ``means``.
The Hugging Face model driver that feeds it (reference calibration.py:134-411)
is not part of this package.
"""

from __future__ import annotations

import torch

from .methods.triattention import kernels as K


class LayerAccumulator:
    """Online calibration sums of one attention layer."""

    def __init__(self) -> None:
        self.real_sum: torch.Tensor | None = None
        self.imag_sum: torch.Tensor | None = None
        self.abs_sum: torch.Tensor | None = None
        self.pass_sum: torch.Tensor | None = None
        self.count = 0
        self._ws: torch.Tensor | None = None

    def add(self, projected: torch.Tensor, heads: int, head_dim: int, rotary_dim: int) -> None:
        expected = heads * head_dim
        if projected.shape[-1] == expected * 2:
            projected = projected[..., :expected]  # Qwen3.5 packs the output gate after Q
        if projected.shape[-1] == expected:
            rows = projected.detach().reshape(-1, expected)
        elif projected.shape[-1] == head_dim and projected.numel() % expected == 0:
            rows = projected.detach().reshape(-1, expected)
        else:
            raise RuntimeError("query projection width does not match model attention shape: "
                               f"got {projected.shape[-1]}, expected {expected}")
        K.require_cuda(rows)
        if rows.stride(-1) != 1:
            rows = rows.contiguous()
        if rows.dtype not in (torch.bfloat16, torch.float16):
            raise RuntimeError("calibration queries must be bfloat16 or float16 on the CUDA path")
        f = rotary_dim // 2
        p = head_dim - rotary_dim
        dev = rows.device
        if self.real_sum is None:
            z = lambda w: torch.zeros(heads, w, dtype=torch.float64, device=dev)
            self.real_sum, self.imag_sum, self.abs_sum = z(f), z(f), z(f)
            self.pass_sum = z(p) if p else None
        need = K.calibration_workspace_doubles(rows.shape[0], heads, head_dim, rotary_dim)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 1), dtype=torch.float64, device=dev)
        K.calibration_accumulate(rows, heads, head_dim, rotary_dim, self.real_sum, self.imag_sum, self.abs_sum,
                                 self.pass_sum, self._ws)
        self.count += rows.shape[0]

    def means(self) -> dict[str, torch.Tensor]:
        """fp32 CPU means in the schema-3 ``layer_stats`` field names."""
        if self.count <= 0 or self.real_sum is None:
            raise RuntimeError("no query values captured for this layer")
        d = float(self.count)
        out = {
            "q_mean_real": (self.real_sum / d).float().cpu(),
            "q_mean_imag": (self.imag_sum / d).float().cpu(),
            "q_abs_mean": (self.abs_sum / d).float().cpu(),
        }
        if self.pass_sum is not None:
            out["q_pass_mean"] = (self.pass_sum / d).float().cpu()
        return out
