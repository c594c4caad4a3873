"""Tensor-core scorers on low-|q| heads (coefficients 1e-6 .. 1e-4), fp16 and bf16 caches.

Calibration artefacts hold heads whose mean query is small, so their folded
scoring coefficients are 1e-4 .. 1e-6.  The tensor-core scorers split every
fp32 coefficient into 16-bit hi + lo halves; in fp16 such values would fall
into the subnormal range and lose the lo half, which is why W is scaled per
(request, layer, head) by a power of two before the split and the sums are
scaled back (kvc_score_tc.cuh, w_scale).  Here each head's raw scores and its
mean / variance must match the fp32 CUDA-core scorer to 2e-5 of that head's
own scale (measured: <= 3.5e-6; without the scaling fp16 caches reach
1.7e-4 .. 3.8e-4).
"""

from __future__ import annotations

import pytest
import torch

import kvc_workloads as W
from gpu_cases import page_offsets

pytestmark = pytest.mark.gpu

GEOMETRIES = {
    # full RoPE, head_dim 128 (rotary/2 = 64, no pass band)
    "full": (W.Geometry(1, 2, 10, 128, 128, 1e6),
             W.Options(kv_budget=512, protected_prefix_window=4, protected_recent_window=64, score_layer_stride=1),
             [900, 1700]),
    # partial RoPE, head_dim 256, rotary 64 (pass band of 192)
    "partial": (W.Geometry(1, 1, 8, 256, 64, 1e7, model_type="qwen3_5_moe_text"),
                W.Options(kv_budget=768, protected_prefix_window=128, protected_recent_window=128,
                          score_layer_stride=1), [2100, 1500]),
}


def _small_stats(w: W.Workload, directory) -> str:
    """The benchmark's random statistics with each query head scaled into 1e-6 .. 1e-4."""
    payload = W.calibration_payload(w.geometry, w.seed)
    scale = torch.logspace(-6, -4, w.geometry.num_q_heads).unsqueeze(1)
    for entry in payload["layer_stats"].values():
        for key in ("q_mean_real", "q_mean_imag", "q_abs_mean", "q_pass_mean"):
            if key in entry:
                entry[key] = (entry[key] * scale).contiguous()
    path = directory / f"{w.name}-small-stats.pt"
    torch.save(payload, path)
    return str(path)


@pytest.mark.parametrize("scorer", ["tensor", "tcgen05"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("which", sorted(GEOMETRIES))
def test_low_magnitude_heads_keep_fp32_agreement(which, dtype, scorer, tmp_path, monkeypatch):
    geo, opts, lengths = GEOMETRIES[which]
    w = W.place_blocks(W.Workload(f"small_{which}", geo, opts, lengths, seed=41))
    stats = _small_stats(w, tmp_path)
    caches = [tuple(t.cuda() for t in W.kv_pages(w, layer, dtype=dtype)) for layer in range(geo.num_layers)]
    idx = w.compressed()
    out = {}
    for kind in (scorer, "fma"):
        monkeypatch.setenv("KVC_B200_SCORER", kind)
        m = W.b200_method(w, caches, stats)
        assert m.use_tensor_scorer == (kind != "fma")
        m.select_many(W.b200_requests(w, indices=idx))
        m.check_device_errors()
        raw, mean, var, _ = (t.detach().clone().cpu() for t in m.last_stats)
        heads = m.local_kv_heads * m.group
        pages = raw.numel() // (m.scoring_layer_count * heads * 128)
        out[kind] = (raw.view(m.scoring_layer_count, pages, heads, 128), mean.view(-1, heads),
                     var.view(-1, heads))
    (rt, mt, vt), (rf, mf, vf) = out[scorer], out["fma"]
    offs = page_offsets(w, idx)
    for row, i in enumerate(idx):
        p0, n = offs[row] // 128, lengths[i]
        pg = -(-n // 128)
        for h in range(rt.shape[2]):
            got = rt[:, p0:p0 + pg, h].reshape(rt.shape[0], -1)[:, :n]
            ref = rf[:, p0:p0 + pg, h].reshape(rf.shape[0], -1)[:, :n]
            unit = float(ref.abs().max())
            assert unit > 0
            err = float((got - ref).abs().max()) / unit
            assert err <= 2e-5, f"request {i} head {h}: raw error {err:.2e} of the head's scale {unit:.2e}"
            sd = float(vf[row, h].sqrt())
            assert abs(float(mt[row, h] - mf[row, h])) <= 2e-5 * (abs(float(mf[row, h])) + sd)
            assert abs(float(vt[row, h] - vf[row, h])) <= 4e-5 * float(vf[row, h])
