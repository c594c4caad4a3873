"""Opt-in online calibration through the method API's query-observation hooks.

The provider hands ``capture_query`` the post-RoPE attention queries of prefill
forwards; the method keeps each request's newest ``online_calibration_window``
rows per scoring layer, and ``complete_query_observation`` reduces them with
the calibration kernel, which undoes RoPE in fp32 at the rows' positions
(ending at ``semantic_num_tokens``) before summing.  Past ``online_calibration_min_tokens`` rows a layer's
online means replace the artefact's in the scoring tensors.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

import kvc_workloads as W
from vllm_ascend_kvcompress.methods.base import LayerCache, ModelShape, QueryBatchSpan, QueryObservation
from vllm_ascend_kvcompress.methods.triattention.config import TriAttentionConfig
from vllm_ascend_kvcompress.methods.triattention.method import TriAttentionMethod


def _options(**extra):
    return {"stats_path": "/tmp/x.pt", "kv_budget": 2048, **extra}


def test_online_options_default_off_and_validate():
    cfg = TriAttentionConfig.from_method_config(_options())
    assert cfg.online_calibration_window == 0 and cfg.online_calibration_min_tokens == 16384
    cfg = TriAttentionConfig.from_method_config(_options(online_calibration_window=512,
                                                         online_calibration_min_tokens=4096))
    assert (cfg.online_calibration_window, cfg.online_calibration_min_tokens) == (512, 4096)
    for bad in ({"online_calibration_window": -1}, {"online_calibration_min_tokens": 0},
                {"online_calibration_window": 1.5}):
        with pytest.raises(ValueError):
            TriAttentionConfig.from_method_config(_options(**bad))


def test_unbound_method_declares_the_scoring_layers(tmp_path):
    w = W.config4(num_seqs=2, stride=8)
    path = W.write_stats_file(w, str(tmp_path))
    g = w.geometry
    shape = ModelShape(model_type=g.model_type, num_layers=g.num_layers, num_attention_heads=g.num_q_heads,
                       num_kv_heads=g.num_kv_heads, head_dim=g.head_dim, rope_theta=g.rope_theta,
                       has_rope_scaling=False)
    vcfg = SimpleNamespace(parallel_config=SimpleNamespace(tensor_parallel_size=1),
                           model_config=SimpleNamespace(max_model_len=65536), speculative_config=None)
    off = TriAttentionMethod(w.options.method_config(path), vcfg, shape)
    assert off.query_window_tokens == 0 and off.query_layer_indices is None
    on = TriAttentionMethod({**w.options.method_config(path), "online_calibration_window": 256}, vcfg, shape)
    assert on.query_window_tokens == 256
    assert on.query_layer_indices == tuple(range(0, g.num_layers, 8))


def _rotate(q_pre: torch.Tensor, heads: int, D: int, rot: int, first: int, omega: torch.Tensor) -> torch.Tensor:
    """Half-style RoPE at positions first.. in fp32, result in q_pre's dtype."""
    F = rot // 2
    x = q_pre.float().view(q_pre.shape[0], heads, D)
    pos = torch.arange(first, first + q_pre.shape[0], device=q_pre.device, dtype=torch.float32)
    th = pos[:, None] * omega[None, :]
    c, s = torch.cos(th)[:, None, :], torch.sin(th)[:, None, :]
    x1, x2 = x[..., :F], x[..., F:rot]
    out = x.clone()
    out[..., :F] = x1 * c - x2 * s
    out[..., F:rot] = x2 * c + x1 * s
    return out.reshape(q_pre.shape).to(q_pre.dtype)


def _unrotate_f64(q_post: torch.Tensor, heads: int, D: int, rot: int, first: int, omega: torch.Tensor):
    """fp64 inverse rotation of captured 16-bit rows; angles formed as fp32(position) * omega in fp32."""
    F = rot // 2
    x = q_post.double().view(q_post.shape[0], heads, D).clone()
    pos = torch.arange(first, first + q_post.shape[0], dtype=torch.float32, device=q_post.device)
    th = (pos[:, None] * omega[None, :].float()).double()  # IEEE fp32 product, as the kernel forms it
    c, s = torch.cos(th)[:, None, :], torch.sin(th)[:, None, :]
    o1, o2 = x[..., :F].clone(), x[..., F:rot].clone()
    x[..., :F] = o1 * c + o2 * s
    x[..., F:rot] = o2 * c - o1 * s
    return x.reshape(q_post.shape[0], heads * D)


@pytest.mark.gpu
def test_unrotate_inverts_rope_within_bf16_rounding():
    from vllm_ascend_kvcompress.methods.triattention import kernels as K

    heads, D, rot = 8, 128, 64
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(300, heads * D, generator=g, device="cuda").to(torch.bfloat16)
    omega = 1.0 / (1e6 ** (torch.arange(0, rot, 2, device="cuda").float() / rot))
    post = _rotate(q, heads, D, rot, 40000, omega)
    K.unrotate_queries(post, heads, D, rot, 40000, omega)
    err = (post.float() - q.float()).abs()
    assert float(err.max()) <= 2 ** -6 * float(q.float().abs().max())
    assert torch.equal(post.view(-1, D)[:, rot:], q.view(-1, D)[:, rot:])  # unrotated dims untouched


@pytest.mark.gpu
def test_capture_complete_and_publish(tmp_path):
    from oracle.triattention_oracle import CalibrationSums

    w = W.config0()
    caches = [tuple(t.cuda() for t in W.kv_pages(w, layer)) for layer in range(w.geometry.num_layers)]
    m = W.b200_method(w, caches, W.write_stats_file(w, str(tmp_path)))
    base = {k: v for k, v in m.config.__dict__.items()}
    m.config = TriAttentionConfig(**{**base, "online_calibration_window": 256, "online_calibration_min_tokens": 500})
    assert m.query_window_tokens == 256 and m.query_layer_indices == (0,)
    heads, D, rot = m.local_kv_heads * m.group, m.head_dim, m.rotary_dim
    layer = LayerCache(name=W.layer_name(0), layer_index=0, k_cache=caches[0][0], v_cache=caches[0][1])
    omega = m.scoring_omega[0]
    g = torch.Generator(device="cuda").manual_seed(11)
    ref = CalibrationSums()     # fp64 un-rotation of the captured rows: the 1e-4 bound
    truth = CalibrationSums()   # the pre-RoPE rows themselves (differ by the capture's bf16 rounding)
    for req, S in (("a", 5000), ("b", 3000)):
        q_pre = (torch.randn(300, heads * D, generator=g, device="cuda") + 0.3).to(torch.bfloat16)
        q_post = _rotate(q_pre, heads, D, rot, S - 300, omega)
        # two forwards of the final prefill, inside batches with another request's rows
        pad = torch.zeros(7, heads * D, device="cuda", dtype=torch.bfloat16)
        m.capture_query(layer, torch.cat([pad, q_post[:100]]), (QueryBatchSpan(req, 7, 107),))
        m.capture_query(layer, torch.cat([q_post[100:], pad]).view(-1, heads, D), (QueryBatchSpan(req, 0, 200),))
        m.capture_query(layer, q_post, (QueryBatchSpan("dropped", 0, 300),))
        m.complete_query_observation(QueryObservation(req, None, S, 256, (0,)))
        ref.add(_unrotate_f64(q_post[-256:], heads, D, rot, S - 256, omega).cpu(), heads, D, rot)  # newest 256
        truth.add(q_pre[-256:].double().cpu(), heads, D, rot)
    m.discard_query_observation("dropped")
    acc = m._online_sums[0]
    assert acc.count == 512 and m.online_published[0] == 512
    scale = float((ref.abs_sum / ref.count).abs().mean())
    for got, want, true in ((acc.real_sum, ref.real_sum, truth.real_sum), (acc.imag_sum, ref.imag_sum, truth.imag_sum),
                            (acc.abs_sum, ref.abs_sum, truth.abs_sum)):
        g_mean, w_mean = got.cpu() / 512, want / 512
        # calibration tolerance: |d| <= 1e-4 * max(|ref|, mean |q|)
        assert float((g_mean - w_mean).abs().max()) <= 1e-4 * max(scale, float(w_mean.abs().max()))
        # and the capture's own bf16 rounding keeps it near the pre-RoPE truth
        assert float((g_mean - true / 512).abs().max()) <= 2e-3 * max(scale, float(w_mean.abs().max()))
    kvh, G, F = m.local_kv_heads, m.group, m.num_freq
    torch.testing.assert_close(m.scoring_q_real[0], (acc.real_sum / 512).float().view(kvh, G, F))
    torch.testing.assert_close(m.scoring_q_imag[0], (acc.imag_sum / 512).float().view(kvh, G, F))
    assert len(m._free_buffers) == 2 and not m._observations  # both requests' buffers and the dropped one's
    keep = m.select_many(W.b200_requests(w))  # scoring runs with the published statistics
    m.check_device_errors()
    assert keep.shape == (len(w.compressed()), w.options.kv_budget)
