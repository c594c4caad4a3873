"""Host-side contracts kept from the reference: method config, registry, stats."""

from __future__ import annotations

from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

import kvc_workloads as W
from vllm_ascend_kvcompress import available_methods, register_method
from vllm_ascend_kvcompress.methods import METHOD_API_VERSION, create_method
from vllm_ascend_kvcompress.methods.base import KVCompressionMethod, ModelShape
from vllm_ascend_kvcompress.methods.registry import MethodRegistry
from vllm_ascend_kvcompress.methods.triattention.config import TriAttentionConfig
from vllm_ascend_kvcompress.methods.triattention.method import TriAttentionMethod, _queries_per_kv_head
from vllm_ascend_kvcompress.methods.triattention.scoring import build_geometric_offsets
from vllm_ascend_kvcompress.methods.triattention.stats import CalibrationStats
from vllm_ascend_kvcompress.plugin import register


def _shape(geo: W.Geometry) -> ModelShape:
    return ModelShape(geo.model_type, geo.num_layers, geo.num_q_heads, geo.num_kv_heads, geo.head_dim,
                      geo.rope_theta, False, None if geo.rotary_dim == geo.head_dim else geo.rotary_dim)


def test_api_version_and_builtin_method():
    assert METHOD_API_VERSION == 1
    assert "triattention" in available_methods()
    register()
    register()  # idempotent


@pytest.mark.parametrize("bad,msg", [
    ({"kv_budget": 100}, "positive multiple of 128"),
    ({"kv_budget": 256, "protected_prefix_window": 200, "protected_recent_window": 100}, "cannot exceed"),
    ({"position_policy": "v4"}, "must be one of"),
    ({"score_layer_stride": 0}, "positive"),
    ({"unknown_option": 1}, "unknown TriAttention method options"),
    ({"kv_budget": True}, "must be an integer"),
    ({"auto_calibrate": "yes"}, "must be a boolean"),
])
def test_config_rejects_like_reference(bad, msg):
    opts = {"stats_path": "/x.pt", **bad}
    with pytest.raises(ValueError, match=msg):
        TriAttentionConfig.from_method_config(opts)


def test_config_defaults_and_threshold():
    c = TriAttentionConfig.from_method_config({"stats_path": "/x.pt", "kv_budget": 4608, "recompute_window": 128})
    assert c.compression_threshold_tokens == 4736
    assert c.position_policy == "global" and c.protected_recent_window == 128 and c.score_layer_stride == 8


def test_registry_fail_closed():
    reg = MethodRegistry()
    with pytest.raises(ValueError):
        reg.register("bad name!", lambda *a: None)
    reg.register("Demo", lambda o, v, s: None)
    with pytest.raises(ValueError, match="already registered"):
        reg.register("demo", lambda *a: None)
    with pytest.raises(TypeError, match="expected KVCompressionMethod"):
        reg.create("demo", {}, None, None)
    with pytest.raises(ValueError, match="unknown compression method"):
        reg.create("nope", {}, None, None)


def test_geometric_offsets_match_reference_count():
    assert build_geometric_offsets(65536, "cpu").numel() == 17
    assert build_geometric_offsets(1, "cpu").tolist() == [1.0]
    with pytest.raises(ValueError):
        build_geometric_offsets(0, "cpu")


def test_gqa_width_invariant_under_tp():
    shape = ModelShape("qwen3_5_moe_text", 40, 16, 2, 256, 1e7, False, 64, tuple(range(3, 40, 4)))
    assert _queries_per_kv_head(shape) == 8


def test_stats_roundtrip_validate_and_tp_shard(tmp_path: Path):
    w = W.config2()
    path = tmp_path / "s.pt"
    torch.save(W.calibration_payload(w.geometry, w.seed), path)
    stats = CalibrationStats.load(path)
    shape = _shape(w.geometry)
    assert stats.validate(shape) == ()
    full = stats.to_device(shape, torch.device("cpu"))
    r1 = stats.to_device(shape, torch.device("cpu"), tensor_parallel_rank=1, tensor_parallel_size=2)
    assert full[0].q_mean_real.shape == (2, 8, 32)
    assert r1[0].q_mean_real.shape == (1, 8, 32)
    assert torch.equal(r1[0].q_mean_real[0], full[0].q_mean_real[1])
    assert r1[0].q_pass_mean.shape == (1, 8, 192)
    with pytest.raises(ValueError, match="divisible"):
        stats.to_device(shape, torch.device("cpu"), tensor_parallel_rank=0, tensor_parallel_size=4)


def test_stats_validation_reasons(tmp_path: Path):
    w = W.config0()
    payload = W.calibration_payload(w.geometry, w.seed)
    payload["metadata"]["head_dim"] = 64
    payload["layer_stats"]["0"]["q_abs_mean"] = -payload["layer_stats"]["0"]["q_abs_mean"]
    path = tmp_path / "s.pt"
    torch.save(payload, path)
    reasons = CalibrationStats.load(path).validate(_shape(w.geometry))
    assert any("head_dim" in r for r in reasons)
    assert any("negative" in r for r in reasons)


def test_flat_stats_schema(tmp_path: Path):
    stats = {f"layer00_head{h:02d}": {"q_mean_real": torch.ones(4), "q_mean_imag": torch.zeros(4),
                                       "q_abs_mean": torch.ones(4)} for h in range(2)}
    path = tmp_path / "flat.pt"
    torch.save({"metadata": {}, "stats": stats}, path)
    loaded = CalibrationStats.load(path)
    assert loaded.layers[0].q_mean_real.shape == (2, 4)
    stats.pop("layer00_head00")
    stats["layer00_head02"] = stats["layer00_head01"]
    torch.save({"metadata": {}, "stats": stats}, path)
    with pytest.raises(ValueError, match="contiguous"):
        CalibrationStats.load(path)


def test_method_requires_cuda_caches(tmp_path: Path):
    w = W.config0()
    stats_path = W.write_stats_file(w, tmp_path)
    vcfg = SimpleNamespace(parallel_config=SimpleNamespace(tensor_parallel_size=1),
                           model_config=SimpleNamespace(max_model_len=65536), speculative_config=None)
    m = create_method("triattention", w.options.method_config(stats_path), vcfg, _shape(w.geometry))
    assert isinstance(m, TriAttentionMethod) and isinstance(m, KVCompressionMethod)
    assert m.runtime_spec.compression_threshold_tokens == 2048 + 128
    assert m.compatibility_reasons(None) == ()
    with pytest.raises(RuntimeError, match="CUDA"):
        m.bind_model_runner(SimpleNamespace(device=torch.device("cpu")), ())
    with pytest.raises(RuntimeError, match="not bound"):
        m.compress_many([SimpleNamespace(physical_num_tokens=3000, semantic_num_tokens=3000,
                                         source_block_ids_device=None, destination_block_ids_device=None)])


def test_external_method_registration():
    class Dummy(KVCompressionMethod):
        name = "dummy-ext"
        runtime_spec = None

        def compatibility_reasons(self, worker):
            return ()

        def bind_model_runner(self, runner, layer_caches):
            pass

        def compress(self, request):
            return None

    register_method("dummy-ext", lambda o, v, s: Dummy())
    assert isinstance(create_method("dummy-ext", {}, None, None), Dummy)


def test_workspaces_grow_only_and_keep_addresses_until_growth():
    import torch

    from vllm_ascend_kvcompress.methods.triattention.method import _Workspaces

    ws = _Workspaces(torch.device("cpu"))
    p1 = ws.ptr("raw", 100, torch.float32)
    assert ws.ptr("raw", 80, torch.float32) == p1  # smaller requests reuse the buffer
    assert ws.get("raw", 50, torch.float32).data_ptr() == p1 and ws.get("raw", 50, torch.float32).numel() == 50
    p2 = ws.ptr("raw", 1000, torch.float32)  # growth reallocates (callers re-read addresses every step)
    assert ws.get("raw", 1000, torch.float32).data_ptr() == p2
    assert ws.ptr("raw", 1010, torch.float32) == p2  # the request plus a little slack fits
    p3 = ws.ptr("raw", 1100, torch.float32)
    assert ws.ptr("raw", int(1016 * 1.25) + 16, torch.float32) == p3  # growth: 1.25x the old buffer (+16)
    assert ws.ptr("keep", 4, torch.int64) != p2
    assert ws.get("keep", 4, torch.int64).dtype == torch.int64
