"""Calibration driver: host logic on CPU, the whole artefact on a GPU.

The GPU test runs the driver on tiny random-weight Qwen2 (q_proj capture) and
Qwen3 (q_norm capture) checkpoints and checks the artefact against the oracle's
restatement of the reference stats builder fed with the same query projections
(tolerance 1e-4 * max(|ref|, mean|q|), as for the calibration reduction).
"""

from __future__ import annotations

import types
from pathlib import Path

import pytest
import torch

from vllm_ascend_kvcompress import calibration as C
from vllm_ascend_kvcompress.model import model_shape_from_config


def _shape(**kw):
    return model_shape_from_config(types.SimpleNamespace(hf_text_config=types.SimpleNamespace(**kw)))


def test_model_shape_from_config_rules():
    s = _shape(num_attention_heads=40, num_key_value_heads=8, hidden_size=5120, num_hidden_layers=48,
               rope_theta=1e6, model_type="qwen2")
    assert (s.head_dim, s.num_layers, s.effective_rotary_dim, s.has_rope_scaling) == (128, 48, 128, False)
    assert s.full_attention_layer_indices == tuple(range(48))
    hybrid = _shape(num_attention_heads=16, num_key_value_heads=2, head_dim=256, num_hidden_layers=4,
                    layer_types=["linear_attention", "linear_attention", "linear_attention", "full_attention"],
                    rope_parameters={"rope_theta": 1e7, "partial_rotary_factor": 0.25, "rope_type": "default"})
    assert hybrid.full_attention_layer_indices == (3,) and hybrid.effective_rotary_dim == 64
    assert hybrid.rope_theta == 1e7 and hybrid.has_rope_scaling  # partial_rotary_factor is a RoPE parameter
    assert _shape(num_attention_heads=4, hidden_size=64, num_hidden_layers=1,
                  rope_scaling={"rope_type": "yarn", "factor": 4.0}).has_rope_scaling
    for bad in (dict(num_attention_heads=6, num_key_value_heads=4, hidden_size=96, num_hidden_layers=1),
                dict(num_attention_heads=4, hidden_size=64, num_hidden_layers=0),
                dict(num_attention_heads=4, hidden_size=64, num_hidden_layers=2, layer_types=["full_attention"]),
                dict(num_attention_heads=4, hidden_size=64, num_hidden_layers=1, rotary_dim=17)):
        with pytest.raises(ValueError):
            _shape(**bad)


def test_request_defaults_parser_and_builtin_text(tmp_path):
    r = C.request_from_args(["--model", "m", "--output", str(tmp_path / "o.pt"), "--max-length", "256"])
    assert r.device == "cuda" and r.dtype == "bfloat16" and r.max_length == 256 and not r.force
    text, source = C._load_calibration_text(r)
    assert source == C.BUILTIN_INPUT_SOURCE and len(text) >= 6 * 256
    f = tmp_path / "in.txt"
    f.write_text("  \n")
    with pytest.raises(ValueError, match="empty"):
        C._load_calibration_text(C.CalibrationRequest(model="m", output=tmp_path / "o.pt", input_path=f))
    f.write_text("hello calibration")
    assert C._load_calibration_text(C.CalibrationRequest(model="m", output=tmp_path / "o.pt", input_path=f))[0] \
        == "hello calibration"
    assert C._dtype_name("torch.bfloat16") == "bfloat16" and C._dtype_name("half") == "float16"
    assert C._rope_type(types.SimpleNamespace(rope_scaling={"type": "linear"})) == "linear"
    assert C._model_source_fingerprint("org/model", None).startswith("identifier:")
    with pytest.raises(ValueError, match="max_length"):
        C.generate_calibration_artifact(C.CalibrationRequest(model="m", output=tmp_path / "o.pt", max_length=64))


def test_driver_refuses_non_cuda_devices(tmp_path):
    with pytest.raises(RuntimeError, match="CUDA"):
        C.generate_calibration_artifact(C.CalibrationRequest(model="m", output=tmp_path / "o.pt", device="cpu"))


def test_local_checkpoint_fingerprint_tracks_files(tmp_path):
    from calib_models import make_checkpoint

    ckpt = make_checkpoint(tmp_path / "ckpt")
    a = C._model_source_fingerprint(str(ckpt), None)
    assert a.startswith("local-manifest:") and a == C._model_source_fingerprint(str(ckpt), "rev")
    (ckpt / "extra.bin").write_bytes(b"x")
    assert C._model_source_fingerprint(str(ckpt), None) != a


@pytest.mark.gpu
@pytest.mark.parametrize("model_type", ["qwen2", "qwen3"])
def test_driver_writes_a_valid_artefact_matching_the_oracle(model_type, tmp_path):
    from transformers import AutoModel

    from calib_models import make_checkpoint
    from oracle.triattention_oracle import CalibrationSums
    from vllm_ascend_kvcompress.methods.triattention.stats import CalibrationStats

    ckpt = make_checkpoint(tmp_path / "ckpt", model_type)
    out = tmp_path / "stats.pt"
    req = C.CalibrationRequest(model=str(ckpt), output=out, max_length=512, local_files_only=True)
    assert C.generate_calibration_artifact(req) is True
    assert C.generate_calibration_artifact(req) is False  # reused, validated
    stats = CalibrationStats.load(out)
    meta = stats.metadata
    assert meta["generator"] == C.GENERATOR and meta["schema_version"] == 3 and meta["model_type"] == model_type
    assert meta["input_source"] == C.BUILTIN_INPUT_SOURCE and 2 <= meta["token_count"] <= 512
    shape = C._model_shape_from_hf_config(AutoModel.from_pretrained(str(ckpt)).config)
    assert stats.validate(shape) == ()
    # the oracle on the same query projections
    model = AutoModel.from_pretrained(str(ckpt), dtype=torch.bfloat16, attn_implementation="eager").cuda().eval()
    sums = {}
    hooks = []
    for i, layer in enumerate(model.layers):
        target = getattr(layer.self_attn, "q_norm", None) or layer.self_attn.q_proj
        sums[i] = CalibrationSums()
        hooks.append(target.register_forward_hook(
            lambda _m, _i, o, s=sums[i]: s.add(o.detach().double().cpu(), shape.num_attention_heads,
                                              shape.head_dim, shape.effective_rotary_dim)))
    text, _ = C._load_calibration_text(req)
    from transformers import AutoTokenizer

    enc = AutoTokenizer.from_pretrained(str(ckpt))(text, return_tensors="pt", truncation=True, max_length=512)
    with torch.inference_mode():
        model(input_ids=enc["input_ids"].cuda(), use_cache=False)
    for h in hooks:
        h.remove()
    payload = torch.load(out, weights_only=True)
    for i, s in sums.items():
        ref = s.means()
        got = payload["layer_stats"][str(i)]
        scale = float(ref["q_abs_mean"].abs().mean())
        for key in ("q_mean_real", "q_mean_imag", "q_abs_mean"):
            r = ref[key].float()
            tol = 1e-4 * torch.maximum(r.abs(), torch.full_like(r, scale))
            assert ((got[key] - r).abs() <= tol).all(), (i, key)
        assert torch.allclose(got["inv_freq"], 1.0 / (1e6 ** (torch.arange(0, shape.effective_rotary_dim, 2).float()
                                                                / shape.effective_rotary_dim)), rtol=1e-6)
