"""TriAttention calibration statistics: loading, validation, device layout, TP shard.

The on-disk contract is the reference plugin's
(src/vllm_ascend_kvcompress/methods/triattention/stats.py:17-482): a
``torch.save``d mapping with ``metadata`` and either a flat ``stats`` mapping
keyed ``layerNN_headMM`` or a schema-3 ``layer_stats`` mapping keyed by layer
index.  Rows are per query head (or per KV head, expanded to the group).  On the
device the statistics are grouped ``[kv_heads, queries_per_kv, width]`` and a
tensor-parallel rank keeps only its contiguous slice of KV heads.
"""

from __future__ import annotations

import math
import re
from collections.abc import Mapping
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch

from ..base import ModelShape

SUPPORTED_MODEL_TYPES = frozenset({
    "llama", "mistral", "qwen2", "qwen2_moe", "qwen3", "qwen3_moe", "qwen3_5_text", "qwen3_5_moe_text",
})
_FLAT_KEY = re.compile(r"^layer(?P<layer>\d+)_head(?P<head>\d+)$")


@dataclass(frozen=True)
class LayerCalibrationStats:
    q_mean_real: torch.Tensor
    q_mean_imag: torch.Tensor
    q_abs_mean: torch.Tensor
    freq_scale_sq: torch.Tensor | None = None
    inv_freq: torch.Tensor | None = None
    q_pass_mean: torch.Tensor | None = None


@dataclass(frozen=True)
class DeviceLayerCalibrationStats:
    q_mean_real: torch.Tensor
    q_mean_imag: torch.Tensor
    q_abs_mean: torch.Tensor
    freq_scale_sq: torch.Tensor
    omega: torch.Tensor
    rope_style: str
    rotary_dim: int | None = None
    q_pass_mean: torch.Tensor | None = None


def _matrix(value: Any, name: str) -> torch.Tensor:
    if not isinstance(value, torch.Tensor):
        raise ValueError(f"calibration field {name!r} must be a tensor")
    t = value.detach().to(device="cpu", dtype=torch.float32)
    if t.ndim == 1:
        t = t.unsqueeze(0)
    if t.ndim != 2:
        raise ValueError(f"calibration field {name!r} must be rank two")
    return t.contiguous()


def _vector(value: Any) -> torch.Tensor | None:
    if isinstance(value, torch.Tensor):
        return value.detach().to(device="cpu", dtype=torch.float32).flatten()
    if isinstance(value, (list, tuple)):
        return torch.tensor(value, dtype=torch.float32).flatten()
    return None


def _parse_flat(raw: Mapping[str, Any]) -> dict[int, LayerCalibrationStats]:
    by_layer: dict[int, dict[int, Mapping[str, Any]]] = {}
    for key, entry in raw.items():
        m = _FLAT_KEY.match(str(key))
        if m is None:
            continue
        if not isinstance(entry, Mapping):
            raise ValueError(f"calibration entry {key!r} must be a mapping")
        by_layer.setdefault(int(m["layer"]), {})[int(m["head"])] = entry
    if not by_layer:
        raise ValueError("flat calibration statistics contain no layer/head entries")
    out = {}
    for layer, heads in by_layer.items():
        order = list(range(max(heads) + 1))
        if sorted(heads) != order:
            raise ValueError(f"layer {layer} calibration heads must be complete and contiguous; got {sorted(heads)}")
        rows = {f: torch.stack([_matrix(heads[h][f], f)[0] for h in order])
                for f in ("q_mean_real", "q_mean_imag", "q_abs_mean")}
        out[layer] = LayerCalibrationStats(rows["q_mean_real"], rows["q_mean_imag"], rows["q_abs_mean"])
    return out


def _parse_layered(raw: Mapping[Any, Any]) -> dict[int, LayerCalibrationStats]:
    out = {}
    for key, entry in raw.items():
        if not isinstance(entry, Mapping):
            raise ValueError(f"layer statistics {key!r} must be a mapping")
        q = entry.get("q_mean_complex")
        if isinstance(q, torch.Tensor) and q.is_complex():
            real, imag = _matrix(q.real, "q_mean_complex.real"), _matrix(q.imag, "q_mean_complex.imag")
        elif isinstance(q, torch.Tensor) and q.ndim == 3:
            if q.shape[-1] != 2:
                raise ValueError("q_mean_complex final dimension must equal two")
            real, imag = _matrix(q[..., 0], "q_mean_complex.real"), _matrix(q[..., 1], "q_mean_complex.imag")
        else:
            real, imag = _matrix(entry.get("q_mean_real"), "q_mean_real"), _matrix(entry.get("q_mean_imag"), "q_mean_imag")
        fs, pm = entry.get("freq_scale_sq"), entry.get("q_pass_mean")
        out[int(key)] = LayerCalibrationStats(
            q_mean_real=real,
            q_mean_imag=imag,
            q_abs_mean=_matrix(entry.get("q_abs_mean"), "q_abs_mean"),
            freq_scale_sq=None if fs is None else _matrix(fs, "freq_scale_sq"),
            inv_freq=_vector(entry.get("inv_freq")) if isinstance(entry.get("inv_freq"), torch.Tensor) else None,
            q_pass_mean=None if pm is None else _matrix(pm, "q_pass_mean"),
        )
    return out


def _metadata_inv_freq(meta: Mapping[str, Any], layer: int) -> torch.Tensor | None:
    per_layer = meta.get("layer_inv_freqs")
    value = None
    if isinstance(per_layer, Mapping):
        value = per_layer.get(layer, per_layer.get(str(layer)))
    elif isinstance(per_layer, (list, tuple)) and layer < len(per_layer):
        value = per_layer[layer]
    if value is None:
        value = meta.get("inv_freq")
    return _vector(value)


def _grouped(t: torch.Tensor, model: ModelShape, group: int, width: int) -> torch.Tensor:
    """Rows per query head ``[q_heads, w]`` or per KV head ``[kv_heads, w]`` -> ``[kv, group, w]``."""
    shape = tuple(t.shape)
    if shape == (model.num_attention_heads, width):
        return t.reshape(model.num_kv_heads, group, width).contiguous()
    if shape == (model.num_kv_heads, width):
        return t.unsqueeze(1).expand(model.num_kv_heads, group, width).contiguous()
    raise ValueError(f"calibration tensor shape {shape} cannot be grouped for "
                     f"{model.num_attention_heads} query heads and {model.num_kv_heads} KV heads")


@dataclass(frozen=True)
class CalibrationStats:
    metadata: Mapping[str, Any]
    layers: Mapping[int, LayerCalibrationStats]

    @classmethod
    def load(cls, path: Path) -> "CalibrationStats":
        path = Path(path)
        if not path.is_file():
            raise ValueError(f"calibration statistics file does not exist: {path}")
        try:
            payload = torch.load(path, map_location="cpu", weights_only=True)
        except TypeError as err:
            raise ValueError("calibration loading requires torch.load(weights_only=True) support") from err
        return cls.from_payload(payload)

    @classmethod
    def from_payload(cls, payload: Any) -> "CalibrationStats":
        if not isinstance(payload, Mapping):
            raise ValueError("calibration statistics payload must be a mapping")
        meta = payload.get("metadata", {})
        if not isinstance(meta, Mapping):
            raise ValueError("calibration metadata must be a mapping")
        flat = payload.get("stats")
        if isinstance(flat, Mapping) and flat:
            layers = _parse_flat(flat)
        else:
            layered = payload.get("layer_stats")
            if not isinstance(layered, Mapping) or not layered:
                raise ValueError("calibration payload must contain non-empty 'stats' or 'layer_stats'")
            layers = _parse_layered(layered)
        return cls(metadata=dict(meta), layers=layers)

    def validate(self, model: ModelShape) -> tuple[str, ...]:
        """Every incompatibility with ``model`` (empty tuple = usable)."""
        why: list[str] = []
        meta = self.metadata
        if model.model_type not in SUPPORTED_MODEL_TYPES:
            why.append(f"model_type {model.model_type!r} has no verified RoPE layout")
        expected = set(model.full_attention_layer_indices)
        if set(self.layers) != expected:
            why.append(f"calibration layer set does not match the model: expected {sorted(expected)}, "
                       f"got {sorted(self.layers)}")
        style = str(meta.get("rope_style", "half"))
        if style != "half":
            why.append(f"calibration rope_style {style!r} is unsupported; expected 'half'")
        scalar_checks = (
            ("head_dim", model.head_dim, int),
            ("rotary_dim", model.effective_rotary_dim, int),
            ("num_layers", model.num_layers, int),
            ("num_attention_heads", model.num_attention_heads, int),
        )
        for key, want, conv in scalar_checks:
            got = meta.get(key)
            if got is not None and conv(got) != want:
                why.append(f"calibration {key} {got} does not match model value {want}")
        kv = meta.get("num_kv_heads", meta.get("num_key_value_heads"))
        if kv is not None and int(kv) != model.num_kv_heads:
            why.append(f"calibration num_kv_heads {kv} does not match model value {model.num_kv_heads}")
        layers_meta = meta.get("attention_layer_indices")
        if layers_meta is not None and tuple(int(v) for v in layers_meta) != model.full_attention_layer_indices:
            why.append("calibration attention_layer_indices do not match the model")
        mt = meta.get("model_type")
        if mt is not None and str(mt) != model.model_type:
            why.append(f"calibration model_type {mt!r} does not match model_type {model.model_type!r}")
        theta = meta.get("rope_theta")
        if theta is not None and not math.isclose(float(theta), model.rope_theta, rel_tol=1e-7, abs_tol=0.0):
            why.append(f"calibration rope_theta {theta} does not match model rope_theta {model.rope_theta}")
        rope_type = meta.get("rope_type", "default") or "default"
        f = model.effective_rotary_dim // 2
        p = model.head_dim - model.effective_rotary_dim
        q_shape, kv_shape = (model.num_attention_heads, f), (model.num_kv_heads, f)
        for idx, layer in self.layers.items():
            for name in ("q_mean_real", "q_mean_imag", "q_abs_mean"):
                t = getattr(layer, name)
                if tuple(t.shape) not in {q_shape, kv_shape}:
                    why.append(f"layer {idx} {name} has shape {tuple(t.shape)}; expected {q_shape} or {kv_shape}")
                if not bool(torch.isfinite(t).all()):
                    why.append(f"layer {idx} {name} contains non-finite values")
            if bool((layer.q_abs_mean < 0).any()):
                why.append(f"layer {idx} q_abs_mean contains negative values")
            if p:
                pm = layer.q_pass_mean
                if pm is None:
                    why.append(f"layer {idx} partial RoPE requires q_pass_mean")
                elif tuple(pm.shape) not in {(model.num_attention_heads, p), (model.num_kv_heads, p)}:
                    why.append(f"layer {idx} q_pass_mean has shape {tuple(pm.shape)}")
                elif not bool(torch.isfinite(pm).all()):
                    why.append(f"layer {idx} q_pass_mean contains non-finite values")
            fs = layer.freq_scale_sq
            if fs is not None:
                if tuple(fs.shape) not in {(1, f), q_shape, kv_shape}:
                    why.append(f"layer {idx} freq_scale_sq has incompatible shape {tuple(fs.shape)}")
                if not bool(torch.isfinite(fs).all()):
                    why.append(f"layer {idx} freq_scale_sq contains non-finite values")
                if bool((fs <= 0).any()):
                    why.append(f"layer {idx} freq_scale_sq must be positive")
            elif model.has_rope_scaling:
                why.append(f"layer {idx} scaled RoPE requires freq_scale_sq calibration values")
            inv = layer.inv_freq if layer.inv_freq is not None else _metadata_inv_freq(meta, idx)
            if inv is None and (model.has_rope_scaling or rope_type != "default"):
                why.append(f"layer {idx} scaled or non-default RoPE requires exact inv_freq calibration values")
            if inv is not None:
                if inv.numel() != f:
                    why.append(f"layer {idx} inv_freq has {inv.numel()} values; expected {f}")
                if not bool(torch.isfinite(inv).all()):
                    why.append(f"layer {idx} inv_freq contains non-finite values")
                if bool((inv <= 0).any()):
                    why.append(f"layer {idx} inv_freq must be positive")
        return tuple(why)

    def to_device(self, model: ModelShape, device: torch.device, *, tensor_parallel_rank: int = 0,
                  tensor_parallel_size: int = 1) -> dict[int, DeviceLayerCalibrationStats]:
        """Grouped fp32 statistics of this rank's KV heads, per layer, on ``device``."""
        if tensor_parallel_size <= 0 or not 0 <= tensor_parallel_rank < tensor_parallel_size:
            raise ValueError("invalid tensor-parallel rank or size")
        if model.num_kv_heads % tensor_parallel_size:
            raise ValueError("TriAttention tensor parallelism requires KV heads divisible by tensor-parallel size")
        group = model.num_attention_heads // model.num_kv_heads
        rot = model.effective_rotary_dim
        f = rot // 2
        local = model.num_kv_heads // tensor_parallel_size
        lo, hi = tensor_parallel_rank * local, (tensor_parallel_rank + 1) * local
        style = str(self.metadata.get("rope_style", "half"))

        def grouped(t: torch.Tensor, width: int) -> torch.Tensor:
            return _grouped(t.to(device=device, dtype=torch.float32), model, group, width)[lo:hi].contiguous()

        out = {}
        for idx, layer in self.layers.items():
            fs = layer.freq_scale_sq
            if fs is None:
                fs = torch.ones(model.num_attention_heads, f, dtype=torch.float32)
            elif fs.shape[0] == 1:
                fs = fs.expand(model.num_attention_heads, -1)
            inv = layer.inv_freq if layer.inv_freq is not None else _metadata_inv_freq(self.metadata, idx)
            if inv is None:
                inv = 1.0 / (model.rope_theta ** (torch.arange(0, rot, 2, dtype=torch.float32) / float(rot)))
            out[idx] = DeviceLayerCalibrationStats(
                q_mean_real=grouped(layer.q_mean_real, f),
                q_mean_imag=grouped(layer.q_mean_imag, f),
                q_abs_mean=grouped(layer.q_abs_mean, f),
                freq_scale_sq=grouped(fs, f),
                omega=inv.to(device=device, dtype=torch.float32).contiguous(),
                rope_style=style,
                rotary_dim=rot,
                q_pass_mean=None if layer.q_pass_mean is None else grouped(layer.q_pass_mean, model.head_dim - rot),
            )
        return out
