"""Method-facing model geometry from a vLLM / Hugging Face config.

Same contract as the reference's ``model_shape_from_config``
(src/vllm_ascend_kvcompress/model.py:12-78): read the text config
(``hf_text_config``, else ``hf_config``), derive head counts, head dim, layer
count, RoPE theta, rotary dim (``rotary_dim``, ``rope_dim``,
``partial_rotary_factor``) and the full-attention layers of hybrid models
(``layer_types``), and reject inconsistent geometry with ``ValueError``.
"""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any

from .methods.base import ModelShape

_LAYER_KINDS = {"full_attention", "linear_attention"}


def model_shape_from_config(model_config: Any) -> ModelShape:
    cfg = getattr(model_config, "hf_text_config", None)
    if cfg is None:
        cfg = getattr(model_config, "hf_config", None)
    if cfg is None:
        raise ValueError("model has no Hugging Face text configuration")
    heads = int(cfg.num_attention_heads)
    kv_heads = int(getattr(cfg, "num_key_value_heads", heads))
    head_dim = getattr(cfg, "head_dim", None)
    head_dim = int(cfg.hidden_size) // heads if head_dim is None else int(head_dim)
    layers = int(getattr(cfg, "num_hidden_layers", getattr(cfg, "num_layers", 0)))
    if layers <= 0:
        raise ValueError("model text configuration has no positive layer count")
    if heads <= 0 or kv_heads <= 0:
        raise ValueError("model attention head counts must be positive")
    if heads % kv_heads:
        raise ValueError("model query heads are not divisible by KV heads")
    if head_dim <= 0 or head_dim % 2:
        raise ValueError("model attention head dimension must be positive and even")
    params = getattr(cfg, "rope_parameters", None)
    scaling = getattr(cfg, "rope_scaling", None)
    theta = getattr(cfg, "rope_theta", None)
    if theta is None and isinstance(params, Mapping):
        theta = params.get("rope_theta")
    theta = 10000.0 if theta is None else float(theta)
    kinds = getattr(cfg, "layer_types", None)
    if kinds is None:
        attention = tuple(range(layers))
    else:
        if len(kinds) != layers:
            raise ValueError("model layer_types length does not match layer count")
        unknown = sorted(set(kinds) - _LAYER_KINDS)
        if unknown:
            raise ValueError("unsupported model layer types: " + ", ".join(unknown))
        attention = tuple(i for i, kind in enumerate(kinds) if kind == "full_attention")
        if not attention:
            raise ValueError("model exposes no full-attention layers")
    return ModelShape(
        model_type=str(getattr(cfg, "model_type", "")),
        num_layers=layers,
        num_attention_heads=heads,
        num_kv_heads=kv_heads,
        head_dim=head_dim,
        rope_theta=theta,
        has_rope_scaling=_scaled(scaling) or _scaled(params),
        rotary_dim=_rotary_dim(cfg, head_dim, params),
        attention_layer_indices=attention,
    )


def _rotary_dim(cfg: Any, head_dim: int, params: Any) -> int:
    value = getattr(cfg, "rotary_dim", None)
    if value is None and isinstance(params, Mapping):
        value = params.get("rope_dim")
    if value is None:
        factor = getattr(cfg, "partial_rotary_factor", None)
        if factor is None and isinstance(params, Mapping):
            factor = params.get("partial_rotary_factor")
        value = head_dim if factor is None else int(head_dim * float(factor))
    value = int(value)
    if value <= 0 or value > head_dim or value % 2:
        raise ValueError("model rotary dimension must be positive, even, and no larger than the attention "
                         "head dimension")
    return value


def _scaled(params: Any) -> bool:
    """True when RoPE parameters describe anything but plain default RoPE."""
    if not params:
        return False
    if not isinstance(params, Mapping):
        return True
    kind = params.get("rope_type", params.get("type", "default")) or "default"
    return str(kind) != "default" or bool(set(params) - {"rope_theta", "rope_type", "type"})
