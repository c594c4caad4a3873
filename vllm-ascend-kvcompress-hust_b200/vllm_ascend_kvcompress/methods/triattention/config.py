"""Options of the TriAttention method and their validation.

Option names, defaults and error conditions follow the reference
(src/vllm_ascend_kvcompress/methods/triattention/config.py:18-198), so a method
configuration accepted there is accepted here with the same meaning.
``score_chunk_size`` only bounded the reference's CPU temporaries; the CUDA
path streams whole pages and validates but does not need it.

Two options exist only here and are off by default: ``online_calibration_window``
(trailing prefill query rows captured per request and scoring layer through the
method API's query-observation hooks, 0 = off) and
``online_calibration_min_tokens`` (rows a layer must have accumulated before its
online statistics replace the artefact's for scoring).
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass
from pathlib import Path
from typing import Literal, cast

from ...config import ASCEND_BLOCK_SIZE, JsonScalar, require_choice, require_int

ScoreAggregation = Literal["mean", "max"]
LayerAggregation = Literal["mean", "max"]
PositionPolicy = Literal["global", "v3"]

_KNOWN = frozenset({
    "stats_path", "auto_calibrate", "calibration_input_path", "calibration_max_length",
    "calibration_device", "calibration_attn_implementation", "calibration_local_files_only",
    "kv_budget", "recompute_window", "position_policy", "protected_prefix_window",
    "protected_recent_window", "position_segments", "score_aggregation", "layer_aggregation",
    "score_chunk_size", "score_layer_stride", "min_output_tokens_for_compression",
    "online_calibration_window", "online_calibration_min_tokens",
})


def _bool_option(options: Mapping[str, JsonScalar], name: str, default: bool) -> bool:
    value = options.get(name, default)
    if not isinstance(value, bool):
        raise ValueError(f"method option {name!r} must be a boolean")
    return value


def _nonempty_str(options: Mapping[str, JsonScalar], name: str, default: str | None) -> str | None:
    value = options.get(name, default)
    if value is None:
        return None
    if not isinstance(value, str) or not value.strip():
        raise ValueError(f"method option {name!r} must be a non-empty string")
    return value


@dataclass(frozen=True)
class TriAttentionConfig:
    """Validated TriAttention options."""

    stats_path: Path
    auto_calibrate: bool = True
    calibration_input_path: Path | None = None
    calibration_max_length: int = 4096
    calibration_device: str = "auto"
    calibration_attn_implementation: str = "eager"
    calibration_local_files_only: bool = False
    kv_budget: int = 2048
    recompute_window: int = ASCEND_BLOCK_SIZE
    position_policy: PositionPolicy = "global"
    protected_prefix_window: int = 0
    protected_recent_window: int = ASCEND_BLOCK_SIZE
    position_segments: int = 8
    score_aggregation: ScoreAggregation = "mean"
    layer_aggregation: LayerAggregation = "mean"
    score_chunk_size: int = 512
    score_layer_stride: int = 8
    min_output_tokens_for_compression: int = 0
    online_calibration_window: int = 0
    online_calibration_min_tokens: int = 16384

    @property
    def compression_threshold_tokens(self) -> int:
        return self.kv_budget + self.recompute_window

    @classmethod
    def from_method_config(cls, options: Mapping[str, JsonScalar]) -> "TriAttentionConfig":
        unknown = sorted(set(options) - _KNOWN)
        if unknown:
            raise ValueError("unknown TriAttention method options: " + ", ".join(unknown))
        stats = _nonempty_str(options, "stats_path", None)
        if stats is None:
            raise ValueError("method option 'stats_path' must be a non-empty string")
        calib_input = _nonempty_str(options, "calibration_input_path", None)
        device = _nonempty_str(options, "calibration_device", "auto")
        cfg = cls(
            stats_path=Path(stats).expanduser(),
            auto_calibrate=_bool_option(options, "auto_calibrate", True),
            calibration_input_path=Path(calib_input).expanduser() if calib_input else None,
            calibration_max_length=require_int(options, "calibration_max_length", 4096),
            calibration_device=cast(str, device).strip(),
            calibration_attn_implementation=require_choice(
                options, "calibration_attn_implementation", "eager", {"eager", "sdpa", "flash_attention_2"}),
            calibration_local_files_only=_bool_option(options, "calibration_local_files_only", False),
            kv_budget=require_int(options, "kv_budget", 2048),
            recompute_window=require_int(options, "recompute_window", ASCEND_BLOCK_SIZE),
            position_policy=cast(PositionPolicy, require_choice(options, "position_policy", "global", {"global", "v3"})),
            protected_prefix_window=require_int(options, "protected_prefix_window", 0),
            protected_recent_window=require_int(options, "protected_recent_window", ASCEND_BLOCK_SIZE),
            position_segments=require_int(options, "position_segments", 8),
            score_aggregation=cast(ScoreAggregation, require_choice(options, "score_aggregation", "mean", {"mean", "max"})),
            layer_aggregation=cast(LayerAggregation, require_choice(options, "layer_aggregation", "mean", {"mean", "max"})),
            score_chunk_size=require_int(options, "score_chunk_size", 512),
            score_layer_stride=require_int(options, "score_layer_stride", 8),
            min_output_tokens_for_compression=require_int(options, "min_output_tokens_for_compression", 0),
            online_calibration_window=require_int(options, "online_calibration_window", 0),
            online_calibration_min_tokens=require_int(options, "online_calibration_min_tokens", 16384),
        )
        cfg._validate()
        return cfg

    def _validate(self) -> None:
        for name in ("kv_budget", "recompute_window", "score_chunk_size"):
            value = getattr(self, name)
            if value <= 0 or value % ASCEND_BLOCK_SIZE:
                raise ValueError(f"method option {name!r} must be a positive multiple of {ASCEND_BLOCK_SIZE}")
        for name in ("protected_prefix_window", "protected_recent_window"):
            value = getattr(self, name)
            if value < 0:
                raise ValueError(f"method option {name!r} must be non-negative")
            if value > self.kv_budget:
                raise ValueError(f"method option {name!r} cannot exceed 'kv_budget'")
        if self.protected_prefix_window + self.protected_recent_window > self.kv_budget:
            raise ValueError("protected prefix and recent windows cannot exceed 'kv_budget'")
        if self.position_segments <= 0:
            raise ValueError("method option 'position_segments' must be positive")
        if self.score_layer_stride <= 0:
            raise ValueError("method option 'score_layer_stride' must be positive")
        if self.min_output_tokens_for_compression < 0:
            raise ValueError("method option 'min_output_tokens_for_compression' must be non-negative")
        if self.online_calibration_window < 0:
            raise ValueError("method option 'online_calibration_window' must be non-negative")
        if self.online_calibration_min_tokens <= 0:
            raise ValueError("method option 'online_calibration_min_tokens' must be positive")
        if self.calibration_max_length < 128:
            raise ValueError("method option 'calibration_max_length' must be at least 128")
