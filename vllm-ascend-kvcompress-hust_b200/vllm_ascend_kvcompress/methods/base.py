"""Method API v1: the stable contracts between the lifecycle adapter and a method.

Field names, order and meaning are part of the public plugin interface
(reference: src/vllm_ascend_kvcompress/methods/base.py:15-189) and are kept so
that external methods and providers written against v1 work unchanged.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import Any

import torch

from ..transaction import CompressionPlan


@dataclass(frozen=True)
class ModelShape:
    """Framework-neutral transformer geometry a method needs."""

    model_type: str
    num_layers: int
    num_attention_heads: int
    num_kv_heads: int
    head_dim: int
    rope_theta: float
    has_rope_scaling: bool
    rotary_dim: int | None = None
    attention_layer_indices: tuple[int, ...] | None = None

    @property
    def effective_rotary_dim(self) -> int:
        return self.head_dim if self.rotary_dim is None else self.rotary_dim

    @property
    def full_attention_layer_indices(self) -> tuple[int, ...]:
        if self.attention_layer_indices is None:
            return tuple(range(self.num_layers))
        return self.attention_layer_indices

    @property
    def is_hybrid(self) -> bool:
        return len(self.full_attention_layer_indices) != self.num_layers


@dataclass(frozen=True)
class MethodRuntimeSpec:
    """Limits the scheduler must know before KV allocation."""

    requires_private_destination: bool
    compression_threshold_tokens: int
    required_recompute_tokens: int
    max_physical_num_tokens: int
    min_output_tokens_for_compression: int = 0


@dataclass(frozen=True)
class LayerCache:
    """A validated full-attention K/V cache pair, ``[blocks, 128, kv_heads, head_dim]``."""

    name: str
    layer_index: int
    k_cache: torch.Tensor
    v_cache: torch.Tensor


@dataclass(frozen=True)
class CompressionRequest:
    """One compression transaction as seen by a method."""

    request_id: str
    semantic_num_tokens: int
    physical_num_tokens: int
    source_block_ids: tuple[tuple[int, ...], ...]
    destination_block_ids: tuple[tuple[int, ...], ...]
    source_block_ids_device: torch.Tensor
    destination_block_ids_device: torch.Tensor
    plan: CompressionPlan | None = None
    per_layer_physical_num_tokens: tuple[tuple[str, int], ...] | None = None


@dataclass(frozen=True)
class CompressionResult:
    """Physical KV state a method produced."""

    physical_num_tokens: int
    per_layer_physical_num_tokens: tuple[tuple[str, int], ...] | None = None


@dataclass(frozen=True)
class QueryBatchSpan:
    """Rows ``[start, end)`` of one request inside a forward's query batch."""

    request_id: str
    start: int
    end: int


@dataclass(frozen=True)
class QueryObservation:
    """A completed final-prefill transaction whose buffered queries may be published."""

    request_id: str
    plan: CompressionPlan
    semantic_num_tokens: int
    window_tokens: int
    layer_indices: tuple[int, ...]


class KVCompressionMethod(ABC):
    """What a compression algorithm implements beneath the lifecycle adapter."""

    @property
    @abstractmethod
    def name(self) -> str:
        """Stable configuration name."""

    @property
    @abstractmethod
    def runtime_spec(self) -> MethodRuntimeSpec:
        """Scheduler-visible limits, known before KV allocation."""

    @abstractmethod
    def compatibility_reasons(self, worker: Any) -> tuple[str, ...]:
        """Incompatibilities with the worker, without side effects (empty = compatible)."""

    @abstractmethod
    def bind_model_runner(self, runner: Any, layer_caches: tuple[LayerCache, ...]) -> None:
        """Bind device state after the KV caches exist."""

    @abstractmethod
    def compress(self, request: CompressionRequest) -> CompressionResult:
        """Materialise one transaction into its private destination blocks."""

    @property
    def query_window_tokens(self) -> int:
        """Trailing prefill query rows needed per full-attention layer (0: no hooks)."""
        return 0

    @property
    def query_layer_indices(self) -> tuple[int, ...] | None:
        """Model layers whose queries are observed; None means every bound layer."""
        return None

    @property
    def requires_per_layer_physical_state(self) -> bool:
        """True when results may differ per layer, so graph capture needs per-layer metadata."""
        return False

    def capture_query(self, layer: LayerCache, query: torch.Tensor, spans: tuple[QueryBatchSpan, ...]) -> None:
        """Copy prefill query rows into method-owned, address-stable buffers."""
        return None

    def complete_query_observation(self, observation: QueryObservation) -> None:
        """Publish buffered queries after a successful forward."""
        return None

    def discard_query_observation(self, request_id: str) -> None:
        """Drop one request's unpublished observation."""
        return None
