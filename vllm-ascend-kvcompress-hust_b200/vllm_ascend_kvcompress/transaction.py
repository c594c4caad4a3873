"""Scheduler-to-worker compression transaction (the plan handed to ``compress``)."""

from __future__ import annotations

from dataclasses import dataclass

PLAN_ATTRIBUTE = "_ascend_kvcompress_plans_v4"


@dataclass(frozen=True)
class CompressionPlan:
    """Source blocks stay immutable until the worker has filled the private destination."""

    semantic_anchor: int
    physical_anchor: int
    source_block_ids: tuple[int, ...]
    destination_block_ids: tuple[int, ...]
