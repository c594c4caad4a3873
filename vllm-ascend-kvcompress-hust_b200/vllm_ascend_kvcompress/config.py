"""Plugin-wide constants and option validators shared by compression methods.

The names mirror the reference plugin (src/vllm_ascend_kvcompress/config.py) so
that method configurations written for it validate identically here.
"""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any, TypeAlias

PROVIDER_NAME = "ascend_kvcompress"
LEGACY_PROVIDER_NAME = "triattention_ascend"
DEFAULT_METHOD = "triattention"
SCHEMA_VERSION = 1
# Tokens per kernel KV-cache block.  The reference names it after the Ascend
# kernel block; the B200 kernels use the same 128-token page.
ASCEND_BLOCK_SIZE = 128
KERNEL_BLOCK_SIZE = ASCEND_BLOCK_SIZE
ENABLE_ENV = "VLLM_ASCEND_KVCOMPRESS_ENABLED"
CONFIG_ENV = "VLLM_ASCEND_KVCOMPRESS_CONFIG"

JsonScalar: TypeAlias = str | int | float | bool | None


def require_int(options: Mapping[str, Any], name: str, default: int) -> int:
    """Integer option (booleans rejected), else ValueError."""
    value = options.get(name, default)
    if isinstance(value, bool) or not isinstance(value, int):
        raise ValueError(f"method option {name!r} must be an integer")
    return value


def require_choice(options: Mapping[str, Any], name: str, default: str, choices: set[str]) -> str:
    """String option restricted to ``choices``, else ValueError."""
    value = options.get(name, default)
    if not isinstance(value, str) or value not in choices:
        raise ValueError(f"method option {name!r} must be one of: {', '.join(sorted(choices))}")
    return value
