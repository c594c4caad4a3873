"""``vllm.general_plugins`` entry point (``ascend_kvcompress = vllm_ascend_kvcompress.plugin:register``).

Registering makes the built-in and entry-point methods resolvable by name.  The
host lifecycle adapter of the reference plugin (scheduler transaction hooks,
model-runner patches, provider) is outside this package; a host integrates the
method through method API v1 (``create_method`` -> ``bind_model_runner`` ->
``compress``/``compress_many``).
"""

from __future__ import annotations

from .config import ENABLE_ENV
from .methods import available_methods

_registered = False


def register() -> None:
    """Idempotent plugin registration: load the method registry once."""
    global _registered
    if _registered:
        return
    available_methods()
    _registered = True


__all__ = ["register", "ENABLE_ENV"]
