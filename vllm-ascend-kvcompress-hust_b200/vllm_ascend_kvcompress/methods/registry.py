"""Fail-closed name -> factory registry with entry-point discovery.

Entry-point group and normalisation rules match the reference
(src/vllm_ascend_kvcompress/methods/registry.py:16-106) so third-party methods
registered for it are discovered here too.
"""

from __future__ import annotations

from collections.abc import Callable, Mapping
from importlib.metadata import entry_points
from typing import Any, TypeAlias

from ..config import JsonScalar
from .base import KVCompressionMethod, ModelShape

MethodFactory: TypeAlias = Callable[[Mapping[str, JsonScalar], Any, ModelShape], KVCompressionMethod]
METHOD_ENTRY_POINT_GROUP = "vllm_ascend_kvcompress.methods"


def _normalize_name(name: str) -> str:
    if not isinstance(name, str) or not name.strip():
        raise ValueError("compression method name must be a non-empty string")
    key = name.strip().lower()
    if not key.replace("_", "").replace("-", "").isalnum():
        raise ValueError("compression method names may contain only letters, digits, '-' and '_'")
    return key


class MethodRegistry:
    """Registered factories; duplicate names and non-method products are errors."""

    def __init__(self) -> None:
        self._factories: dict[str, MethodFactory] = {}

    def register(self, name: str, factory: MethodFactory) -> None:
        key = _normalize_name(name)
        if key in self._factories:
            raise ValueError(f"compression method {key!r} is already registered")
        if not callable(factory):
            raise TypeError("compression method factory must be callable")
        self._factories[key] = factory

    def create(self, name: str, options: Mapping[str, JsonScalar], vllm_config: Any,
               model_shape: ModelShape) -> KVCompressionMethod:
        key = _normalize_name(name)
        factory = self._factories.get(key)
        if factory is None:
            known = ", ".join(self.names()) or "<none>"
            raise ValueError(f"unknown compression method {key!r}; available: {known}")
        method = factory(options, vllm_config, model_shape)
        if not isinstance(method, KVCompressionMethod):
            raise TypeError(f"compression method factory {key!r} returned "
                            f"{type(method).__name__}, expected KVCompressionMethod")
        if method.name != key:
            raise ValueError(f"compression method factory {key!r} returned method named {method.name!r}")
        return method

    def names(self) -> tuple[str, ...]:
        return tuple(sorted(self._factories))


METHOD_REGISTRY = MethodRegistry()
_entry_points_loaded = False


def register_method(name: str, factory: MethodFactory) -> None:
    """Register an in-process method factory."""
    METHOD_REGISTRY.register(name, factory)


def load_method_entry_points() -> None:
    """Import third-party methods of the public entry-point group, once."""
    global _entry_points_loaded
    if _entry_points_loaded:
        return
    _entry_points_loaded = True
    for ep in entry_points(group=METHOD_ENTRY_POINT_GROUP):
        METHOD_REGISTRY.register(ep.name, ep.load())


def create_method(name: str, options: Mapping[str, JsonScalar], vllm_config: Any,
                  model_shape: ModelShape) -> KVCompressionMethod:
    load_method_entry_points()
    return METHOD_REGISTRY.create(name, options, vllm_config, model_shape)


def available_methods() -> tuple[str, ...]:
    load_method_entry_points()
    return METHOD_REGISTRY.names()
