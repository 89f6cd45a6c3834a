"""String-keyed plugin registries with the reference's semantics.

Restates ``snapmind.core.registry.Registry`` (snapmind/core/registry.py:17-88):
``register(key, cls=None, *, override=False)`` works as a call or a decorator,
rejects a class that does not subclass the expected type with ``TypeError``,
rejects a duplicate key without ``override`` with ``RegistryError``;
``create(key, **kw)`` instantiates, ``get(key)`` returns the stored object, both
raise ``RegistryError`` for unknown keys; ``list()`` and ``in`` enumerate keys.
The singletons mirror ``KV_CACHE``, ``ATTENTION`` and ``INDEXER``
(snapmind/core/registry.py:92-111), so this package's plugins can be created
by key on a host that does not ship snapmind.  Where snapmind is importable,
:func:`snapmind_b200.integration.register_with_snapmind` registers the same
plugins into snapmind's own ``KV_CACHE`` / ``ATTENTION`` / ``INDEXER``.
"""
from __future__ import annotations

from collections.abc import Callable
from typing import Any


class RegistryError(Exception):
    """Raised on registry conflicts (duplicate key) or lookups (unknown key)."""


class Registry:
    def __init__(self, name: str, expected_type: type):
        self._name = name
        self._expected_type = expected_type
        self._registry: dict[str, Any] = {}

    @property
    def name(self) -> str:
        return self._name

    def register(self, key: str, cls: Any = None, *, override: bool = False) -> Callable:
        def _register(obj: Any) -> Any:
            if isinstance(obj, type) and not issubclass(obj, self._expected_type):
                raise TypeError(
                    f"Cannot register {obj.__name__} with key '{key}': "
                    f"must subclass {self._expected_type.__name__}"
                )
            if key in self._registry and not override:
                raise RegistryError(f"already registered: '{key}' in '{self._name}' registry")
            self._registry[key] = obj
            return obj

        if cls is not None:
            return _register(cls)
        return _register

    def create(self, key: str, **kwargs) -> Any:
        if key not in self._registry:
            raise RegistryError(f"unknown key '{key}' in '{self._name}' registry")
        return self._registry[key](**kwargs)

    def get(self, key: str) -> Any:
        if key not in self._registry:
            raise RegistryError(f"unknown key '{key}' in '{self._name}' registry")
        return self._registry[key]

    def list(self) -> list[str]:
        return list(self._registry.keys())

    def __contains__(self, key: str) -> bool:
        return key in self._registry


KV_CACHE: Registry = Registry("kv_cache", expected_type=object)
ATTENTION: Registry = Registry("attention", expected_type=object)
INDEXER: Registry = Registry("indexer", expected_type=object)

__all__ = ["Registry", "RegistryError", "KV_CACHE", "ATTENTION", "INDEXER"]
