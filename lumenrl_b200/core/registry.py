"""Named component registries (reference: ``lumenrl/core/registry.py:11-58``)."""

from __future__ import annotations

import logging
from typing import Any, Callable

logger = logging.getLogger(__name__)


class Registry:
    def __init__(self, name: str) -> None:
        self.name = name
        self._items: dict[str, Any] = {}

    def register(self, key: str, value: Any) -> None:
        if key in self._items and self._items[key] is not value:
            logger.warning("Overwriting %s registry entry %r", self.name, key)
        self._items[key] = value

    def get(self, key: str) -> Any:
        try:
            return self._items[key]
        except KeyError:
            known = ", ".join(sorted(self._items)) or "(none registered)"
            raise KeyError(f"{self.name} registry has no entry {key!r}; registered: {known}") from None

    def __contains__(self, key: str) -> bool:
        return key in self._items

    def keys(self) -> list[str]:
        return list(self._items)

    def decorator(self, key: str) -> Callable[[Any], Any]:
        def wrap(obj: Any) -> Any:
            self.register(key, obj)
            return obj
        return wrap


WORKER_REGISTRY = Registry("worker")
ALGORITHM_REGISTRY = Registry("algorithm")
REWARD_REGISTRY = Registry("reward")
ENV_REGISTRY = Registry("environment")
