"""Quantization registry — same contract as draco/quantization/registry.py.

``QuantizationRegistry`` (registry.py:21-86) maps lower-cased method names to
backend instances: ``register`` warns when a name is re-registered (:31-42),
``get`` raises ValueError listing the available methods (:44-52), plus
``has``/``list_methods``/``list_backends``/``detect_from_config`` and the
container dunders.  ``QUANT_REGISTRY`` is the process-wide singleton (:90).
"""

from __future__ import annotations

import logging
from typing import Any, Dict, List, Optional

from dracort_b200.quantization.base import QuantizationBackend

logger = logging.getLogger("dracort_b200.quantization.registry")


class QuantizationRegistry:
    """Central registry for quantization backends."""

    def __init__(self) -> None:
        self._backends: Dict[str, QuantizationBackend] = {}

    def register(self, name: str, backend: QuantizationBackend) -> None:
        name = name.lower()
        if name in self._backends:
            logger.warning(
                "Re-registering quantization backend '%s': %s -> %s",
                name,
                type(self._backends[name]).__name__,
                type(backend).__name__,
            )
        self._backends[name] = backend

    def get(self, name: str) -> QuantizationBackend:
        name = name.lower()
        if name not in self._backends:
            raise ValueError(f"Unknown quantization method: {name!r}. Available: {self.list_methods()}")
        return self._backends[name]

    def has(self, name: str) -> bool:
        return name.lower() in self._backends

    def list_methods(self) -> List[str]:
        return sorted(self._backends.keys())

    def list_backends(self) -> Dict[str, QuantizationBackend]:
        return dict(self._backends)

    def detect_from_config(self, quantization_config: Dict[str, Any]) -> Optional[str]:
        method = quantization_config.get("quant_method", quantization_config.get("quantization_method"))
        if method and method.lower() in self._backends:
            return method.lower()
        return None

    def __contains__(self, name: str) -> bool:
        return self.has(name)

    def __len__(self) -> int:
        return len(self._backends)

    def __repr__(self) -> str:
        return f"QuantizationRegistry(methods={self.list_methods()})"


QUANT_REGISTRY = QuantizationRegistry()
