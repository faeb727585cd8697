"""Name -> backend lookup for the quantization plugins.

Callers of draco/quantization/registry.py rely on a few behaviours, which
this table provides: names are case-insensitive (stored lower-cased),
registering a taken name replaces the entry and logs a warning, an unknown
name raises ValueError naming what is available, and a model's
``quantization_config`` can be matched to a registered name.  The public
method names are the ones the reference's callers use (register, get, has,
list_methods, list_backends, detect_from_config, ``in``, ``len``), so the
GGUF backends can be registered here or in the reference's own registry
(``register_into`` in this package).
"""

from __future__ import annotations

import logging
from typing import Any, Dict, List, Mapping, Optional

from dracort_b200.quantization.base import QuantizationBackend

_log = logging.getLogger(__name__)

# keys a quantization_config may name its method under, in lookup order
_CONFIG_KEYS = ("quant_method", "quantization_method")


def _key(name: str) -> str:
    return str(name).lower()


class QuantizationRegistry:
    """A case-insensitive table of quantization backends."""

    def __init__(self) -> None:
        self._table: Dict[str, QuantizationBackend] = {}

    def register(self, name: str, backend: QuantizationBackend) -> None:
        key = _key(name)
        previous = self._table.get(key)
        if previous is not None:
            _log.warning("quantization backend %r replaced (%s by %s)", key, type(previous).__name__,
                         type(backend).__name__)
        self._table[key] = backend

    def get(self, name: str) -> QuantizationBackend:
        try:
            return self._table[_key(name)]
        except KeyError:
            raise ValueError(f"no quantization backend named {_key(name)!r}; "
                             f"registered: {', '.join(self.list_methods()) or 'none'}") from None

    def has(self, name: str) -> bool:
        return _key(name) in self._table

    def list_methods(self) -> List[str]:
        return sorted(self._table)

    def list_backends(self) -> Dict[str, QuantizationBackend]:
        return self._table.copy()

    def detect_from_config(self, quantization_config: Mapping[str, Any]) -> Optional[str]:
        """The registered name a model's quantization_config asks for, or None."""
        for field in _CONFIG_KEYS:
            method = quantization_config.get(field)
            if method:
                return _key(method) if self.has(method) else None
        return None

    __contains__ = has

    def __len__(self) -> int:
        return len(self._table)

    def __repr__(self) -> str:
        return f"{type(self).__name__}({self.list_methods()})"


#: the process-wide table the GGUF backends register into at import
QUANT_REGISTRY = QuantizationRegistry()
