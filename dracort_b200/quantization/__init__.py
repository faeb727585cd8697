"""Quantization plugin API (mirror of draco/quantization) with the GGUF GPU backends.

Importing this package registers the GGUF backends in ``QUANT_REGISTRY``, the
way draco/quantization/_register_all.py:9-19 registers the reference's
backends at import time.  ``register_into(registry)`` registers the same
backends into any registry with a ``register(name, backend)`` method — the
reference's own ``draco.quantization.QUANT_REGISTRY`` included.
"""

from dracort_b200.format.gguf_types import GGML_TYPE_Q6_K, Q6K_D_LAST, TYPE_NAMES
from dracort_b200.quantization.base import QuantizationBackend
from dracort_b200.quantization.gguf import GGUFBackend, GGUFLinear, gguf_linear
from dracort_b200.quantization.registry import QUANT_REGISTRY, QuantizationRegistry


def gguf_backends():
    """Fresh instances of every GGUF backend, keyed by registry name."""
    bes = [GGUFBackend(qt) for qt in TYPE_NAMES] + [GGUFBackend(GGML_TYPE_Q6_K, q6k_order=Q6K_D_LAST)]
    return {b.name: b for b in bes}


def register_into(registry) -> list:
    """Register the GGUF backends into `registry`; returns the names."""
    names = []
    for name, be in gguf_backends().items():
        registry.register(name, be)
        names.append(name)
    return names


register_into(QUANT_REGISTRY)

__all__ = [
    "QUANT_REGISTRY",
    "QuantizationRegistry",
    "QuantizationBackend",
    "GGUFBackend",
    "GGUFLinear",
    "gguf_linear",
    "gguf_backends",
    "register_into",
]
