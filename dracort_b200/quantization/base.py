"""Quantization backend interface — same contract as draco/quantization/base.py.

``QuantizationBackend`` keeps the reference's abstract members and defaults
(draco/quantization/base.py:17-133) so a backend written for either package
plugs into the other's registry:

* properties ``name``, ``supported_bits``, ``supported_schemes`` (:25-41)
* ``load_quantized_weights(model_path, target_model, config, device)`` (:43-62)
* ``dequantize(weights, scales, zeros=None, group_size=128)`` (:64-84)
* ``quantized_linear(input, weight, scales, zeros=None, bias=None)`` (:86-99)
* ``supports_gpu_kernel(device)`` (:101-103), ``get_kernel_info()`` (:105-111),
  ``estimate_memory(num_params, bits, group_size)`` (:113-126)

One deliberate difference: the reference's default ``quantized_linear``
passes ``weight`` as the scales argument (base.py:98); the default here passes
``scales``.  The GGUF backend overrides the method anyway.
"""

from __future__ import annotations

import abc
from typing import Any, Dict, List, Optional

import torch
import torch.nn as nn


class QuantizationBackend(abc.ABC):
    """The contract a quantization method implements to plug into the registry."""

    @property
    @abc.abstractmethod
    def name(self) -> str:
        """The method's registry name (lower case)."""

    @property
    @abc.abstractmethod
    def supported_bits(self) -> List[int]:
        """Weight bit widths the method stores."""

    @property
    @abc.abstractmethod
    def supported_schemes(self) -> List[str]:
        """Which tensors are quantized: e.g. 'weight_only' or 'w8a8'."""

    @abc.abstractmethod
    def load_quantized_weights(
        self,
        model_path: str,
        target_model: nn.Module,
        config: Dict[str, Any],
        device: torch.device,
    ) -> nn.Module:
        """Load quantized weights into a model and return it."""

    @abc.abstractmethod
    def dequantize(
        self,
        weights: torch.Tensor,
        scales: torch.Tensor,
        zeros: Optional[torch.Tensor] = None,
        group_size: int = 128,
    ) -> torch.Tensor:
        """Dequantize weights to a float tensor."""

    def quantized_linear(
        self,
        input: torch.Tensor,
        weight: torch.Tensor,
        scales: torch.Tensor,
        zeros: Optional[torch.Tensor] = None,
        bias: Optional[torch.Tensor] = None,
    ) -> torch.Tensor:
        """input @ dequant(weight).T + bias.  Override with a fused kernel."""
        dequant_weight = self.dequantize(weight, scales, zeros)
        return torch.nn.functional.linear(input, dequant_weight, bias)

    def supports_gpu_kernel(self, device: torch.device) -> bool:
        """True when `device` runs this method with its own kernels rather than a dequantize-then-matmul fallback."""
        return device.type == "cuda"

    def get_kernel_info(self) -> Dict[str, Any]:
        return {"backend": self.name, "gpu_kernel": False, "optimized": False}

    def estimate_memory(self, num_params: int, bits: int, group_size: int = 128) -> int:
        """Estimated bytes: packed weights plus fp16 scale and zero per group."""
        quantized_bytes = num_params * bits // 8
        num_groups = num_params // group_size
        scale_bytes = num_groups * 2
        zero_bytes = num_groups * 2 if group_size > 0 else 0
        return quantized_bytes + scale_bytes + zero_bytes

    def __repr__(self) -> str:
        return f"{self.__class__.__name__}(name={self.name!r}, bits={self.supported_bits})"
