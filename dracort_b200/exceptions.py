"""Exception classes of the hot path, with the reference's names and hierarchy.

Mirrors the subset of draco/exceptions.py that the GGUF path raises:
``DracoFormatError`` (draco/exceptions.py:65; raised by gguf.py:284-296 for an
unsupported type or a size that is not a multiple of the block size),
``QuantizationError`` (:29), ``KernelError`` (:45, a CUDA kernel failed or is
unavailable) and ``CPUQuantizationError`` (:97).  Names, base classes and
meaning match the reference so that ``except DracoFormatError`` code ports
unchanged.
"""

from __future__ import annotations


class DracoError(Exception):
    """Base error for all Draco exceptions (draco/exceptions.py:6)."""


class QuantizationError(DracoError):
    """Raised when quantization operations fail (draco/exceptions.py:29)."""


class GPUError(DracoError):
    """Raised when GPU operations fail (draco/exceptions.py:33)."""


class KernelError(DracoError):
    """Raised when a CUDA kernel is unavailable or fails (draco/exceptions.py:45)."""


class DracoFormatError(DracoError):
    """Raised when a GGUF/.draco payload is malformed (draco/exceptions.py:65)."""


class CPUError(DracoError):
    """Raised when native CPU runtime operations fail (draco/exceptions.py:81)."""


class CPUQuantizationError(CPUError):
    """Raised when CPU-native (de)quantization fails (draco/exceptions.py:97)."""


class CollectiveTimeoutError(DracoError):
    """A tensor/expert-parallel collective did not complete in time."""
