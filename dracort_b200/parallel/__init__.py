"""Tensor-parallel sharding of GGUF linear layers (mirror of draco/parallel)."""
