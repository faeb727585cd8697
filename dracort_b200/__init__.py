"""dracort_b200 — B200-native (sm_100a) GGUF quantized-linear hot path.

A drop-in for DracoRT's GGUF linear path: block dequantization (Q4_0, Q4_1,
Q5_0, Q5_1, Q8_0, Q4_K, Q5_K, Q6_K) fused into decode GEMV and prefill GEMM
kernels, behind the reference's
QuantizationBackend / registry API (draco/quantization) and fused-op
signatures (draco/kernels).  All compute runs in libdraco_gguf.so (CUDA,
sm_100a); see ``dracort_b200.build`` to compile it.
"""

__version__ = "0.1.0"
