"""GGUF type ids and block geometry for the quantized-linear hot path.

Values are identical to draco/format/gguf.py: the ggml_type enum
(gguf.py:56-71) and ``_BLOCK_LAYOUTS`` (gguf.py:75-87), restricted to the
block formats this library runs on the GPU (Q4_0, Q4_1, Q5_0, Q5_1, Q8_0,
Q4_K, Q5_K, Q6_K).
"""

from __future__ import annotations

from typing import Dict, Tuple

GGML_TYPE_F32 = 0
GGML_TYPE_F16 = 1
GGML_TYPE_Q4_0 = 2
GGML_TYPE_Q4_1 = 3
GGML_TYPE_Q5_0 = 6
GGML_TYPE_Q5_1 = 7
GGML_TYPE_Q8_0 = 8
GGML_TYPE_Q4_K = 12
GGML_TYPE_Q5_K = 13
GGML_TYPE_Q6_K = 14
GGML_TYPE_BF16 = 30

#: (block_size, block_bytes) per supported quantized type (gguf.py:75-87)
BLOCK_LAYOUTS: Dict[int, Tuple[int, int]] = {
    GGML_TYPE_Q4_0: (32, 18),  # d: f16 + qs: uint8[16]
    GGML_TYPE_Q4_1: (32, 20),  # d: f16 + m: f16 + qs: uint8[16]
    GGML_TYPE_Q5_0: (32, 22),  # d: f16 + qh: uint8[4] + qs: uint8[16]
    GGML_TYPE_Q5_1: (32, 24),  # d: f16 + m: f16 + qh: uint8[4] + qs: uint8[16]
    GGML_TYPE_Q8_0: (32, 34),  # d: f16 + qs: int8[32]
    GGML_TYPE_Q4_K: (256, 144),  # d: f16 + dmin: f16 + scales: uint8[12] + qs: uint8[128]
    GGML_TYPE_Q5_K: (256, 176),  # d: f16 + dmin: f16 + scales: uint8[12] + qh: uint8[32] + qs: uint8[128]
    GGML_TYPE_Q6_K: (256, 210),  # d: f16 + ql: uint8[128] + qh: uint8[64] + scales: int8[16]
}

TYPE_NAMES = {GGML_TYPE_Q4_0: "Q4_0", GGML_TYPE_Q4_1: "Q4_1", GGML_TYPE_Q5_0: "Q5_0", GGML_TYPE_Q5_1: "Q5_1",
              GGML_TYPE_Q8_0: "Q8_0", GGML_TYPE_Q4_K: "Q4_K", GGML_TYPE_Q5_K: "Q5_K", GGML_TYPE_Q6_K: "Q6_K"}
NAME_TO_TYPE = {v: k for k, v in TYPE_NAMES.items()}
#: "Q4_0=2, Q4_1=3, ..." for error messages
SUPPORTED_TYPES_TEXT = ", ".join(f"{n}={t}" for t, n in TYPE_NAMES.items())

#: Q6_K field order.  "d_first" is the order draco/format/gguf.py:470-474
#: decodes (d at bytes 0:2); "d_last" is the order llama.cpp writes in .gguf
#: files (d at bytes 208:210).  Every other type has a single order.
Q6K_D_FIRST = "d_first"
Q6K_D_LAST = "d_last"


def packed_nbytes(qtype: int, n_rows: int, k: int) -> int:
    """Payload bytes of an [n_rows, k] tensor (gguf.py:639-645)."""
    bs, bb = BLOCK_LAYOUTS[qtype]
    if k % bs:
        raise ValueError(f"row length {k} is not a multiple of block size {bs} for ggml type {qtype}")
    return n_rows * (k // bs) * bb


def bits_per_weight(qtype: int) -> float:
    bs, bb = BLOCK_LAYOUTS[qtype]
    return 8.0 * bb / bs
