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

#: (block_size, block_bytes) per supported quantized type (gguf.py:75-87).
#: Byte budget of one block, in field order: Q4_0 scale 2 + 16 nibble bytes;
#: Q4_1 scale 2 + min 2 + 16; Q5_0 scale 2 + 4 fifth-bit bytes + 16; Q5_1
#: scale 2 + min 2 + 4 + 16; Q8_0 scale 2 + 32 signed bytes; Q4_K super-scale
#: 2 + super-min 2 + 12 packed 6-bit sub-scales/mins + 128 nibble bytes; Q5_K
#: the same with 32 fifth-bit bytes before the nibbles; Q6_K (the order the
#: reference decodes) scale 2 + 128 low-nibble bytes + 64 high-pair bytes + 16
#: signed sub-scales.
BLOCK_LAYOUTS: Dict[int, Tuple[int, int]] = {
    GGML_TYPE_Q4_0: (32, 2 + 16),
    GGML_TYPE_Q4_1: (32, 2 + 2 + 16),
    GGML_TYPE_Q5_0: (32, 2 + 4 + 16),
    GGML_TYPE_Q5_1: (32, 2 + 2 + 4 + 16),
    GGML_TYPE_Q8_0: (32, 2 + 32),
    GGML_TYPE_Q4_K: (256, 2 + 2 + 12 + 128),
    GGML_TYPE_Q5_K: (256, 2 + 2 + 12 + 32 + 128),
    GGML_TYPE_Q6_K: (256, 2 + 128 + 64 + 16),
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
