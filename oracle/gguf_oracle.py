"""CPU oracle for the GGUF quantized-linear path — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only tests/, the smoke() entry
of __graft_entry__.py and bench.py's CPU-baseline / reference arm may import it.
The product (dracort_b200) never calls it and has no CPU fallback.

It restates, in numpy, the algorithm of the reference's own implementation of
the path (sadrasa97/DracoRT, paths relative to that project):

* ``f16_from_u8``      — draco/format/gguf.py:256-259 (_f16_from_u8)
* ``dequantize``       — draco/format/gguf.py:272-497 (_dequantize), branches
  Q8_0 (:300-303), Q4_0 / Q4_1 (:310-324), Q5_0 / Q5_1 (:326-353), Q4_K and
  Q5_K (:425-468, _scale_min :436-442), Q6_K (:470-495),
  plus the argument checks of :284-296.  Each element is produced with the
  same fp32 operations in the same order, so results are bit-identical.
* ``matmul_f32``       — draco/runtime/cpu/kernels/generic.py:32-33
  (activation.astype(f32) @ weight.astype(f32).T)
* ``linear``           — draco/runtime/cpu/executor.py:47-79 (_linear: dequant
  then matmul_f32, plus bias)

Q6_K field order: the reference decodes d from bytes 0:2 (gguf.py:470-474,
"d_first").  ``q6k_order="d_last"`` decodes the order llama.cpp writes to .gguf
files (d at bytes 208:210) by moving d to the front and running the same
reference decode; that variant is pinned against the `gguf` 0.19.0 Python
package (llama.cpp's own decoder) by tests/golden/make_golden.py.

Pinning: tests/golden/*.npz hold outputs of the reference's _dequantize run in
the build container (tests/golden/make_golden.py), and test_oracle.py checks
this module against them and against the reference tests' plain-loop Q4_K
known-answer decoder (tests/format/test_gguf.py:281-301).
"""

from __future__ import annotations

import numpy as np

GGML_TYPE_Q4_0 = 2
GGML_TYPE_Q4_1 = 3
GGML_TYPE_Q5_0 = 6
GGML_TYPE_Q5_1 = 7
GGML_TYPE_Q8_0 = 8
GGML_TYPE_Q4_K = 12
GGML_TYPE_Q5_K = 13
GGML_TYPE_Q6_K = 14

BLOCK_LAYOUTS = {GGML_TYPE_Q4_0: (32, 18), GGML_TYPE_Q4_1: (32, 20), GGML_TYPE_Q5_0: (32, 22),
                 GGML_TYPE_Q5_1: (32, 24), GGML_TYPE_Q8_0: (32, 34), GGML_TYPE_Q4_K: (256, 144),
                 GGML_TYPE_Q5_K: (256, 176), GGML_TYPE_Q6_K: (256, 210)}
# 32-element types with 4-bit quants: (has m, has qh) per type
_LEGACY = {GGML_TYPE_Q4_0: (False, False), GGML_TYPE_Q4_1: (True, False), GGML_TYPE_Q5_0: (False, True),
           GGML_TYPE_Q5_1: (True, True)}


class OracleFormatError(ValueError):
    """Raised where the reference raises DracoFormatError (gguf.py:284-296)."""


def f16_from_u8(u8: np.ndarray) -> np.ndarray:
    """(..., 2) little-endian uint8 -> (...) fp32 (gguf.py:256-259)."""
    u = u8[..., 0].astype(np.uint32) | (u8[..., 1].astype(np.uint32) << 8)
    return u.astype(np.uint16).view(np.float16).astype(np.float32)


def _blocks(qtype: int, payload, n: int) -> np.ndarray:
    if qtype not in BLOCK_LAYOUTS:
        raise OracleFormatError(f"GGUF quantization type {qtype} is not supported by the oracle")
    bs, bb = BLOCK_LAYOUTS[qtype]
    if n % bs != 0:
        raise OracleFormatError(f"element count {n} is not divisible by block size {bs} for ggml type {qtype}")
    nb = n // bs
    return np.frombuffer(bytes(payload) if not isinstance(payload, np.ndarray) else payload.tobytes(),
                         dtype=np.uint8).reshape(nb, bb)


def _q6k_to_d_first(b: np.ndarray) -> np.ndarray:
    out = np.empty_like(b)
    out[:, 0:2] = b[:, 208:210]
    out[:, 2:210] = b[:, 0:208]
    return out


def dequantize(qtype: int, payload, n: int, q6k_order: str = "d_first") -> np.ndarray:
    """Flat fp32 array of n elements, bit-identical to gguf._dequantize."""
    b = _blocks(qtype, payload, n)
    nb = b.shape[0]
    if qtype == GGML_TYPE_Q8_0:
        d = f16_from_u8(b[:, 0:2])
        qs = b[:, 2:34].view(np.int8).astype(np.float32)
        return (qs * d[:, None]).reshape(-1)
    if qtype in _LEGACY:
        # gguf.py:310-353.  Fields in order: d, m (Q4_1 / Q5_1), qh (Q5_x, a
        # little-endian uint32 whose bit e is the fifth bit of element e),
        # qs[16]: element e < 16 is the low nibble of byte e, element e >= 16
        # the high nibble of byte e - 16.
        has_m, has_h = _LEGACY[qtype]
        d = f16_from_u8(b[:, 0:2])
        pos = 2
        if has_m:
            m = f16_from_u8(b[:, 2:4])
            pos = 4
        q = np.concatenate([b[:, pos + 4 * has_h:] & 15, b[:, pos + 4 * has_h:] >> 4], axis=1).astype(np.int32)
        if has_h:
            qh = np.ascontiguousarray(b[:, pos:pos + 4]).view("<u4")[:, 0]
            q |= ((qh[:, None] >> np.arange(32, dtype=np.uint32)) & 1).astype(np.int32) << 4
        if has_m:  # q * d + m: the product is exact, one rounding in the add
            return (q.astype(np.float32) * d[:, None] + m[:, None]).reshape(-1)
        return ((q - (16 if has_h else 8)).astype(np.float32) * d[:, None]).reshape(-1)

    if qtype in (GGML_TYPE_Q4_K, GGML_TYPE_Q5_K):
        # Q5_K (gguf.py:425-468) shares Q4_K's scales; its fifth bits sit in
        # qh[l] bit j for element l of sub-block j, and numpy forms
        # d*sc * (q + 16 h) - dmin*m in float64 before the one rounding to
        # fp32 (same value: the product and the difference are exact there)
        d = f16_from_u8(b[:, 0:2])
        dmin = f16_from_u8(b[:, 2:4])
        sc = b[:, 4:16]
        qh = b[:, 16:48] if qtype == GGML_TYPE_Q5_K else None
        qs = b[:, 48:176] if qtype == GGML_TYPE_Q5_K else b[:, 16:144]

        def scale_min(j):
            if j < 4:
                return sc[:, j] & 63, sc[:, j + 4] & 63
            return ((sc[:, j + 4] & 0x0F) | ((sc[:, j - 4] >> 6) << 4),
                    (sc[:, j + 4] >> 4) | ((sc[:, j] >> 6) << 4))

        out = np.empty((nb, 256), dtype=np.float32)
        for g in range(4):
            s0, m0 = scale_min(2 * g)
            s1, m1 = scale_min(2 * g + 1)
            d1 = d * s0.astype(np.float32)
            mm1 = dmin * m0.astype(np.float32)
            d2 = d * s1.astype(np.float32)
            mm2 = dmin * m1.astype(np.float32)
            q = qs[:, 32 * g : 32 * g + 32]
            if qh is None:
                out[:, 64 * g : 64 * g + 32] = d1[:, None] * (q & 0x0F).astype(np.float32) - mm1[:, None]
                out[:, 64 * g + 32 : 64 * g + 64] = d2[:, None] * (q >> 4).astype(np.float32) - mm2[:, None]
            else:
                h1 = np.where((qh & np.uint8(1 << (2 * g))) != 0, 16, 0)
                h2 = np.where((qh & np.uint8(1 << (2 * g + 1))) != 0, 16, 0)
                v1 = d1[:, None].astype(np.float64) * ((q & 0x0F).astype(np.int64) + h1) - mm1[:, None]
                v2 = d2[:, None].astype(np.float64) * ((q >> 4).astype(np.int64) + h2) - mm2[:, None]
                out[:, 64 * g : 64 * g + 32] = v1.astype(np.float32)
                out[:, 64 * g + 32 : 64 * g + 64] = v2.astype(np.float32)
        return out.reshape(-1)

    # Q6_K
    if q6k_order == "d_last":
        b = _q6k_to_d_first(b)
    elif q6k_order != "d_first":
        raise OracleFormatError(f"unknown Q6_K order {q6k_order!r}")
    d = f16_from_u8(b[:, 0:2])
    ql = b[:, 2:130]
    qh = b[:, 130:194]
    sc = b[:, 194:210].view(np.int8).astype(np.int32)
    out = np.empty((nb, 256), dtype=np.float32)
    for n_ in range(2):
        ql_ = ql[:, 64 * n_ : 64 * n_ + 64].astype(np.int32)
        qh_ = qh[:, 32 * n_ : 32 * n_ + 32].astype(np.int32)
        sc_ = sc[:, 8 * n_ : 8 * n_ + 8]
        l = np.arange(32)
        is_ = l // 16
        q1 = ((ql_[:, l] & 0x0F) | (((qh_[:, l] >> 0) & 3) << 4)) - 32
        q2 = ((ql_[:, l + 32] & 0x0F) | (((qh_[:, l] >> 2) & 3) << 4)) - 32
        q3 = ((ql_[:, l] >> 4) | (((qh_[:, l] >> 4) & 3) << 4)) - 32
        q4 = ((ql_[:, l + 32] >> 4) | (((qh_[:, l] >> 6) & 3) << 4)) - 32
        # d * sc in fp32 (exact), then the product with the integer quant is
        # formed in float64 and rounded once to fp32, as numpy's
        # float32 * int32 promotion does in the reference
        dl0 = d[:, None] * sc_[:, is_ + 0].astype(np.float32)
        dl1 = d[:, None] * sc_[:, is_ + 2].astype(np.float32)
        dl2 = d[:, None] * sc_[:, is_ + 4].astype(np.float32)
        dl3 = d[:, None] * sc_[:, is_ + 6].astype(np.float32)
        base = 128 * n_
        out[:, base + l] = (dl0.astype(np.float64) * q1).astype(np.float32)
        out[:, base + 32 + l] = (dl1.astype(np.float64) * q2).astype(np.float32)
        out[:, base + 64 + l] = (dl2.astype(np.float64) * q3).astype(np.float32)
        out[:, base + 96 + l] = (dl3.astype(np.float64) * q4).astype(np.float32)
    return out.reshape(-1)


def dequantize_matrix(qtype: int, packed: np.ndarray, n_rows: int, k: int, q6k_order: str = "d_first") -> np.ndarray:
    """GGUF [n_rows, k] weight -> fp32 matrix (gguf.py:820-834 without the cache)."""
    return dequantize(qtype, np.ascontiguousarray(packed), n_rows * k, q6k_order).reshape(n_rows, k)


def matmul_f32(activation: np.ndarray, weight: np.ndarray) -> np.ndarray:
    """generic.py:32-33."""
    return activation.astype(np.float32, copy=False) @ weight.astype(np.float32, copy=False).T


def linear(x: np.ndarray, qtype: int, packed: np.ndarray, n_rows: int, k: int, bias=None,
           q6k_order: str = "d_first") -> np.ndarray:
    """executor._linear (executor.py:47-79) for a GGUF tensor: dequantize, matmul, + bias."""
    w = dequantize_matrix(qtype, packed, n_rows, k, q6k_order)
    out = matmul_f32(x, w)
    if bias is not None:
        out = out + bias
    return out


def linear_f64(x: np.ndarray, qtype: int, packed: np.ndarray, n_rows: int, k: int, bias=None,
               q6k_order: str = "d_first") -> np.ndarray:
    """Same as ``linear`` but accumulated in float64 (a tighter yardstick for error budgets)."""
    w = dequantize_matrix(qtype, packed, n_rows, k, q6k_order).astype(np.float64)
    out = x.astype(np.float64) @ w.T
    if bias is not None:
        out = out + bias
    return out


def rel_l2(got: np.ndarray, ref: np.ndarray) -> float:
    """||got - ref||_2 / ||ref||_2 (the tolerance metric of the parity rules)."""
    g = np.asarray(got, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    den = np.linalg.norm(r)
    return float(np.linalg.norm(g - r) / (den if den > 0 else 1.0))
