"""Synthetic GGUF encoders (numpy) for Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K,
Q5_K and Q6_K.

The reference ships no GGUF K-quant quantizer (draco/format/gguf.py only
decodes), so these encoders are written from the block formats that
gguf.py:_dequantize decodes:

* Q8_0 — exactly the rule the benchmark configuration states and the
  reference's own test encoder uses (tests/format/test_gguf.py:145-155): per
  32-element block, d = max|w| / 127 stored as fp16, q = clip(rint(w / d),
  -127, 127).
* Q4_0 / Q5_0 — per 32-element block d = max|w| / 8 (/ 16), q = rint(w / d)
  + 8 (+ 16) clipped to 4 (5) bits; Q4_1 / Q5_1 — per block the affine fit
  m = min w, d = (max - min) / 15 (/ 31), q = rint((w - m) / d).  Element e
  goes to the low nibble of qs byte e (e < 16) or the high nibble of byte
  e - 16, its fifth bit to bit e of the little-endian qh word
  (gguf.py:310-353).
* Q4_K — per 32-element sub-block an affine fit (scale = (max - min) / 15,
  min clipped at 0), the 8 scales and mins quantized to 6 bits against the
  super-block's fp16 d and dmin (d = max scale / 63, dmin = max min / 63), then
  4-bit quants q = rint((w + dmin*m) / (d*sc)).  Packing follows the decode
  in gguf.py:425-456 (6-bit pairs, gguf.py:436-442).
* Q5_K — the Q4_K fit with 31 levels; the fifth bit of element l of sub-block
  j goes to bit j of qh[l] (gguf.py:457-467).
* Q6_K — per 16-element sub-block scale = max|w| / 31, the 16 scales quantized
  to int8 against an fp16 d = max scale / 127, 6-bit quants
  q = rint(w / (d*sc)) + 32 split into low nibbles (ql) and high 2 bits (qh) as
  gguf.py:470-495 unpacks them.

This is not llama.cpp's iterative quantizer; any valid packing serves, since
the GPU kernels and the parity oracle decode the same bytes.
"""

from __future__ import annotations

import numpy as np

from dracort_b200.format.gguf_types import (
    BLOCK_LAYOUTS,
    GGML_TYPE_Q4_0,
    GGML_TYPE_Q4_1,
    GGML_TYPE_Q4_K,
    GGML_TYPE_Q5_0,
    GGML_TYPE_Q5_1,
    GGML_TYPE_Q5_K,
    GGML_TYPE_Q6_K,
    GGML_TYPE_Q8_0,
    Q6K_D_FIRST,
    Q6K_D_LAST,
)


def _f16_bytes(v: np.ndarray) -> np.ndarray:
    """float array (n,) -> (n, 2) uint8 little-endian fp16."""
    return np.ascontiguousarray(v.astype(np.float16)).view(np.uint8).reshape(-1, 2)


def encode_q8_0(w: np.ndarray) -> np.ndarray:
    """[n_rows, k] float -> packed uint8 [n_rows, k/32*34]."""
    w = np.asarray(w, dtype=np.float32)
    n_rows, k = w.shape
    if k % 32:
        raise ValueError("Q8_0 needs k % 32 == 0")
    a = w.reshape(-1, 32)
    nb = a.shape[0]
    amax = np.max(np.abs(a), axis=1)
    d = np.maximum(amax, np.float32(1e-12)) / np.float32(127.0)
    qs = np.clip(np.rint(a / d[:, None]), -127, 127).astype(np.int8)
    out = np.empty((nb, 34), dtype=np.uint8)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:34] = qs.view(np.uint8)
    return out.reshape(n_rows, (k // 32) * 34)


def encode_q4_legacy(qtype: int, w: np.ndarray) -> np.ndarray:
    """[n_rows, k] float -> packed uint8 [n_rows, k/32*bb] for Q4_0, Q4_1,
    Q5_0 or Q5_1 (fields d, m, qh, qs as gguf.py:310-353 decodes them)."""
    affine = qtype in (GGML_TYPE_Q4_1, GGML_TYPE_Q5_1)
    bits = 5 if qtype in (GGML_TYPE_Q5_0, GGML_TYPE_Q5_1) else 4
    if qtype not in (GGML_TYPE_Q4_0, GGML_TYPE_Q4_1, GGML_TYPE_Q5_0, GGML_TYPE_Q5_1):
        raise ValueError(f"ggml type {qtype} is not a 32-element 4/5-bit type")
    w = np.asarray(w, dtype=np.float32)
    n_rows, k = w.shape
    if k % 32:
        raise ValueError("32-element block types need k % 32 == 0")
    a = w.reshape(-1, 32)
    nb = a.shape[0]
    top = (1 << bits) - 1
    with np.errstate(divide="ignore", invalid="ignore"):
        if affine:
            m = a.min(axis=1).astype(np.float16).astype(np.float32)
            d = ((a.max(axis=1) - m) / np.float32(top)).astype(np.float16).astype(np.float32)
            q = np.where(d[:, None] > 0, np.rint((a - m[:, None]) / d[:, None]), 0)
        else:
            half = 1 << (bits - 1)
            d = (np.abs(a).max(axis=1) / np.float32(half)).astype(np.float16).astype(np.float32)
            q = np.where(d[:, None] > 0, np.rint(a / d[:, None]), 0) + half
    q = np.clip(q, 0, top).astype(np.uint8)
    bb = BLOCK_LAYOUTS[qtype][1]
    out = np.empty((nb, bb), dtype=np.uint8)
    out[:, 0:2] = _f16_bytes(d)
    pos = 2
    if affine:
        out[:, 2:4] = _f16_bytes(m)
        pos = 4
    if bits == 5:
        qh = (((q >> 4) & 1).astype(np.uint32) << np.arange(32, dtype=np.uint32)).sum(axis=1, dtype=np.uint32)
        out[:, pos:pos + 4] = qh.astype("<u4").view(np.uint8).reshape(nb, 4)
        pos += 4
    out[:, pos:pos + 16] = (q[:, :16] & 15) | ((q[:, 16:] & 15) << 4)
    return out.reshape(n_rows, (k // 32) * bb)


def _q4k_pack_scales(sc: np.ndarray, m: np.ndarray) -> np.ndarray:
    """sc, m: (nb, 8) ints in [0, 63] -> (nb, 12) packed bytes (inverse of gguf.py:436-442)."""
    sc = sc.astype(np.uint8)
    m = m.astype(np.uint8)
    b = np.zeros((sc.shape[0], 12), dtype=np.uint8)
    for j in range(4):
        b[:, j] = (sc[:, j] & 63) | ((sc[:, j + 4] >> 4) << 6)
        b[:, j + 4] = (m[:, j] & 63) | ((m[:, j + 4] >> 4) << 6)
        b[:, j + 8] = (sc[:, j + 4] & 15) | ((m[:, j + 4] & 15) << 4)
    return b


def _affine_super_blocks(w: np.ndarray, levels: int):
    """Per 32-element sub-block affine fit q = rint((w + m) / s) in [0, levels],
    s and m quantised to 6 bits against the super-block's fp16 d / dmin."""
    a = w.reshape(-1, 8, 32)
    mn = np.minimum(a.min(axis=2), 0.0)
    mx = a.max(axis=2)
    scale = (mx - mn) / np.float32(levels)
    mins = -mn
    d = (scale.max(axis=1) / np.float32(63.0)).astype(np.float16).astype(np.float32)
    dmin = (mins.max(axis=1) / np.float32(63.0)).astype(np.float16).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d[:, None] > 0, np.clip(np.rint(scale / d[:, None]), 0, 63), 0).astype(np.int32)
        m = np.where(dmin[:, None] > 0, np.clip(np.rint(mins / dmin[:, None]), 0, 63), 0).astype(np.int32)
        eff_s = d[:, None] * sc.astype(np.float32)
        eff_m = dmin[:, None] * m.astype(np.float32)
        q = np.where(
            eff_s[:, :, None] > 0,
            np.clip(np.rint((a + eff_m[:, :, None]) / eff_s[:, :, None]), 0, levels),
            0,
        ).astype(np.uint8)
    return d, dmin, sc, m, q


def encode_q5_k(w: np.ndarray) -> np.ndarray:
    """[n_rows, k] float -> packed uint8 [n_rows, k/256*176]: the Q4_K fields
    with 5-bit quants, the fifth bit of element l of sub-block j in bit j of
    qh[l] (the layout gguf.py:425-468 decodes)."""
    w = np.asarray(w, dtype=np.float32)
    n_rows, k = w.shape
    if k % 256:
        raise ValueError("Q5_K needs k % 256 == 0")
    d, dmin, sc, m, q = _affine_super_blocks(w, 31)
    nb = q.shape[0]
    out = np.empty((nb, 176), dtype=np.uint8)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:4] = _f16_bytes(dmin)
    out[:, 4:16] = _q4k_pack_scales(sc, m)
    qh = np.zeros((nb, 32), dtype=np.uint8)
    for j in range(8):
        qh |= ((q[:, j, :] >> 4) & 1) << j
    out[:, 16:48] = qh
    qs = np.empty((nb, 128), dtype=np.uint8)
    for g in range(4):
        qs[:, 32 * g : 32 * g + 32] = (q[:, 2 * g, :] & 15) | ((q[:, 2 * g + 1, :] & 15) << 4)
    out[:, 48:176] = qs
    return out.reshape(n_rows, (k // 256) * 176)


def encode_q4_k(w: np.ndarray) -> np.ndarray:
    """[n_rows, k] float -> packed uint8 [n_rows, k/256*144]."""
    w = np.asarray(w, dtype=np.float32)
    n_rows, k = w.shape
    if k % 256:
        raise ValueError("Q4_K needs k % 256 == 0")
    a = w.reshape(-1, 8, 32)
    nb = a.shape[0]
    mn = np.minimum(a.min(axis=2), 0.0)
    mx = a.max(axis=2)
    scale = (mx - mn) / np.float32(15.0)
    mins = -mn
    d = (scale.max(axis=1) / np.float32(63.0)).astype(np.float16).astype(np.float32)
    dmin = (mins.max(axis=1) / np.float32(63.0)).astype(np.float16).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d[:, None] > 0, np.clip(np.rint(scale / d[:, None]), 0, 63), 0).astype(np.int32)
        m = np.where(dmin[:, None] > 0, np.clip(np.rint(mins / dmin[:, None]), 0, 63), 0).astype(np.int32)
        eff_s = d[:, None] * sc.astype(np.float32)
        eff_m = dmin[:, None] * m.astype(np.float32)
        q = np.where(
            eff_s[:, :, None] > 0,
            np.clip(np.rint((a + eff_m[:, :, None]) / eff_s[:, :, None]), 0, 15),
            0,
        ).astype(np.uint8)
    out = np.empty((nb, 144), dtype=np.uint8)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:4] = _f16_bytes(dmin)
    out[:, 4:16] = _q4k_pack_scales(sc, m)
    qs = np.empty((nb, 128), dtype=np.uint8)
    for g in range(4):
        qs[:, 32 * g : 32 * g + 32] = q[:, 2 * g, :] | (q[:, 2 * g + 1, :] << 4)
    out[:, 16:144] = qs
    return out.reshape(n_rows, (k // 256) * 144)


def q6k_field_offsets(order: str = Q6K_D_FIRST):
    """(d, ql, qh, scales) byte offsets inside a 210-byte Q6_K block."""
    if order == Q6K_D_FIRST:
        return 0, 2, 130, 194
    if order == Q6K_D_LAST:
        return 208, 0, 128, 192
    raise ValueError(f"unknown Q6_K field order {order!r}")


def encode_q6_k(w: np.ndarray, order: str = Q6K_D_FIRST) -> np.ndarray:
    """[n_rows, k] float -> packed uint8 [n_rows, k/256*210]."""
    w = np.asarray(w, dtype=np.float32)
    n_rows, k = w.shape
    if k % 256:
        raise ValueError("Q6_K needs k % 256 == 0")
    a = w.reshape(-1, 16, 16)
    nb = a.shape[0]
    scale = np.abs(a).max(axis=2) / np.float32(31.0)
    d = (scale.max(axis=1) / np.float32(127.0)).astype(np.float16).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d[:, None] > 0, np.clip(np.rint(scale / d[:, None]), -128, 127), 0).astype(np.int8)
        eff = d[:, None] * sc.astype(np.float32)
        q = np.where(eff[:, :, None] != 0, np.clip(np.rint(a / eff[:, :, None]), -32, 31), 0).astype(np.int32)
    q6 = (q + 32).astype(np.uint8).reshape(nb, 256)  # element order
    ql = np.zeros((nb, 128), dtype=np.uint8)
    qh = np.zeros((nb, 64), dtype=np.uint8)
    for n in range(2):
        for i in range(4):
            e0 = 128 * n + 32 * i
            v = q6[:, e0 : e0 + 32]
            dst = 64 * n + 32 * (i & 1)
            if i < 2:
                ql[:, dst : dst + 32] |= v & 15
            else:
                ql[:, dst : dst + 32] |= (v & 15) << 4
            qh[:, 32 * n : 32 * n + 32] |= (v >> 4) << (2 * i)
    od, oql, oqh, osc = q6k_field_offsets(order)
    out = np.empty((nb, 210), dtype=np.uint8)
    out[:, od : od + 2] = _f16_bytes(d)
    out[:, oql : oql + 128] = ql
    out[:, oqh : oqh + 64] = qh
    out[:, osc : osc + 16] = sc.view(np.uint8)
    return out.reshape(n_rows, (k // 256) * 210)


def q6k_reorder(packed: np.ndarray, src: str, dst: str) -> np.ndarray:
    """Convert Q6_K payload bytes between the d-first and d-last field orders."""
    if src == dst:
        return packed
    shape = packed.shape
    b = np.ascontiguousarray(packed).reshape(-1, 210)
    so, do = q6k_field_offsets(src), q6k_field_offsets(dst)
    out = np.empty_like(b)
    for (s0, ln), d0 in zip(((so[0], 2), (so[1], 128), (so[2], 64), (so[3], 16)), do):
        out[:, d0 : d0 + ln] = b[:, s0 : s0 + ln]
    return out.reshape(shape)


def encode(qtype: int, w: np.ndarray, q6k_order: str = Q6K_D_FIRST) -> np.ndarray:
    """Encode a float [n_rows, k] matrix into packed GGUF blocks of `qtype`."""
    if qtype == GGML_TYPE_Q8_0:
        return encode_q8_0(w)
    if qtype in (GGML_TYPE_Q4_0, GGML_TYPE_Q4_1, GGML_TYPE_Q5_0, GGML_TYPE_Q5_1):
        return encode_q4_legacy(qtype, w)
    if qtype == GGML_TYPE_Q4_K:
        return encode_q4_k(w)
    if qtype == GGML_TYPE_Q5_K:
        return encode_q5_k(w)
    if qtype == GGML_TYPE_Q6_K:
        return encode_q6_k(w, q6k_order)
    raise ValueError(f"no encoder for ggml type {qtype}; supported: {sorted(BLOCK_LAYOUTS)}")


def random_weight(rng: np.random.Generator, n_rows: int, k: int, std: float = 0.02) -> np.ndarray:
    """Weights drawn from N(0, std) as fp32 (the benchmark configurations use std 0.02)."""
    return rng.standard_normal((n_rows, k), dtype=np.float32) * np.float32(std)
