"""Kernel-level entry points with the reference's signatures.

* ``fused_swiGLU(x, gate_proj, up_proj, down_proj)`` — draco/kernels/ops.py:
  114-137, ``down_proj(silu(gate_proj(x)) * up_proj(x))``.  When the three
  projections are ``GGUFLinear`` modules (no bias) the MLP runs as three
  device steps: gate and up in one grouped launch (the decode GEMV for fp32
  or short inputs, the tcgen05 GEMM for bf16/fp16 prefill batches), the
  SwiGLU product in one elementwise kernel (in place over gate), and down.
  Any other callables are composed exactly as the reference does, which is
  its contract ("accepts any callables").
* ``GGUFGemmKernel`` — the executor's kernel interface (``CPUGemmKernel``,
  draco/runtime/cpu/kernels/base.py:15-45: ``name``, ``tier``,
  ``supports``, ``matmul_f32``, ``matmul(activation, tensor_info,
  payload_bytes)``) served by the GPU: numpy in, numpy out, the packed GGUF
  payload regrouped once per named tensor and kept on the device.
"""

from __future__ import annotations

import threading
from collections import OrderedDict
from typing import Any, Optional

import numpy as np
import torch
import torch.nn.functional as F

from dracort_b200 import gguf_ops as G
from dracort_b200.exceptions import DracoFormatError
from dracort_b200.format.gguf_types import GGML_TYPE_Q6_K, SUPPORTED_TYPES_TEXT, TYPE_NAMES
from dracort_b200.quantization.gguf import GEMV_MAX_ROWS, PREFILL_MIN_ROWS, GGUFLinear, gguf_linear


def _fusable(x: torch.Tensor, gate: Any, up: Any, down: Any) -> bool:
    if not all(isinstance(m, GGUFLinear) for m in (gate, up, down)):
        return False
    if any(m.bias is not None for m in (gate, up, down)):
        return False
    if not x.is_cuda or any(m.tiled.device != x.device for m in (gate, up, down)):
        return False
    return (gate.in_features == up.in_features == x.shape[-1] and gate.out_features == up.out_features
            and down.in_features == gate.out_features)


def fused_swiGLU(x: torch.Tensor, gate_proj, up_proj, down_proj) -> torch.Tensor:
    """down_proj(silu(gate_proj(x)) * up_proj(x)) (draco/kernels/ops.py:114-137)."""
    if not _fusable(x, gate_proj, up_proj, down_proj):
        return down_proj(F.silu(gate_proj(x)) * up_proj(x))
    k, f, h = gate_proj.in_features, gate_proj.out_features, down_proj.out_features
    lead = x.shape[:-1]
    x2 = x.reshape(-1, k)
    m = x2.shape[0]
    if m == 0:
        return x.new_empty(*lead, h)
    if x2.dtype in (torch.bfloat16, torch.float16) and m >= PREFILL_MIN_ROWS:
        xb = x2.to(torch.bfloat16).contiguous()
        gu = torch.empty((2, m, f), dtype=torch.bfloat16, device=x.device)
        G.gemm_grouped([G.GemmProblem(gate_proj.qtype, gate_proj.tiled, xb, gu[0], f, k),
                        G.GemmProblem(up_proj.qtype, up_proj.tiled, xb, gu[1], f, k)])
        G.swiglu_bf16(gu[0], gu[1], out=gu[0])
        ydt = x.dtype if x.dtype in (torch.bfloat16, torch.float32) else torch.float32
        y = G.gemm(down_proj.qtype, down_proj.tiled, gu[0], h, f, out_dtype=ydt)
        return y.reshape(*lead, h).to(x.dtype)
    xf = x2.float().contiguous()
    y = torch.empty((m, h), dtype=torch.float32, device=x.device)
    for r0 in range(0, m, GEMV_MAX_ROWS):
        r1 = min(m, r0 + GEMV_MAX_ROWS)
        gu = torch.empty((2, r1 - r0, f), dtype=torch.float32, device=x.device)
        G.gemv_grouped([G.GemvProblem(gate_proj.qtype, gate_proj.tiled, xf[r0:r1], gu[0], f, k),
                        G.GemvProblem(up_proj.qtype, up_proj.tiled, xf[r0:r1], gu[1], f, k)])
        # the SwiGLU product is formed as the down GEMV reads its input
        G.gemv_grouped([G.GemvProblem(down_proj.qtype, down_proj.tiled, gu[0], y[r0:r1], h, f, up=gu[1])])
    return y.reshape(*lead, h).to(x.dtype)


def fused_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x * rsqrt(mean(x^2, -1) + eps) * weight (draco/kernels/ops.py:29-50) on
    the GPU for contiguous fp32 / bf16 CUDA tensors; other inputs take the
    reference's own formula."""
    if x.is_cuda and x.dtype in (torch.float32, torch.bfloat16) and x.is_contiguous():
        return G.rms_norm(x, weight, eps)
    variance = x.pow(2).mean(-1, keepdim=True)
    return x * torch.rsqrt(variance + eps) * weight


def fused_rms_norm_linear(x: torch.Tensor, norm_weight: torch.Tensor, eps: float, projections) -> list:
    """[proj(fused_rms_norm(x, norm_weight, eps)) for proj in projections] for
    GGUFLinear projections sharing the normalised input (q/k/v after the
    input norm, gate/up after the post-attention norm): one grouped GEMV
    launch that applies the norm as it reads x (decode batches of fp32 rows)."""
    k = projections[0].in_features
    x2 = x.reshape(-1, k).float().contiguous()
    w = norm_weight.to(device=x.device, dtype=torch.float32).contiguous()
    outs = [torch.empty((x2.shape[0], p.out_features), dtype=torch.float32, device=x.device) for p in projections]
    G.gemv_grouped([G.GemvProblem(p.qtype, p.tiled, x2, o, p.out_features, k, p.bias, norm_weight=w, norm_eps=eps)
                    for p, o in zip(projections, outs)])
    return [o.reshape(*x.shape[:-1], o.shape[-1]) for o in outs]


_TYPE_OF_NAME = {"gguf_" + n.lower(): t for t, n in TYPE_NAMES.items()}


class GGUFGemmKernel:
    """GPU kernel behind the executor's kernel interface.

    ``matmul(activation, tensor_info, payload_bytes)`` takes a tensor
    description with ``ggml_type`` (a ``GgufTensorInfo``, gguf.py:505-520) or a
    ``quantization`` name ``gguf_<type>`` (``gguf_q4_0`` ... ``gguf_q6_k``), and
    ``shape == (n_rows, k)``; the payload is the tensor's packed GGUF bytes
    (Q6_K in the reference's byte order unless ``q6k_order="d_last"``).  The
    regrouped weight is cached per (name, offset), up to ``cache_bytes`` of
    device memory, least recently used first out; a tensor description
    without a name and offset is regrouped on every call.
    """

    tier = "b200"

    def __init__(self, device: Optional[torch.device] = None, cache_bytes: int = 8 << 30,
                 q6k_order: str = "d_first") -> None:
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.cache_bytes = int(cache_bytes)
        self.q6k_order = q6k_order
        self._cache: "OrderedDict[Any, torch.Tensor]" = OrderedDict()
        self._held = 0
        self._lock = threading.Lock()

    @property
    def name(self) -> str:
        return "b200 (sm_100a GGUF dequant-GEMV / tcgen05 GEMM)"

    def supports(self, quantization: Optional[str]) -> bool:
        return quantization is None or quantization in _TYPE_OF_NAME

    def matmul_f32(self, activation: np.ndarray, weight: np.ndarray) -> np.ndarray:
        """``activation @ weight.T`` for an already dequantized fp32 weight (the
        reference's GGUF path, generic.py:32-33): a plain fp32 GEMM on the device."""
        a = torch.from_numpy(np.ascontiguousarray(activation, dtype=np.float32)).to(self.device)
        w = torch.from_numpy(np.ascontiguousarray(weight, dtype=np.float32)).to(self.device)
        return (a @ w.T).cpu().numpy()

    def _qtype(self, tensor_info) -> int:
        qt = getattr(tensor_info, "ggml_type", None)
        if qt in TYPE_NAMES:
            return int(qt)
        q = getattr(tensor_info, "quantization", None)
        if q in _TYPE_OF_NAME:
            return _TYPE_OF_NAME[q]
        raise DracoFormatError(f"GGUFGemmKernel: tensor type {qt!r} / {q!r} is not a supported GGUF type "
                               f"({SUPPORTED_TYPES_TEXT})")

    def _tiled(self, tensor_info, qtype: int, payload_bytes, n_rows: int, k: int) -> torch.Tensor:
        key = (getattr(tensor_info, "name", None), getattr(tensor_info, "offset", None))
        cacheable = key != (None, None)
        if cacheable:
            with self._lock:
                t = self._cache.get(key)
                if t is not None:
                    self._cache.move_to_end(key)
                    return t
        raw = torch.frombuffer(bytearray(payload_bytes), dtype=torch.uint8).to(self.device)
        layout = G.layout_for_q6k_order(self.q6k_order) if qtype == GGML_TYPE_Q6_K else "gguf"
        t = G.repack(qtype, raw, n_rows, k, layout=layout)
        if not cacheable:
            return t
        with self._lock:
            self._cache[key] = t
            self._held += t.numel()
            while self._held > self.cache_bytes and len(self._cache) > 1:
                _, old = self._cache.popitem(last=False)
                self._held -= old.numel()
        return t

    def matmul(self, activation: np.ndarray, tensor_info, payload_bytes, **kw) -> np.ndarray:
        """``activation @ dequant(W).T`` (fp32 numpy [B, k] -> [B, n_rows])."""
        qtype = self._qtype(tensor_info)
        n_rows, k = (int(d) for d in tensor_info.shape)
        if activation.shape[-1] != k:
            raise DracoFormatError(f"activation feature size {activation.shape[-1]} != weight row length {k}")
        w = self._tiled(tensor_info, qtype, payload_bytes, n_rows, k)
        x = torch.from_numpy(np.ascontiguousarray(activation, dtype=np.float32)).to(self.device)
        return gguf_linear(x, qtype, w, n_rows, k).cpu().numpy()
