"""GGUF quantization backend and drop-in linear module (CUDA, sm_100a).

``GGUFBackend`` implements the QuantizationBackend contract
(draco/quantization/base.py:17-133) for the GGUF block formats Q4_0, Q4_1,
Q5_0, Q5_1, Q8_0, Q4_K, Q5_K and Q6_K, with the payload layout the reference decodes (draco/format/gguf.py:
_BLOCK_LAYOUTS :75-87, _dequantize :272-497):

* ``weights`` is the packed uint8 payload of a GGUF tensor, shaped
  [n_rows, k / block_size * block_bytes]; ``scales``/``zeros`` are not used
  (GGUF interleaves them inside each block) and must be None;
* ``group_size`` is the block size (32 for Q4_0 ... Q8_0, 256 for the K-quants).

``dequantize`` returns the fp32 weight bit-identical to gguf._dequantize.
``quantized_linear`` runs the fused dequant kernels: the weight is regrouped
once into the TILED device layout (cached per weight tensor, the way
GGUFReader.get_tensor caches its first-access transform, gguf.py:827-834, but
at 4.5-8.5 bits per weight instead of 32) and every call streams the packed
blocks through the tensor cores: the dequant-GEMV for decode batches, the
tcgen05 dequant-GEMM for bf16 prefill batches (see ``gguf_linear``).

``GGUFLinear`` is an nn.Module drop-in for the nn.Linear projections of the
model adapters (e.g. draco/models/llama/adapter.py:91-94, 153-155) and of the
MoE ``Expert`` (draco/models/moe/expert.py:34-36).
"""

from __future__ import annotations

import threading
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.nn as nn
from torch.utils.weak import WeakIdKeyDictionary

from dracort_b200 import _native as N
from dracort_b200 import gguf_ops as G
from dracort_b200.exceptions import DracoFormatError, KernelError
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
    SUPPORTED_TYPES_TEXT,
    TYPE_NAMES,
)
from dracort_b200.quantization.base import QuantizationBackend

_BITS = {GGML_TYPE_Q4_0: 4, GGML_TYPE_Q4_1: 4, GGML_TYPE_Q5_0: 5, GGML_TYPE_Q5_1: 5, GGML_TYPE_Q8_0: 8,
         GGML_TYPE_Q4_K: 4, GGML_TYPE_Q5_K: 5, GGML_TYPE_Q6_K: 6}

#: largest activation row count handled by one GEMV launch
GEMV_MAX_ROWS = N.GEMV_MAX_BATCH
#: rows (tokens) from which bf16/fp16 activations take the prefill GEMM
PREFILL_MIN_ROWS = 64


def infer_k(qtype: int, row_bytes: int) -> int:
    """Row length k of a packed GGUF tensor from its bytes per row."""
    bs, bb = BLOCK_LAYOUTS[qtype]
    if row_bytes % bb:
        raise DracoFormatError(f"{row_bytes} bytes per row is not a whole number of {TYPE_NAMES[qtype]} blocks ({bb} B)")
    return row_bytes // bb * bs


def _as_cuda_u8(payload, device) -> torch.Tensor:
    if isinstance(payload, np.ndarray):
        payload = torch.from_numpy(np.ascontiguousarray(payload).view(np.uint8))
    if payload.dtype != torch.uint8:
        raise DracoFormatError("GGUF payload must be uint8 bytes")
    return payload.to(device).contiguous()


class _TiledCache:
    """Packed GGUF weight tensor -> its TILED device copy.

    Entries are keyed on the weight tensor object itself (held weakly) plus its
    in-place version counter, never on its device address: a weight that is
    freed drops its entry, and a new tensor that the caching allocator places
    at the freed address is a different object, so it can never be served the
    old weight's copy.  An in-place write to the weight bumps its version and
    forces a fresh repack."""

    def __init__(self) -> None:
        self._d = WeakIdKeyDictionary()
        self._lock = threading.Lock()

    def get(self, w: torch.Tensor, qtype: int, layout: str, n_rows: int, k: int) -> torch.Tensor:
        params = (w._version, qtype, layout, n_rows, k)
        with self._lock:
            hit = self._d.get(w)
            if hit is not None and hit[0] == params:
                return hit[1]
        t = G.repack(qtype, w, n_rows, k, layout=layout)
        with self._lock:
            self._d[w] = (params, t)
        return t

    def __len__(self) -> int:
        with self._lock:
            return len(self._d)

    def clear(self) -> None:
        with self._lock:
            self._d.clear()


class GGUFBackend(QuantizationBackend):
    """QuantizationBackend for one GGUF block type on B200 (sm_100a)."""

    def __init__(self, qtype: int, q6k_order: str = Q6K_D_FIRST) -> None:
        if qtype not in _BITS:
            raise DracoFormatError(f"GGUF type {qtype} has no GPU kernel here (supported: {SUPPORTED_TYPES_TEXT})")
        if q6k_order not in (Q6K_D_FIRST, Q6K_D_LAST):
            raise ValueError(f"unknown Q6_K field order {q6k_order!r}")
        self.qtype = qtype
        self.q6k_order = q6k_order
        self.layout = G.layout_for_q6k_order(q6k_order) if qtype == GGML_TYPE_Q6_K else "gguf"
        self._cache = _TiledCache()

    # -- identity ---------------------------------------------------------
    @property
    def name(self) -> str:
        base = "gguf_" + TYPE_NAMES[self.qtype].lower()
        return base + ("_dlast" if self.qtype == GGML_TYPE_Q6_K and self.q6k_order == Q6K_D_LAST else "")

    @property
    def supported_bits(self) -> List[int]:
        return [_BITS[self.qtype]]

    @property
    def supported_schemes(self) -> List[str]:
        return ["weight_only"]

    @property
    def block_size(self) -> int:
        return BLOCK_LAYOUTS[self.qtype][0]

    # -- weights ----------------------------------------------------------
    def load_quantized_weights(self, model_path: str, target_model: nn.Module, config: Dict[str, Any],
                               device: torch.device) -> nn.Module:
        """Replace nn.Linear submodules with GGUFLinear from packed GGUF tensors.

        Two sources, in this order:
        * ``model_path`` naming a .gguf file: its quantized tensors are loaded
          onto ``device`` by dracort_b200.gguf_loader (pinned staging, on-device
          regroup) and matched to modules by their llama-family canonical names
          (``blk.N.attn_q.weight`` -> ``model.layers.N.self_attn.q_proj.weight``,
          the naming of draco/format/gguf.py:104-171) or their own names;
          ``config["q6k_order"]`` (default "d_last", llama.cpp's order) gives
          the Q6_K byte order of the file;
        * ``config["tensors"]`` mapping ``<module>.weight`` to
          ``(ggml_type, payload)`` (packed uint8 [out_features, row_bytes]).
        Tensors of another type than this backend's keep their own type.
        """
        replaced = 0
        device = torch.device(device)

        def swap(mod_name: str, new: nn.Module) -> None:
            parent_name, _, child = mod_name.rpartition(".")
            parent = target_model.get_submodule(parent_name) if parent_name else target_model
            setattr(parent, child, new)

        linears = {n: m for n, m in target_model.named_modules() if isinstance(m, nn.Linear)}
        if isinstance(model_path, str) and model_path.endswith(".gguf"):
            from dracort_b200.format.gguf_file import GGUFFile, canonical_name
            from dracort_b200.gguf_loader import load_gguf

            with GGUFFile(model_path) as gf:
                plan = {}
                for t in gf:
                    for cand in (canonical_name(t.name), t.name):
                        mod = cand[:-len(".weight")] if cand.endswith(".weight") else None
                        if t.is_quantized and mod in linears and mod not in plan:
                            plan[mod] = t
                            break
                for mod_name, t in plan.items():
                    m = linears[mod_name]
                    if (t.n_rows, t.k) != (m.out_features, m.in_features):
                        raise DracoFormatError(f"GGUF tensor '{t.name}' has shape {t.shape}, module '{mod_name}' "
                                               f"expects [{m.out_features}, {m.in_features}]")
                loaded = load_gguf(gf, device, names=[t.name for t in plan.values()],
                                   q6k_order=config.get("q6k_order", Q6K_D_LAST))
                for mod_name, t in plan.items():
                    m, dw = linears[mod_name], loaded[t.name]
                    bias = m.bias.detach().to(device) if m.bias is not None else None
                    swap(mod_name, GGUFLinear(m.in_features, m.out_features, dw.qtype, dw.tiled, bias))
                    replaced += 1
        tensors = config.get("tensors") or {}
        for mod_name, mod in linears.items():
            entry = tensors.get(f"{mod_name}.weight")
            if entry is None:
                continue
            qtype, payload = entry
            bias = mod.bias.detach() if mod.bias is not None else None
            swap(mod_name, GGUFLinear.from_packed(qtype, payload, mod.in_features, mod.out_features, bias=bias,
                                                  q6k_order=self.q6k_order, device=device))
            replaced += 1
        target_model._gguf_replaced = replaced  # type: ignore[attr-defined]
        return target_model.to(device)

    def _shape(self, weights: torch.Tensor) -> Tuple[int, int]:
        if weights.dim() != 2:
            raise DracoFormatError("GGUF weights must be a 2-D packed uint8 tensor [n_rows, row_bytes]")
        return weights.shape[0], infer_k(self.qtype, weights.shape[1])

    def dequantize(self, weights: torch.Tensor, scales: Optional[torch.Tensor] = None,
                   zeros: Optional[torch.Tensor] = None, group_size: int = 0) -> torch.Tensor:
        """Packed GGUF weight -> fp32 [n_rows, k], bit-exact with gguf._dequantize."""
        if group_size not in (0, self.block_size, 128):
            raise DracoFormatError(f"group_size {group_size} does not match the GGUF block size {self.block_size}")
        n_rows, k = self._shape(weights)
        return G.dequantize(self.qtype, weights.contiguous(), n_rows, k, layout=self.layout)

    def quantized_linear(self, input: torch.Tensor, weight: torch.Tensor, scales: Optional[torch.Tensor] = None,
                         zeros: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        """input @ dequant(weight).T + bias with the fused dequant kernels."""
        n_rows, k = self._shape(weight)
        tiled = self._cache.get(weight.contiguous(), self.qtype, self.layout, n_rows, k)
        return gguf_linear(input, self.qtype, tiled, n_rows, k, bias)

    # -- info ---------------------------------------------------------------
    def supports_gpu_kernel(self, device: torch.device) -> bool:
        if device.type != "cuda" or not torch.cuda.is_available():
            return False
        try:
            N.load()
        except KernelError:
            return False
        return torch.cuda.get_device_capability(device) == (10, 0)

    def get_kernel_info(self) -> Dict[str, Any]:
        info = {"backend": self.name, "gpu_kernel": True, "optimized": True,
                "ggml_type": self.qtype, "block": BLOCK_LAYOUTS[self.qtype], "arch": "sm_100a",
                "kernels": ["dequant", "repack", "gemv_grouped"]}
        try:
            info["library"] = N.version()
        except KernelError as e:
            info["library"] = None
            info["gpu_kernel"] = False
            info["error"] = str(e)
        return info

    def estimate_memory(self, num_params: int, bits: int = 0, group_size: int = 0) -> int:
        """Exact GGUF payload bytes: num_params / block_size * block_bytes."""
        bs, bb = BLOCK_LAYOUTS[self.qtype]
        return (num_params + bs - 1) // bs * bb


def gguf_linear(x: torch.Tensor, qtype: int, w_tiled: torch.Tensor, n_rows: int, k: int,
                bias: Optional[torch.Tensor] = None, prefill: Optional[bool] = None) -> torch.Tensor:
    """y = x @ dequant(W)^T (+ bias) over the TILED weight; x [..., k] -> [..., n_rows].

    Two kernels serve the call, as the reference's executor._linear serves both
    decode and prefill from one fp32 path (draco/runtime/cpu/executor.py:47-79):
    * decode (fp32 activations, or fewer than PREFILL_MIN_ROWS rows): the
      dequant-GEMV, fp32 throughout (1e-3 relative L2 bar);
    * prefill (bf16/fp16 activations with at least PREFILL_MIN_ROWS rows, or
      prefill=True): the tcgen05 dequant-GEMM on bf16 activations with fp32
      accumulation (the bf16 prefill bar, 5e-3 relative L2).
    Returns the input's floating dtype.
    """
    if x.shape[-1] != k:
        raise DracoFormatError(f"input feature size {x.shape[-1]} != weight row length {k}")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, k)
    m = x2.shape[0]
    if prefill is None:
        prefill = x2.dtype in (torch.bfloat16, torch.float16) and m >= PREFILL_MIN_ROWS
    if prefill and m > 0:
        ydt = x.dtype if x.dtype in (torch.bfloat16, torch.float32) else torch.float32
        y = G.gemm(qtype, w_tiled, x2, n_rows, k, out_dtype=ydt)
        if bias is not None:
            y = y + bias.to(device=y.device, dtype=y.dtype)
        out = y.reshape(*lead, n_rows)
        return out if out.dtype == x.dtype else out.to(x.dtype)
    if x2.dtype != torch.float32:
        x2 = x2.float()
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    y = torch.empty((m, n_rows), dtype=torch.float32, device=x2.device)
    b = None
    if bias is not None:
        b = bias.to(device=x2.device, dtype=torch.float32).contiguous()
    for r0 in range(0, m, GEMV_MAX_ROWS):
        r1 = min(m, r0 + GEMV_MAX_ROWS)
        G.gemv_grouped([G.GemvProblem(qtype, w_tiled, x2[r0:r1], y[r0:r1], n_rows, k, b)])
    out = y.reshape(*lead, n_rows)
    return out if x.dtype == torch.float32 else out.to(x.dtype)


class GGUFLinear(nn.Module):
    """nn.Linear drop-in holding a GGUF weight in the TILED device layout."""

    def __init__(self, in_features: int, out_features: int, qtype: int, tiled: torch.Tensor,
                 bias: Optional[torch.Tensor] = None) -> None:
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.qtype = qtype
        self.register_buffer("tiled", tiled, persistent=True)
        if bias is not None:
            self.register_buffer("bias", bias.detach().to(torch.float32).contiguous(), persistent=True)
        else:
            self.bias = None

    @classmethod
    def from_packed(cls, qtype: int, payload, in_features: int, out_features: int,
                    bias: Optional[torch.Tensor] = None, q6k_order: str = Q6K_D_FIRST,
                    device: Optional[torch.device] = None) -> "GGUFLinear":
        """Build from a packed GGUF payload ([out_features, in_features] tensor)."""
        device = torch.device(device) if device is not None else torch.device("cuda")
        raw = _as_cuda_u8(payload, device).reshape(-1)
        layout = G.layout_for_q6k_order(q6k_order) if qtype == GGML_TYPE_Q6_K else "gguf"
        tiled = G.repack(qtype, raw, out_features, in_features, layout=layout)
        b = bias.to(device) if bias is not None else None
        return cls(in_features, out_features, qtype, tiled, b)

    @classmethod
    def from_float(cls, weight: torch.Tensor, qtype: int, bias: Optional[torch.Tensor] = None,
                   device: Optional[torch.device] = None) -> "GGUFLinear":
        """Quantize a float [out, in] weight with the synthetic encoder, then pack."""
        from dracort_b200.format.quantize import encode

        w = weight.detach().float().cpu().numpy()
        packed = encode(qtype, w)
        return cls.from_packed(qtype, packed, w.shape[1], w.shape[0], bias=bias,
                               device=device or (weight.device if weight.is_cuda else None))

    def dequantized_weight(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        return G.dequantize(self.qtype, self.tiled, self.out_features, self.in_features, layout="tiled",
                            out_dtype=dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return gguf_linear(x, self.qtype, self.tiled, self.out_features, self.in_features, self.bias)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"qtype={TYPE_NAMES.get(self.qtype, self.qtype)}, bias={self.bias is not None}")
