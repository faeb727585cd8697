"""Torch-facing functions over the C ABI (libdraco_gguf.so).

Every function here takes CUDA tensors, passes raw pointers and the current
CUDA stream to the library, and raises the reference exception classes on
failure.  There is no CPU path: a CPU tensor or a missing library raises.

Functions and the reference code they replace:

* ``dequantize``       — draco/format/gguf.py:_dequantize (gguf.py:272-497)
* ``repack``           — GGUFReader.get_tensor's first-access transform
                          (gguf.py:820-834), here into the TILED device layout
* ``gemv``/``gemv_grouped`` — executor._linear (executor.py:47-79) with
                          GenericGemmKernel.matmul_f32 (generic.py:32-33)
"""

from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from dracort_b200 import _native as N
from dracort_b200.exceptions import DracoFormatError, KernelError
from dracort_b200.format.gguf_types import BLOCK_LAYOUTS, Q6K_D_FIRST, Q6K_D_LAST

LAYOUTS = {"gguf": N.LAYOUT_GGUF, "gguf_dlast": N.LAYOUT_GGUF_DLAST, "tiled": N.LAYOUT_TILED}


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this library has no CPU path)")


def _layout_id(layout: str) -> int:
    try:
        return LAYOUTS[layout]
    except KeyError:
        raise ValueError(f"unknown layout {layout!r}; expected one of {sorted(LAYOUTS)}") from None


def layout_for_q6k_order(order: str) -> str:
    return "gguf_dlast" if order == Q6K_D_LAST else "gguf"


def packed_nbytes(qtype: int, n_rows: int, k: int) -> int:
    n = N.load().draco_gguf_packed_bytes(qtype, n_rows, k)
    if n < 0:
        raise DracoFormatError(f"ggml type {qtype} with row length {k} is not a supported GGUF block tensor")
    return int(n)


def tiled_nbytes(qtype: int, n_rows: int, k: int) -> int:
    n = N.load().draco_gguf_tiled_bytes(qtype, n_rows, k)
    if n < 0:
        raise DracoFormatError(f"ggml type {qtype} with row length {k} is not a supported GGUF block tensor")
    return int(n)


def dequantize(qtype: int, blocks: torch.Tensor, n_rows: int, k: int, layout: str = "gguf",
               out_dtype: torch.dtype = torch.float32, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Dequantize a GGUF weight on the GPU into an [n_rows, k] fp32 (bit-exact) or bf16 tensor."""
    _require_cuda(blocks, "blocks")
    lib = N.load()
    if out is None:
        out = torch.empty((n_rows, k), dtype=out_dtype, device=blocks.device)
    if out_dtype == torch.float32:
        fn = lib.draco_gguf_dequant
    elif out_dtype == torch.bfloat16:
        fn = lib.draco_gguf_dequant_bf16
    else:
        raise ValueError("out_dtype must be float32 or bfloat16")
    need = tiled_nbytes(qtype, n_rows, k) if layout == "tiled" else packed_nbytes(qtype, n_rows, k)
    if blocks.numel() * blocks.element_size() < need:
        raise DracoFormatError(f"payload of {blocks.numel() * blocks.element_size()} bytes, {need} needed")
    rc = fn(qtype, _layout_id(layout), blocks.data_ptr(), out.data_ptr(), n_rows, k, _stream_ptr(blocks.device))
    N.check(rc, "dequant")
    return out


def repack(qtype: int, blocks: torch.Tensor, n_rows: int, k: int, layout: str = "gguf") -> torch.Tensor:
    """GGUF-layout payload (CUDA uint8) -> TILED payload (new CUDA uint8 tensor)."""
    _require_cuda(blocks, "blocks")
    if blocks.numel() * blocks.element_size() < packed_nbytes(qtype, n_rows, k):
        raise DracoFormatError("payload shorter than the tensor's block count")
    dst = torch.empty(tiled_nbytes(qtype, n_rows, k), dtype=torch.uint8, device=blocks.device)
    rc = N.load().draco_gguf_repack(qtype, _layout_id(layout), blocks.data_ptr(), dst.data_ptr(), n_rows, k,
                                    _stream_ptr(blocks.device))
    N.check(rc, "repack")
    return dst


# ---------------------------------------------------------------------------
# GEMV workspace: one zero-initialised buffer per (device, stream), grown on
# demand.  The kernels leave their counters at zero after every call.
# ---------------------------------------------------------------------------
_ws_lock = threading.Lock()
_workspaces: Dict[Tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(), _stream_ptr(device))
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _workspaces[key] = ws
        return ws


def reset_workspaces() -> None:
    """Drop cached workspaces (after an error their counters may be stale)."""
    with _ws_lock:
        _workspaces.clear()


def workspace_status(device: Optional[torch.device] = None) -> int:
    """Status word the GEMV kernels record (0 = ok, else a DRACO_ERR_* code).  Synchronises."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), _stream_ptr(dev))
    ws = _workspaces.get(key)
    if ws is None:
        return 0
    return int(ws[:4].view(torch.int32).item())


@dataclass
class GemvProblem:
    """One linear layer of a grouped GEMV call (host-side mirror of
    draco_gemv_problem, with its draco_gemv_input transform).

    norm_weight: x is taken through RMSNorm with this fp32 [k] weight and
        norm_eps first (the model's norm fused into the read of x);
    up: x is the gate output and this the up output ([B, k] fp32): the GEMV
        multiplies silu(x) * up (the SwiGLU product fused into the read)."""

    qtype: int
    w_tiled: torch.Tensor
    x: torch.Tensor  # [B, k] fp32 CUDA
    y: torch.Tensor  # [B, n_rows] fp32 CUDA
    n_rows: int
    k: int
    bias: Optional[torch.Tensor] = None
    norm_weight: Optional[torch.Tensor] = None
    norm_eps: float = 1e-6
    up: Optional[torch.Tensor] = None
    accumulate: bool = False  # y += result (a residual add folded into the GEMV)


def _to_struct(p: GemvProblem) -> N.GemvProblem:
    for t, nm in ((p.w_tiled, "w_tiled"), (p.x, "x"), (p.y, "y")):
        _require_cuda(t, nm)
    if p.x.dtype != torch.float32 or p.y.dtype != torch.float32:
        raise ValueError("gemv: x and y must be float32")
    if p.x.dim() != 2 or p.y.dim() != 2 or p.x.stride(1) != 1 or p.y.stride(1) != 1:
        raise ValueError("gemv: x and y must be 2-D with unit inner stride")
    if p.x.shape[1] != p.k or p.y.shape[1] != p.n_rows or p.x.shape[0] != p.y.shape[0]:
        raise DracoFormatError(
            f"gemv: x {tuple(p.x.shape)} / y {tuple(p.y.shape)} do not match weight [{p.n_rows}, {p.k}]")
    if p.bias is not None:
        _require_cuda(p.bias, "bias")
        if p.bias.dtype != torch.float32 or p.bias.numel() != p.n_rows or not p.bias.is_contiguous():
            raise ValueError("gemv: bias must be a contiguous float32 [n_rows] tensor")
    s = N.GemvProblem()
    s.qtype = p.qtype
    s.w = p.w_tiled.data_ptr()
    s.x = p.x.data_ptr()
    s.y = p.y.data_ptr()
    s.bias = p.bias.data_ptr() if p.bias is not None else None
    s.n_rows = p.n_rows
    s.k = p.k
    s.ldx = p.x.stride(0)
    s.ldy = p.y.stride(0)
    s.flags = N.GEMV_ACCUMULATE if p.accumulate else 0
    return s


def _input_struct(p: GemvProblem) -> N.GemvInput:
    s = N.GemvInput()
    s.mode, s.eps, s.aux, s.ldaux = N.INPUT_PLAIN, 0.0, None, 0
    if p.norm_weight is not None and p.up is not None:
        raise ValueError("gemv: a problem takes either an RMSNorm or a SwiGLU input, not both")
    if p.norm_weight is not None:
        w = p.norm_weight
        _require_cuda(w, "norm_weight")
        if w.dtype != torch.float32 or w.numel() != p.k or not w.is_contiguous():
            raise ValueError("gemv: norm_weight must be a contiguous float32 [k] tensor")
        s.mode, s.eps, s.aux = N.INPUT_RMSNORM, float(p.norm_eps), w.data_ptr()
    elif p.up is not None:
        u = p.up
        _require_cuda(u, "up")
        if u.dtype != torch.float32 or u.shape != p.x.shape or u.stride(1) != 1:
            raise ValueError("gemv: up must be a float32 tensor shaped like x with unit inner stride")
        s.mode, s.aux, s.ldaux = N.INPUT_SWIGLU, u.data_ptr(), u.stride(0)
    return s


def _inputs(problems: Sequence[GemvProblem]):
    """ctypes array of the problems' input transforms, or None when all are plain."""
    if all(p.norm_weight is None and p.up is None for p in problems):
        return None
    return (N.GemvInput * len(problems))(*[_input_struct(p) for p in problems])


def gemv_grouped(problems: Sequence[GemvProblem]) -> None:
    """y_i = x_i @ dequant(W_i)^T (+ bias_i) for up to 8 weights in one launch.

    All x_i share one batch size (1..32).  Outputs are written in place.
    """
    if not problems:
        return
    if len(problems) > N.GEMV_MAX_PROBLEMS:
        for i in range(0, len(problems), N.GEMV_MAX_PROBLEMS):
            gemv_grouped(problems[i:i + N.GEMV_MAX_PROBLEMS])
        return
    batch = problems[0].x.shape[0]
    if any(p.x.shape[0] != batch for p in problems):
        raise ValueError("gemv_grouped: all problems must share one batch size")
    if batch == 0:
        return
    if batch > N.GEMV_MAX_BATCH:
        for b0 in range(0, batch, N.GEMV_MAX_BATCH):
            sub = [GemvProblem(p.qtype, p.w_tiled, p.x[b0:b0 + N.GEMV_MAX_BATCH], p.y[b0:b0 + N.GEMV_MAX_BATCH],
                               p.n_rows, p.k, p.bias, p.norm_weight, p.norm_eps,
                               None if p.up is None else p.up[b0:b0 + N.GEMV_MAX_BATCH], p.accumulate)
                   for p in problems]
            gemv_grouped(sub)
        return
    lib = N.load()
    arr = (N.GemvProblem * len(problems))(*[_to_struct(p) for p in problems])
    need = lib.draco_gguf_gemv_workspace_bytes(arr, len(problems), batch)
    if need == 0:
        N.check(N.DRACO_ERR_ARG, "gemv workspace query failed")
    dev = problems[0].x.device
    ws = _workspace(dev, int(need))
    ins = _inputs(problems)
    if ins is None:
        rc = lib.draco_gguf_gemv_grouped(arr, len(problems), batch, ws.data_ptr(), ws.numel(), _stream_ptr(dev))
    else:
        rc = lib.draco_gguf_gemv_grouped_ex(arr, ins, len(problems), batch, ws.data_ptr(), ws.numel(),
                                            _stream_ptr(dev))
    N.check(rc, "gemv")


class GemvPlan:
    """A fixed grouped-GEMV call (same buffers every time), validated once.

    ``run()`` enqueues the prep + GEMV kernels on the current stream with no
    per-call Python validation, so decode loops and CUDA-graph capture pay
    only the C launch cost.  The problems' tensors must stay alive and keep
    their storage while the plan is used.
    """

    def __init__(self, problems: Sequence[GemvProblem]) -> None:
        if not problems or len(problems) > N.GEMV_MAX_PROBLEMS:
            raise ValueError(f"GemvPlan takes 1..{N.GEMV_MAX_PROBLEMS} problems")
        self.problems = list(problems)
        self.batch = problems[0].x.shape[0]
        if any(p.x.shape[0] != self.batch for p in problems) or not 1 <= self.batch <= N.GEMV_MAX_BATCH:
            raise ValueError("GemvPlan: all problems need one batch size in 1..32")
        self._lib = N.load()
        self._arr = (N.GemvProblem * len(problems))(*[_to_struct(p) for p in problems])
        self._ins = _inputs(problems)
        need = self._lib.draco_gguf_gemv_workspace_bytes(self._arr, len(problems), self.batch)
        if need == 0:
            N.check(N.DRACO_ERR_ARG, "gemv workspace query failed")
        self.device = problems[0].x.device
        self.workspace = torch.zeros(int(need), dtype=torch.uint8, device=self.device)
        self.bytes_weights = sum(tiled_nbytes(p.qtype, p.n_rows, p.k) for p in problems)
        with torch.cuda.device(self.device):
            #: kernel launches one run() makes (activation conversion, GEMV, split-row-group sums)
            self.launches = int(self._lib.draco_gguf_gemv_launch_count(self._arr, len(problems), self.batch))

    def run(self) -> None:
        if self._ins is None:
            rc = self._lib.draco_gguf_gemv_grouped(self._arr, len(self.problems), self.batch,
                                                   self.workspace.data_ptr(), self.workspace.numel(),
                                                   _stream_ptr(self.device))
        else:
            rc = self._lib.draco_gguf_gemv_grouped_ex(self._arr, self._ins, len(self.problems), self.batch,
                                                      self.workspace.data_ptr(), self.workspace.numel(),
                                                      _stream_ptr(self.device))
        if rc:
            N.check(rc, "gemv")

    def status(self) -> int:
        """Kernel-recorded status word (0 = ok).  Synchronises.  A nonzero status
        means a launch aborted (its outputs are invalid) and left the
        workspace's arrival counters stale; the workspace is zeroed here so
        that the plan can run again."""
        st = int(self.workspace[:4].view(torch.int32).item())
        if st:
            self.workspace.zero_()
        return st


def gemv(qtype: int, w_tiled: torch.Tensor, x: torch.Tensor, n_rows: int, k: int,
         bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ dequant(W)^T (+ bias); x [B, k] fp32 CUDA -> y [B, n_rows] fp32."""
    squeeze = x.dim() == 1
    x2 = x.reshape(1, -1) if squeeze else x
    if x2.dtype != torch.float32:
        x2 = x2.float()
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    y = out if out is not None else torch.empty((x2.shape[0], n_rows), dtype=torch.float32, device=x2.device)
    gemv_grouped([GemvProblem(qtype, w_tiled, x2, y, n_rows, k, bias)])
    return y.reshape(-1) if squeeze else y


# ---------------------------------------------------------------------------
# prefill dequant-GEMM (tcgen05)
# ---------------------------------------------------------------------------
@dataclass
class GemmProblem:
    """One weight of a grouped prefill GEMM: y = x @ dequant(W)^T (x bf16 [m, k])."""

    qtype: int
    w_tiled: torch.Tensor
    x: torch.Tensor  # [m, k] bf16 CUDA
    y: torch.Tensor  # [m, n_rows] bf16 or fp32 CUDA
    n_rows: int
    k: int


def _gemm_struct(p: GemmProblem) -> N.GemmProblem:
    for t, nm in ((p.w_tiled, "w_tiled"), (p.x, "x"), (p.y, "y")):
        _require_cuda(t, nm)
    if p.x.dtype != torch.bfloat16:
        raise ValueError("gemm: x must be bfloat16")
    if p.y.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("gemm: y must be bfloat16 or float32")
    if p.x.dim() != 2 or p.y.dim() != 2 or p.x.stride(1) != 1 or p.y.stride(1) != 1:
        raise ValueError("gemm: x and y must be 2-D with unit inner stride")
    if p.x.shape[1] != p.k or p.y.shape[1] != p.n_rows or p.x.shape[0] != p.y.shape[0]:
        raise DracoFormatError(
            f"gemm: x {tuple(p.x.shape)} / y {tuple(p.y.shape)} do not match weight [{p.n_rows}, {p.k}]")
    s = N.GemmProblem()
    s.qtype = p.qtype
    s.ydtype = N.DTYPE_BF16 if p.y.dtype == torch.bfloat16 else N.DTYPE_F32
    s.w, s.x, s.y = p.w_tiled.data_ptr(), p.x.data_ptr(), p.y.data_ptr()
    s.m, s.n_rows, s.k = p.x.shape[0], p.n_rows, p.k
    s.ldx, s.ldy = p.x.stride(0), p.y.stride(0)
    return s


def gemm_grouped(problems: Sequence[GemmProblem], status: Optional[torch.Tensor] = None) -> None:
    """Y_i = X_i @ dequant(W_i)^T for up to 16 weights in one tcgen05 launch."""
    if not problems:
        return
    if len(problems) > N.GEMM_MAX_PROBLEMS:
        for i in range(0, len(problems), N.GEMM_MAX_PROBLEMS):
            gemm_grouped(problems[i:i + N.GEMM_MAX_PROBLEMS], status)
        return
    lib = N.load()
    arr = (N.GemmProblem * len(problems))(*[_gemm_struct(p) for p in problems])
    dev = problems[0].x.device
    st = status.data_ptr() if status is not None else None
    N.check(lib.draco_gguf_gemm(arr, len(problems), st, _stream_ptr(dev)), "gemm")


def gemm_grouped_unchecked(entries: Sequence[tuple], device: torch.device,
                           status: Optional[torch.Tensor] = None) -> None:
    """gemm_grouped for internal callers whose tensors are already known valid
    (CUDA, bf16 x, contiguous rows): entries are (qtype, w_tiled, x, y, n_rows, k),
    at most GEMM_MAX_PROBLEMS; only the C ABI's own checks run."""
    if not entries:
        return
    lib = N.load()
    arr = (N.GemmProblem * len(entries))()
    for s, (qt, w, x, y, n, k) in zip(arr, entries):
        s.qtype = qt
        s.ydtype = N.DTYPE_BF16 if y.dtype == torch.bfloat16 else N.DTYPE_F32
        s.w, s.x, s.y = w.data_ptr(), x.data_ptr(), y.data_ptr()
        s.m, s.n_rows, s.k = x.shape[0], n, k
        s.ldx, s.ldy = x.stride(0), y.stride(0)
    st = status.data_ptr() if status is not None else None
    N.check(lib.draco_gguf_gemm(arr, len(entries), st, _stream_ptr(device)), "gemm")


def gemm_grouped_raw(entries: Sequence[tuple], device: torch.device, status: Optional[torch.Tensor] = None) -> None:
    """gemm_grouped on raw device pointers for internal callers that slice one
    buffer into many problems (the MoE experts' row blocks) and would otherwise
    pay for a tensor view per problem: entries are (qtype, w_ptr, x_ptr, y_ptr,
    m, n_rows, k, ldx, ldy, ydtype) with ydtype N.DTYPE_BF16 or N.DTYPE_F32, at
    most GEMM_MAX_PROBLEMS; only the C ABI's own checks run."""
    if not entries:
        return
    arr = (N.GemmProblem * len(entries))()
    for s, (qt, w, x, y, m, n, k, ldx, ldy, ydt) in zip(arr, entries):
        s.qtype, s.ydtype = qt, ydt
        s.w, s.x, s.y = w, x, y
        s.m, s.n_rows, s.k = m, n, k
        s.ldx, s.ldy = ldx, ldy
    st = status.data_ptr() if status is not None else None
    N.check(N.load().draco_gguf_gemm(arr, len(entries), st, _stream_ptr(device)), "gemm")


def gemm_rows_raw(entries: Sequence[tuple], rows: torch.Tensor, device: torch.device,
                  status: Optional[torch.Tensor] = None) -> None:
    """gemm_grouped_raw whose problems' token counts live on the device: each
    entry's m is the capacity of its x / y blocks, rows (CUDA int32, one per
    entry, in entry order) the tokens present (draco_gguf_gemm_rows).  No host
    synchronisation; rows of y past the count up to the next 32 may be
    written with values of no meaning."""
    if not entries:
        return
    if rows.dtype != torch.int32 or not rows.is_cuda or rows.numel() < len(entries) or not rows.is_contiguous():
        raise ValueError("gemm_rows: rows must be a contiguous CUDA int32 tensor with one count per problem")
    arr = (N.GemmProblem * len(entries))()
    for s, (qt, w, x, y, m, n, k, ldx, ldy, ydt) in zip(arr, entries):
        s.qtype, s.ydtype = qt, ydt
        s.w, s.x, s.y = w, x, y
        s.m, s.n_rows, s.k = m, n, k
        s.ldx, s.ldy = ldx, ldy
    st = status.data_ptr() if status is not None else None
    N.check(N.load().draco_gguf_gemm_rows(arr, len(entries), rows.data_ptr(), st, _stream_ptr(device)), "gemm_rows")


def swiglu_bf16_rows(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
    """out[g, r] = bf16(silu(gate[g, r]) * up[g, r]) for r < rows[g] over
    [groups, cap_rows, width] bf16 blocks; rows is a CUDA int32 [groups]
    (draco_swiglu_bf16_rows).  out may be gate."""
    for t, nm in ((gate, "gate"), (up, "up"), (out, "out")):
        _require_cuda(t, nm)
        if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.dim() != 3:
            raise ValueError(f"swiglu_rows: {nm} must be a contiguous [groups, rows, width] bfloat16 CUDA tensor")
    if gate.shape != up.shape or gate.shape != out.shape:
        raise DracoFormatError(f"swiglu_rows: shapes {tuple(gate.shape)}, {tuple(up.shape)}, {tuple(out.shape)} differ")
    if rows.dtype != torch.int32 or not rows.is_cuda or rows.numel() != gate.shape[0]:
        raise ValueError("swiglu_rows: rows must be a CUDA int32 tensor with one count per group")
    g, c, w = gate.shape
    N.check(N.load().draco_swiglu_bf16_rows(gate.data_ptr(), up.data_ptr(), out.data_ptr(), g, c, w,
                                            rows.data_ptr(), _stream_ptr(gate.device)), "swiglu_rows")
    return out


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
             out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x * rsqrt(mean(x^2, -1) + eps) * weight on the GPU (draco_rmsnorm): x
    fp32 or bf16 CUDA, contiguous, last dim k; weight [k] (cast to fp32)."""
    _require_cuda(x, "x")
    if x.dtype not in (torch.float32, torch.bfloat16) or not x.is_contiguous():
        raise ValueError("rms_norm: x must be a contiguous float32 or bfloat16 CUDA tensor")
    k = x.shape[-1]
    w = weight.to(device=x.device, dtype=torch.float32).contiguous()
    if w.numel() != k:
        raise DracoFormatError(f"rms_norm: weight of {w.numel()} values for rows of {k}")
    out = out if out is not None else torch.empty_like(x)
    dt = N.DTYPE_BF16 if x.dtype == torch.bfloat16 else N.DTYPE_F32
    N.check(N.load().draco_rmsnorm(x.data_ptr(), w.data_ptr(), out.data_ptr(), x.numel() // max(k, 1), k, float(eps),
                                   dt, _stream_ptr(x.device)), "rms_norm")
    return out


def swiglu_bf16(gate: torch.Tensor, up: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16(silu(gate) * up) in fp32 with one rounding (C ABI draco_swiglu_bf16)."""
    for t, nm in ((gate, "gate"), (up, "up")):
        _require_cuda(t, nm)
        if t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise ValueError(f"swiglu: {nm} must be a contiguous bfloat16 CUDA tensor")
    if gate.shape != up.shape:
        raise DracoFormatError(f"swiglu: gate {tuple(gate.shape)} and up {tuple(up.shape)} differ")
    out = out if out is not None else torch.empty_like(gate)
    N.check(N.load().draco_swiglu_bf16(gate.data_ptr(), up.data_ptr(), out.data_ptr(), gate.numel(),
                                       _stream_ptr(gate.device)), "swiglu")
    return out


def swiglu(gate: torch.Tensor, up: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """silu(gate) * up on the GPU for bf16 (one rounding, draco_swiglu_bf16) or
    fp32 (draco_swiglu_f32) contiguous CUDA tensors of one shape; `out` may be
    `gate`.  Pointers must be 16-byte aligned (fresh allocations are)."""
    if gate.dtype == torch.bfloat16:
        return swiglu_bf16(gate, up, out)
    for t, nm in ((gate, "gate"), (up, "up")):
        _require_cuda(t, nm)
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError(f"swiglu: {nm} must be a contiguous float32 or bfloat16 CUDA tensor")
    if gate.shape != up.shape:
        raise DracoFormatError(f"swiglu: gate {tuple(gate.shape)} and up {tuple(up.shape)} differ")
    out = out if out is not None else torch.empty_like(gate)
    N.check(N.load().draco_swiglu_f32(gate.data_ptr(), up.data_ptr(), out.data_ptr(), gate.numel(),
                                      _stream_ptr(gate.device)), "swiglu")
    return out


def gemm(qtype: int, w_tiled: torch.Tensor, x: torch.Tensor, n_rows: int, k: int,
         out_dtype: torch.dtype = torch.bfloat16, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Y = X @ dequant(W)^T with X cast to bf16; returns [m, n_rows] of out_dtype."""
    x2 = x.reshape(-1, k)
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    y = out if out is not None else torch.empty((x2.shape[0], n_rows), dtype=out_dtype, device=x2.device)
    gemm_grouped([GemmProblem(qtype, w_tiled, x2, y, n_rows, k)])
    return y
