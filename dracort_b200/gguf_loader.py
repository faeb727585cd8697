"""GGUF file -> GPU: packed weights staged through pinned memory and regrouped
into the TILED layout on the device.

Replaces the reference's first-access path for GGUF weights,
GGUFReader.get_tensor (draco/format/gguf.py:820-834), which dequantizes every
tensor on the host into an fp32 cache (4 bytes per weight; ~26 GB for a
Llama-7B) before the executor's ``_linear`` multiplies with it.  Here the
packed bytes (4.5-8.5 bits per weight) are the resident form:

1. the payload (or this rank's shard of it) is copied from the memory-mapped
   file into one of two pinned staging buffers, whole rows at a time;
2. a cudaMemcpyAsync moves the staging buffer into a device buffer on a
   loader stream, while the host fills the other staging buffer;
3. ``draco_gguf_repack`` regroups the GGUF blocks into the TILED layout the
   GEMV / GEMM kernels read (bytes moved, never changed).

Tensor-parallel shards are cut from the packed rows with the rules of
``dracort_b200.parallel.tp``: a column shard is a contiguous row range (one
contiguous byte range of the file), a row shard a super-block range of every
row (gathered row by row into the staging buffer).

Q6_K byte order: llama.cpp writes the fp16 ``d`` of a Q6_K block last, the
reference decodes it first (gguf.py:470-474).  ``q6k_order`` says which one a
file uses; "d_last" (real .gguf files) is the default.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Iterable, Optional, Tuple, Union

import numpy as np
import torch

from dracort_b200 import gguf_ops as G
from dracort_b200.exceptions import DracoFormatError
from dracort_b200.format.gguf_file import GGUFFile, GGUFTensor
from dracort_b200.format.gguf_types import (
    BLOCK_LAYOUTS,
    GGML_TYPE_BF16,
    GGML_TYPE_F16,
    GGML_TYPE_F32,
    GGML_TYPE_Q6_K,
    Q6K_D_FIRST,
    Q6K_D_LAST,
)
from dracort_b200.parallel.tp import SUPER_BLOCK, even_split

_DENSE_TORCH = {GGML_TYPE_F32: torch.float32, GGML_TYPE_F16: torch.float16, GGML_TYPE_BF16: torch.bfloat16}


@dataclass(frozen=True)
class Shard:
    """This rank's part of a weight: 'col' (output rows, dim 0) or 'row'
    (reduction super-blocks, dim 1) of `world` parts."""

    kind: str
    rank: int
    world: int

    def __post_init__(self) -> None:
        if self.kind not in ("col", "row") or not 0 <= self.rank < self.world:
            raise ValueError(f"invalid shard {self}")


@dataclass
class DeviceWeight:
    """A quantized weight resident on the GPU in the TILED layout, ready for
    gguf_ops.gemv / gemm / GemvProblem.  (r0, r1) and (k0, k1) are the row and
    reduction ranges of the full tensor this shard holds."""

    name: str
    qtype: int
    tiled: torch.Tensor
    n_rows: int
    k: int
    r0: int
    r1: int
    k0: int
    k1: int


class _Stager:
    """Two pinned staging buffers feeding device buffers through a copy stream.

    Host fills of one staging buffer overlap the device copy of the other.
    Device buffers are allocated, and repacked, on the caller's current stream,
    which waits for the copy stream before it reads them."""

    def __init__(self, device: torch.device, chunk_bytes: int) -> None:
        self.device = device
        self.chunk = chunk_bytes
        self.pinned = [torch.empty(chunk_bytes, dtype=torch.uint8).pin_memory() for _ in range(2)]
        self.done = [None, None]  # event after each staging buffer's last copy
        self.turn = 0
        self.stream = torch.cuda.Stream(device=device)
        self.main = torch.cuda.current_stream(device)
        self.land = torch.empty(0, dtype=torch.uint8, device=device)

    def landing(self, nbytes: int) -> torch.Tensor:
        """A device buffer of nbytes that no queued work still reads."""
        if self.land.numel() < nbytes:
            self.land = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        self.stream.wait_stream(self.main)  # the previous repack has read it
        return self.land[:nbytes]

    def put(self, dst: torch.Tensor, fill) -> None:
        """fill(host_view) writes len(dst) bytes into a staging buffer, which is
        then copied into dst (device) on the copy stream."""
        n = dst.numel()
        if n > self.chunk:
            raise ValueError("staging chunk too small")
        i = self.turn
        self.turn ^= 1
        if self.done[i] is not None:
            self.done[i].synchronize()  # its previous copy has left the buffer
        host = self.pinned[i][:n]
        fill(host.numpy())
        with torch.cuda.stream(self.stream):
            dst.copy_(host, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        self.done[i] = ev

    def landed(self) -> None:
        """The current stream waits for every copy issued so far."""
        self.main.wait_stream(self.stream)


def _shard_ranges(t: GGUFTensor, shard: Optional[Shard]) -> Tuple[int, int, int, int]:
    n, k = t.n_rows, t.k
    if shard is None or shard.world == 1:
        return 0, n, 0, k
    if shard.kind == "col":
        align = 16 if n % 16 == 0 else 1
        r0, r1 = even_split(n, shard.world, align)[shard.rank]
        return r0, r1, 0, k
    if k % SUPER_BLOCK:
        raise DracoFormatError(f"row-parallel shard of '{t.name}' needs k % {SUPER_BLOCK} == 0, got {k}")
    k0, k1 = even_split(k, shard.world, SUPER_BLOCK)[shard.rank]
    if k1 == k0:
        raise DracoFormatError(f"row-parallel shard {shard.rank} of {shard.world} of '{t.name}' holds no "
                               f"super-block (k = {k})")
    return 0, n, k0, k1


def _load_quantized(gf: GGUFFile, t: GGUFTensor, st: _Stager, shard: Optional[Shard], q6k_order: str) -> DeviceWeight:
    bs, bb = BLOCK_LAYOUTS[t.ggml_type]
    n, k = t.n_rows, t.k
    row_bytes = k // bs * bb
    r0, r1, k0, k1 = _shard_ranges(t, shard)
    c0, c1 = k0 // bs * bb, k1 // bs * bb  # byte columns of the shard in every row
    width = c1 - c0
    rows = gf.payload(t.name).reshape(n, row_bytes)
    land = st.landing((r1 - r0) * width)
    step = max(1, st.chunk // width)
    for a in range(r0, r1, step):
        b = min(r1, a + step)
        src = rows[a:b, c0:c1]

        def fill(h, src=src):
            np.copyto(h.reshape(src.shape), src)

        st.put(land[(a - r0) * width:(b - r0) * width], fill)
    layout = "gguf"
    if t.ggml_type == GGML_TYPE_Q6_K and q6k_order == Q6K_D_LAST:
        layout = "gguf_dlast"
    st.landed()
    tiled = G.repack(t.ggml_type, land, r1 - r0, k1 - k0, layout=layout)
    return DeviceWeight(t.name, t.ggml_type, tiled, r1 - r0, k1 - k0, r0, r1, k0, k1)


def _load_dense(gf: GGUFFile, t: GGUFTensor, st: _Stager) -> torch.Tensor:
    dt = _DENSE_TORCH.get(t.ggml_type)
    if dt is None:
        raise DracoFormatError(f"tensor '{t.name}' has ggml type {t.ggml_type}; dense loads support F32/F16/BF16")
    out = torch.empty(t.shape, dtype=dt, device=st.device)
    st.stream.wait_stream(st.main)  # the allocation is ordered on the current stream
    raw = out.view(-1).view(torch.uint8)
    src = gf.payload(t.name)
    for a in range(0, t.nbytes, st.chunk):
        b = min(t.nbytes, a + st.chunk)

        def fill(h, a=a, b=b):
            np.copyto(h, src[a:b])

        st.put(raw[a:b], fill)
    st.landed()
    return out


def load_gguf(source: Union[str, GGUFFile], device: Union[str, torch.device] = "cuda",
              names: Optional[Iterable[str]] = None, shards: Optional[Dict[str, Shard]] = None,
              q6k_order: str = Q6K_D_LAST, dense: bool = True,
              chunk_bytes: int = 64 << 20) -> Dict[str, Union[DeviceWeight, torch.Tensor]]:
    """Load tensors of a GGUF file onto one GPU.

    names  : tensors to load (default: all); quantized ones (Q4_0, Q4_1, Q5_0, Q5_1,
             Q8_0, Q4_K, Q5_K, Q6_K)
             become DeviceWeight (TILED layout), dense ones (F32/F16/BF16)
             torch tensors of their own dtype (skipped when dense=False).
    shards : per-name Shard for tensor-parallel ranks (others load whole).
    Returns {name: ...}; the call returns once every copy and repack is done.
    """
    if q6k_order not in (Q6K_D_FIRST, Q6K_D_LAST):
        raise ValueError(f"unknown Q6_K order {q6k_order!r}")
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("load_gguf places weights on a CUDA device (this library has no CPU path)")
    own = not isinstance(source, GGUFFile)
    gf = GGUFFile(source) if own else source
    try:
        wanted = list(gf.tensors) if names is None else list(names)
        st = _Stager(device, chunk_bytes)
        out: Dict[str, Union[DeviceWeight, torch.Tensor]] = {}
        for name in wanted:
            t = gf.tensor(name)
            if t.is_quantized:
                out[name] = _load_quantized(gf, t, st, (shards or {}).get(name), q6k_order)
            elif dense:
                if shards and name in shards:
                    raise DracoFormatError(f"dense tensor '{name}' cannot be sharded by the loader")
                out[name] = _load_dense(gf, t, st)
            elif t.nbytes < 0:
                raise DracoFormatError(f"tensor '{name}' has ggml type {t.ggml_type}, which has no GPU kernel here")
        torch.cuda.current_stream(device).synchronize()
        return out
    finally:
        if own:
            gf.close()
