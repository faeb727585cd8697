"""Tensor parallelism for GGUF linear layers — mirror of draco/parallel/tp.py.

The reference splits dense weights with ``split_tensor`` (tp.py:44-73), pads
non-divisible dims (invalid for packed blocks) and leaves the all-reduce as a
comment (tp.py:182-183).  Here the shards are cut from the packed GGUF payload
and the collectives are real (torch.distributed; NCCL on GPUs, gloo on CPU):

* column-parallel (q/k/v/gate/up, dim 0): each rank holds a contiguous range of
  output rows — packed rows are independent, so any row split is valid; the
  outputs are concatenated with an all-gather;
* row-parallel (o/down, dim 1): each rank holds a contiguous range of 256-element
  super-blocks of every row (K = 11008 has 43 super-blocks, so the ranges are
  uneven: 22/21 at 2 ranks, 11/11/11/10 at 4, 6/6/6/5/5/5/5/5 at 8); each rank
  multiplies its slice of x and the partial outputs are summed with an
  all-reduce.

``partition_parameters`` keeps the reference's name rules (tp.py:189-214).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.nn as nn

from dracort_b200.format.gguf_types import BLOCK_LAYOUTS

SUPER_BLOCK = 256


@dataclass
class TensorParallelConfig:
    """Same fields as draco.parallel.tp.TensorParallelConfig (tp.py:27-41)."""

    world_size: int = 1
    rank: int = 0
    local_rank: int = 0
    device: str = "cpu"

    @property
    def is_parallel(self) -> bool:
        return self.world_size > 1

    @property
    def is_main(self) -> bool:
        return self.rank == 0


def even_split(total: int, parts: int, align: int = 1) -> List[Tuple[int, int]]:
    """Contiguous [start, end) ranges of `total` units in multiples of `align`,
    sizes differing by at most one align unit (first ranges get the extra)."""
    if total % align:
        raise ValueError(f"{total} is not a multiple of {align}")
    units = total // align
    base, extra = divmod(units, parts)
    out, s = [], 0
    for r in range(parts):
        n = base + (1 if r < extra else 0)
        out.append((s * align, (s + n) * align))
        s += n
    return out


def shard_rows(packed: np.ndarray, qtype: int, n_rows: int, k: int, rank: int, world: int,
               align: int = 16) -> Tuple[np.ndarray, int, int]:
    """Column-parallel shard: rows [r0, r1) of a packed GGUF weight [n_rows, row_bytes]."""
    if n_rows % align:
        align = 1
    r0, r1 = even_split(n_rows, world, align)[rank]
    return np.ascontiguousarray(packed.reshape(n_rows, -1)[r0:r1]), r0, r1


def shard_k(packed: np.ndarray, qtype: int, n_rows: int, k: int, rank: int,
            world: int) -> Tuple[np.ndarray, int, int]:
    """Row-parallel shard: elements [k0, k1) of every row, on super-block boundaries."""
    bs, bb = BLOCK_LAYOUTS[qtype]
    if k % SUPER_BLOCK:
        raise ValueError(f"row-parallel sharding needs k % {SUPER_BLOCK} == 0, got {k}")
    k0, k1 = even_split(k, world, SUPER_BLOCK)[rank]
    rows = packed.reshape(n_rows, -1)
    return np.ascontiguousarray(rows[:, (k0 // bs) * bb:(k1 // bs) * bb]), k0, k1


def split_tensor(packed, qtype: int, n_rows: int, k: int, world_size: int, dim: int = 0):
    """All ranks' shards of a packed GGUF weight (dim 0: rows, dim 1: super-blocks)."""
    fn = shard_rows if dim == 0 else shard_k
    return [fn(packed, qtype, n_rows, k, r, world_size)[0] for r in range(world_size)]


def merge_tensor(shards: Sequence[torch.Tensor], dim: int = 0) -> torch.Tensor:
    """Concatenate dense shards back (tp.py:76-92)."""
    return shards[0] if len(shards) == 1 else torch.cat(list(shards), dim=dim)


def partition_parameters(model: nn.Module, config: TensorParallelConfig) -> Dict[str, Tuple[str, int]]:
    """Parameter partition plan with the reference's rules (tp.py:189-214)."""
    plan = {}
    named = list(model.named_parameters()) + [(n, b) for n, b in model.named_buffers() if n.endswith("tiled")]
    for name, p in named:
        if name.endswith("tiled") or p.ndim == 2:
            if any(s in name for s in ("out_proj", "o_proj", "down_proj", "dense")):
                plan[name] = ("row", 1)
            else:
                plan[name] = ("column", 0)
        else:
            plan[name] = ("replicate", -1)
    return plan


def _default_group():
    import torch.distributed as dist

    return dist.group.WORLD if dist.is_available() and dist.is_initialized() else None


class _GGUFShardLinear(nn.Module):
    """Local GGUF shard plus the hook that computes it (the GPU GEMV by default)."""

    def __init__(self, qtype: int, packed_shard: np.ndarray, n_rows: int, k: int, device,
                 local_matmul: Optional[Callable] = None) -> None:
        super().__init__()
        self.qtype, self.n_local, self.k_local = qtype, n_rows, k
        self.local_matmul = local_matmul
        if local_matmul is None:
            from dracort_b200 import gguf_ops as G

            raw = torch.from_numpy(np.ascontiguousarray(packed_shard).reshape(-1)).to(device)
            self.register_buffer("tiled", G.repack(qtype, raw, n_rows, k), persistent=True)
        else:
            self.packed = packed_shard

    def local(self, x: torch.Tensor) -> torch.Tensor:
        if self.local_matmul is not None:
            return self.local_matmul(x, self.qtype, self.packed, self.n_local, self.k_local)
        from dracort_b200.quantization.gguf import gguf_linear

        return gguf_linear(x, self.qtype, self.tiled, self.n_local, self.k_local)


class ColumnParallelGGUFLinear(_GGUFShardLinear):
    """Output rows split across ranks; forward returns the full output on every rank."""

    def __init__(self, qtype: int, packed: np.ndarray, in_features: int, out_features: int,
                 config: TensorParallelConfig, bias: Optional[torch.Tensor] = None, group=None,
                 local_matmul: Optional[Callable] = None) -> None:
        shard, r0, r1 = shard_rows(packed, qtype, out_features, in_features, config.rank, config.world_size)
        super().__init__(qtype, shard, r1 - r0, in_features, config.device, local_matmul)
        self.in_features, self.out_features, self.config = in_features, out_features, config
        self.r0, self.r1 = r0, r1
        self.group = group
        self.bias = None if bias is None else bias[r0:r1].float()
        self.ranges = even_split(out_features, config.world_size, 16 if out_features % 16 == 0 else 1)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.local(x)
        if self.bias is not None:
            y = y + self.bias.to(y.device)
        if not self.config.is_parallel:
            return y
        import torch.distributed as dist

        lead = y.shape[:-1]
        y2 = y.reshape(-1, y.shape[-1]).contiguous()
        parts = [torch.empty((y2.shape[0], b - a), dtype=y2.dtype, device=y2.device) for a, b in self.ranges]
        dist.all_gather(parts, y2, group=self.group or _default_group())
        return torch.cat(parts, dim=1).reshape(*lead, self.out_features)


class RowParallelGGUFLinear(_GGUFShardLinear):
    """Reduction dim split on super-block boundaries; outputs summed by all-reduce."""

    def __init__(self, qtype: int, packed: np.ndarray, in_features: int, out_features: int,
                 config: TensorParallelConfig, bias: Optional[torch.Tensor] = None, group=None,
                 local_matmul: Optional[Callable] = None) -> None:
        shard, k0, k1 = shard_k(packed, qtype, out_features, in_features, config.rank, config.world_size)
        super().__init__(qtype, shard, out_features, k1 - k0, config.device, local_matmul)
        self.in_features, self.out_features, self.config = in_features, out_features, config
        self.k0, self.k1 = k0, k1
        self.group = group
        self.bias = None if bias is None else bias.float()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.local(x[..., self.k0:self.k1].contiguous())
        if self.config.is_parallel:
            import torch.distributed as dist

            dist.all_reduce(y, group=self.group or _default_group())
        if self.bias is not None:
            y = y + self.bias.to(y.device)
        return y
