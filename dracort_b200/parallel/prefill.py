"""Tensor-parallel prefill of one decoder layer's MLP projections (gate, up,
down) — the multi-GPU form of the config-3 workload.

Per rank: one grouped dequant-GEMM launch over the rank's shards, bf16
activations, fp32 accumulation: gate and up column-parallel (a range of output
rows), down row-parallel (a super-block range of the reduction dim, fed by the
matching slice of the down-projection input); then one NCCL all-reduce of the
down output.  These are the shard boundaries of draco/parallel/tp.py
(ColumnParallelLinear / RowParallelLinear, tp.py:140-183): the column outputs
stay sharded because the row-parallel down consumes exactly the slice the
column shards produce, and the row-parallel partial sums are reduced once.
At world size 1 the same object runs the unsharded step with no collective.
"""

from __future__ import annotations

from typing import Sequence

import numpy as np
import torch

from dracort_b200 import gguf_ops as G
from dracort_b200.parallel.tp import shard_k, shard_rows

COLUMN = ("gate_proj", "up_proj")
ROW = ("down_proj",)


class TPPrefillLayer:
    """Sharded gate/up/down with bf16 activations; `step(i)` runs one prefill step."""

    def __init__(self, specs: Sequence, packed: Sequence[np.ndarray], rank: int, world: int, m: int,
                 device: torch.device, seed: int = 0, group=None, copies: int = 2) -> None:
        self.rank, self.world, self.m, self.device = rank, world, m, device
        self.group = group
        if world > 1 and group is None:
            import torch.distributed as dist

            self.group = dist.group.WORLD
        self.specs = list(specs)
        rng = torch.Generator(device="cpu").manual_seed(seed + 3)
        self.local = []  # (spec, qtype, n_local, k_local, shard, kind, k0)
        for s, p in zip(specs, packed):
            if s.name in ROW:
                shard, k0, k1 = shard_k(p, s.qtype, s.n_rows, s.k, rank, world)
                self.local.append((s, s.qtype, s.n_rows, k1 - k0, shard, "row", k0))
            else:
                shard, r0, r1 = shard_rows(p, s.qtype, s.n_rows, s.k, rank, world)
                self.local.append((s, s.qtype, r1 - r0, s.k, shard, "col", 0))
        tiled0 = [G.repack(qt, torch.from_numpy(sh.reshape(-1)).to(device), n, k)
                  for (_, qt, n, k, sh, _, _) in self.local]
        self.local_weight_bytes = int(sum(t.numel() for t in tiled0))
        self.n_copies = max(1, copies)
        self.weights = [tiled0] + [[t.clone() for t in tiled0] for _ in range(self.n_copies - 1)]
        # activations (identical on every rank): the layer input for gate/up, the
        # down-projection input for down (each rank reads its K slice)
        self.x_full = {}
        for s in specs:
            key = "down_in" if s.name in ROW else "hidden"
            if key not in self.x_full:
                self.x_full[key] = torch.randn((m, s.k), generator=rng).to(torch.bfloat16).to(device)
        self.x_local, self.y_local = [], []
        for (s, qt, n, k, _, kind, k0) in self.local:
            if kind == "col":
                self.x_local.append(self.x_full["hidden"])
            else:
                self.x_local.append(self.x_full["down_in"][:, k0:k0 + k].contiguous())
            self.y_local.append(torch.empty((m, n), dtype=torch.bfloat16, device=device))
        self.problems = [[G.GemmProblem(qt, w[i], self.x_local[i], self.y_local[i], n, k)
                          for i, (_, qt, n, k, _, _, _) in enumerate(self.local)] for w in self.weights]
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.launches_per_step = 1  # our GEMM kernel; NCCL adds its collective kernels
        self.flops_local = sum(2 * m * n * k for (_, _, n, k, _, _, _) in self.local)
        self.flops_total = sum(2 * m * s.n_rows * s.k for s in self.specs)

    def step(self, i: int) -> None:
        G.gemm_grouped(self.problems[i % self.n_copies], self.status)
        if self.world > 1:
            import torch.distributed as dist

            for (s, _, _, _, _, kind, _), y in zip(self.local, self.y_local):
                if kind == "row":
                    dist.all_reduce(y, group=self.group)

    def outputs(self) -> dict:
        """Per-projection outputs after a step: column shards (local rows), reduced rows."""
        return {s.name: y for (s, *_), y in zip(self.local, self.y_local)}

    def check_status(self) -> int:
        return int(self.status.item())

    def close(self) -> None:
        self.problems.clear()
        self.weights.clear()
