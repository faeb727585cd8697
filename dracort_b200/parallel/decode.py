"""Tensor-parallel decode of one decoder layer's projection set (q, k, v, o,
gate, up, down) — the multi-GPU form of the config-2 / config-4 workload.

Per rank: one grouped GEMV launch over the rank's shards of the seven weights
(column-parallel q/k/v/gate/up: a range of output rows; row-parallel o/down: a
super-block range of the reduction dim), writing straight into two fused
communication buffers; then one NCCL all-gather for the five column-parallel
outputs and one NCCL all-reduce for the two row-parallel ones.  These are the
shard-boundary exchanges of draco/parallel/tp.py (ColumnParallelLinear /
RowParallelLinear, whose all-reduce the reference leaves as a comment,
tp.py:182-183), fused per layer.
"""

from __future__ import annotations

import math
from typing import List, Sequence

import numpy as np
import torch

from dracort_b200 import gguf_ops as G
from dracort_b200.parallel.tp import shard_k, shard_rows

COLUMN = ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj")
ROW = ("o_proj", "down_proj")


class TPDecodeLayer:
    """Sharded layer set with fused collectives; `step(i)` runs one decode step."""

    def __init__(self, specs: Sequence, packed: Sequence[np.ndarray], rank: int, world: int, batch: int,
                 device: torch.device, seed: int = 0, group=None, l2_bytes: int = 126 << 20,
                 min_copies: int = 2, copies: int = 0) -> None:
        """copies: weight copies to rotate through (0: enough to exceed 4x L2)."""
        import torch.distributed as dist

        self.rank, self.world, self.batch, self.device = rank, world, batch, device
        self.group = group if group is not None else dist.group.WORLD
        self.specs = list(specs)
        col = [(s, p) for s, p in zip(specs, packed) if s.name in COLUMN]
        row = [(s, p) for s, p in zip(specs, packed) if s.name in ROW]
        rng = torch.Generator(device="cpu").manual_seed(seed + 1)

        # shards (weights are identical on every rank: same seed)
        self.local = []  # (spec, qtype, n_local, k_local, tiled, kind, k0)
        for s, p in col:
            shard, r0, r1 = shard_rows(p, s.qtype, s.n_rows, s.k, rank, world)
            self.local.append((s, s.qtype, r1 - r0, s.k, shard, "col", 0))
        for s, p in row:
            shard, k0, k1 = shard_k(p, s.qtype, s.n_rows, s.k, rank, world)
            self.local.append((s, s.qtype, s.n_rows, k1 - k0, shard, "row", k0))
        tiled0 = [G.repack(qt, torch.from_numpy(sh.reshape(-1)).to(device), n, k)
                  for (_, qt, n, k, sh, _, _) in self.local]
        self.local_weight_bytes = int(sum(t.numel() for t in tiled0))
        self.n_copies = copies or max(min_copies, math.ceil(4 * l2_bytes / max(1, self.local_weight_bytes)))
        copies = [tiled0] + [[t.clone() for t in tiled0] for _ in range(self.n_copies - 1)]

        # activations: full x for column shards, the rank's K slice for row shards
        self.x_full = {s.name: torch.randn((batch, s.k), generator=rng).to(device) for s, _ in col + row}
        self.x_local = []
        for (s, qt, n, k, _, kind, k0) in self.local:
            xf = self.x_full[s.name]
            self.x_local.append(xf if kind == "col" else xf[:, k0:k0 + k].contiguous())

        # fused communication buffers; GEMV outputs are views into them
        self.wc = sum(n for (_, _, n, _, _, kind, _) in self.local if kind == "col")
        self.wr = sum(n for (_, _, n, _, _, kind, _) in self.local if kind == "row")
        self.gbuf = torch.empty((batch, self.wc), device=device)
        self.gout = torch.empty((world * batch, self.wc), device=device)
        self.rbuf = torch.empty((batch, self.wr), device=device)
        self.y_local = []
        oc = orr = 0
        for (_, _, n, _, _, kind, _) in self.local:
            if kind == "col":
                self.y_local.append(self.gbuf[:, oc:oc + n])
                oc += n
            else:
                self.y_local.append(self.rbuf[:, orr:orr + n])
                orr += n
        self.plans = [G.GemvPlan([G.GemvProblem(qt, c[i], self.x_local[i], self.y_local[i], n, k)
                                  for i, (_, qt, n, k, _, _, _) in enumerate(self.local)]) for c in copies]
        self.launches_per_step = 1  # our GEMV kernel; NCCL adds its own collective kernels
        self.graph_safe = False

    def step(self, i: int) -> None:
        import torch.distributed as dist

        self.plans[i % self.n_copies].run()
        dist.all_gather_into_tensor(self.gout, self.gbuf, group=self.group)
        dist.all_reduce(self.rbuf, group=self.group)

    def outputs(self) -> dict:
        """Full outputs of every projection (after a step): gathered columns, reduced rows."""
        out = {}
        g = self.gout.view(self.world, self.batch, self.wc)
        oc = orr = 0
        for (s, _, n, _, _, kind, _) in self.local:
            if kind == "col":
                out[s.name] = torch.cat([g[r, :, oc:oc + n] for r in range(self.world)], dim=1)
                oc += n
            else:
                out[s.name] = self.rbuf[:, orr:orr + n]
                orr += n
        return out

    def e2e(self, K: int, timed) -> dict:
        """Same step with pinned-host activations in and results out, eager."""
        xh = {k: v.cpu().pin_memory() for k, v in self.x_full.items()}
        gh = torch.empty(self.gout.shape).pin_memory()
        rh = torch.empty(self.rbuf.shape).pin_memory()

        def steps():
            for i in range(K):
                for (s, _, _, k, _, kind, k0), xl in zip(self.local, self.x_local):
                    src = xh[s.name] if kind == "col" else xh[s.name][:, k0:k0 + k]
                    xl.copy_(src, non_blocking=True)
                self.step(i)
                gh.copy_(self.gout, non_blocking=True)
                rh.copy_(self.rbuf, non_blocking=True)

        ms, _, _ = timed(steps)
        h2d = sum(xl.numel() * 4 for xl in self.x_local)
        return {"ms_per_step": round(ms / K, 5), "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": (self.gout.numel() + self.rbuf.numel()) * 4}

    def close(self) -> None:
        self.plans.clear()
