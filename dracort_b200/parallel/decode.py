"""Tensor-parallel decode of one decoder layer's projection set (q, k, v, o,
gate, up, down) — the multi-GPU form of the config-2 / config-4 workload.

Per rank: one grouped GEMV launch over the rank's shards of the seven weights
(column-parallel q/k/v/gate/up: a range of output rows; row-parallel o/down: a
super-block range of the reduction dim).  These are the shard-boundary
exchanges of draco/parallel/tp.py (ColumnParallelLinear / RowParallelLinear,
whose all-reduce the reference leaves as a comment, tp.py:182-183), done per
layer in one of two ways:

* ``fused=False`` (the NCCL baseline): the GEMV writes two local
  communication buffers, then one NCCL all-gather for the five
  column-parallel outputs and one NCCL all-reduce for the two row-parallel
  ones.
* ``fused=True``: the GEMV (draco_gguf_gemv_grouped_tp) stores every output
  value straight into every rank's exchange buffer over NVLink and signals
  each rank when done; draco_tp_finish then waits for every rank's signal,
  copies the gathered columns out and sums the row partials in rank order.
  Two kernel launches per step and no host collective, so the step can be
  captured in a CUDA graph.
"""

from __future__ import annotations

import math
from typing import List, Sequence

import numpy as np
import torch

import ctypes

from dracort_b200 import _native as N
from dracort_b200 import gguf_ops as G
from dracort_b200.parallel.tp import shard_k, shard_rows

COLUMN = ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj")
ROW = ("o_proj", "down_proj")


class TPDecodeLayer:
    """Sharded layer set with fused collectives; `step(i)` runs one decode step."""

    def __init__(self, specs: Sequence, packed: Sequence[np.ndarray], rank: int, world: int, batch: int,
                 device: torch.device, seed: int = 0, group=None, l2_bytes: int = 126 << 20,
                 min_copies: int = 2, copies: int = 0, fused: bool = False) -> None:
        """copies: weight copies to rotate through (0: enough to exceed 4x L2);
        fused: exchange over NVLink inside the kernels instead of NCCL."""
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
        self.fused = fused
        self.exchange = None
        if fused:
            self._init_fused(copies)
            self.launches_per_step = 2  # the tensor-parallel GEMV and the finish kernel
            self.graph_safe = True
            return
        self.plans = [G.GemvPlan([G.GemvProblem(qt, c[i], self.x_local[i], self.y_local[i], n, k)
                                  for i, (_, qt, n, k, _, _, _) in enumerate(self.local)]) for c in copies]
        self.launches_per_step = 1  # our GEMV kernel; NCCL adds its own collective kernels
        self.graph_safe = False

    def _init_fused(self, copies) -> None:
        """Exchange buffer layout (identical on every rank): flags[2][8] int32 at
        0, the step counter at 128, then per step parity the gathered column
        block [world][batch][wc] and the row-partial block [world][batch][wr]."""
        from dracort_b200.parallel.exchange import ExchangeBuffer

        B, W, r = self.batch, self.world, self.rank

        def a256(v):
            return (v + 255) // 256 * 256

        self.g_stride = W * B * self.wc * 4
        self.r_stride = W * B * self.wr * 4
        self.g_off = 256
        self.r_off = a256(self.g_off + 2 * self.g_stride)
        self.exchange = ExchangeBuffer(a256(self.r_off + 2 * self.r_stride), r, W, self.group)
        ex = N.TpExchange()
        ex.world, ex.rank = W, r
        for q, ptr in enumerate(self.exchange.ptrs):
            ex.buffers[q] = ptr
        ex.flags_off, ex.counter_off = 0, 128
        ldys = []
        oc = orr = 0
        for j, (_, _, n, _, _, kind, _) in enumerate(self.local):
            if kind == "col":
                ex.y_off[j] = self.g_off + (r * B * self.wc + oc) * 4
                ex.parity_stride[j] = self.g_stride
                ldys.append(self.wc)
                oc += n
            else:
                ex.y_off[j] = self.r_off + (r * B * self.wr + orr) * 4
                ex.parity_stride[j] = self.r_stride
                ldys.append(self.wr)
                orr += n
        self.ex = ex
        self._lib = N.load()
        self.tp_status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.tp_plans = []
        for c in copies:
            arr = (N.GemvProblem * len(self.local))()
            for j, ((_, qt, n, k, _, _, _), xl) in enumerate(zip(self.local, self.x_local)):
                arr[j] = N.GemvProblem(qt, 0, c[j].data_ptr(), xl.data_ptr(), None, None, n, k, xl.stride(0),
                                       ldys[j])
            need = self._lib.draco_gguf_gemv_workspace_bytes(arr, len(self.local), B)
            if need == 0:
                N.check(N.DRACO_ERR_ARG, "gemv_tp workspace query failed")
            ws = torch.zeros(int(need), dtype=torch.uint8, device=self.device)
            self.tp_plans.append((arr, ws, c))

    def _step_fused(self, i: int) -> None:
        arr, ws, _ = self.tp_plans[i % len(self.tp_plans)]
        stream = torch.cuda.current_stream(self.device).cuda_stream
        rc = self._lib.draco_gguf_gemv_grouped_tp(arr, len(self.local), self.batch, ctypes.byref(self.ex),
                                                  ws.data_ptr(), ws.numel(), stream)
        if rc:
            N.check(rc, "gemv_tp")
        rc = self._lib.draco_tp_finish(ctypes.byref(self.ex), self.batch, self.g_off, self.g_stride, self.wc,
                                       self.gout.data_ptr(), self.r_off, self.r_stride, self.wr,
                                       self.rbuf.data_ptr(), self.tp_status.data_ptr(), stream)
        if rc:
            N.check(rc, "tp_finish")

    def status(self) -> int:
        """First nonzero device status of the fused path (finish, then the GEMV
        workspaces), 0 when every step succeeded.  Synchronises."""
        if not self.fused:
            return 0
        st = int(self.tp_status.item())
        for _, ws, _ in self.tp_plans:
            st = st or int(ws[:4].view(torch.int32).item())
        return st

    def step(self, i: int) -> None:
        import torch.distributed as dist

        if self.fused:
            self._step_fused(i)
            return
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
        if self.fused:
            self.tp_plans.clear()
            if self.exchange is not None:
                self.exchange.close()
                self.exchange = None
            return
        self.plans.clear()
