"""Mixture-of-experts FFN with GGUF-quantized experts, expert-parallel across
ranks — the config-5 workload (Mixtral-8x7B-shaped layer).

Mirrors draco/models/moe:
* ``TopKRouter`` — router.py:55-120: top-k of the router logits, softmax over
  the k selected logits, renormalised (``norm_topk_prob``).
* ``GGUFExpertGroup`` — expert.py:16-129 (``Expert``: down(silu(gate(x)) *
  up(x)); ``ExpertGroup.forward``: every routed token's expert outputs summed
  with its routing weights) over TILED GGUF weights: the gate and up
  projections of all local experts go through one grouped tcgen05
  dequant-GEMM launch, the down projections through a second.
* ``EPMoELayer`` — the dispatch/combine of dispatch.py:17-79 made
  expert-parallel: rank r owns experts [r*E/W, (r+1)*E/W); each rank routes
  its own tokens, sends every (token, expert) copy to the expert's rank with
  one NCCL all-to-all (the variable split sizes are exchanged first), runs
  its experts on what it received, and returns the outputs with a second
  all-to-all; the source rank adds them with the routing weights.  At world
  size 1 there is no collective.

The hot path is the quantized linear (the GEMM kernel) and the SwiGLU product
between gate/up and down (draco_swiglu_bf16); routing and the token
permutation are small tensor ops around them.
"""

from __future__ import annotations

from typing import Sequence, Tuple

import numpy as np
import torch
import torch.nn.functional as F

from dracort_b200 import gguf_ops as G


class TopKRouter:
    """Top-k routing over router logits (router.py:55-120)."""

    def __init__(self, num_experts: int, top_k: int = 2, norm_topk_prob: bool = True) -> None:
        if not 1 <= top_k <= num_experts:
            raise ValueError(f"top_k must be in 1..{num_experts}, got {top_k}")
        self.num_experts = num_experts
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob

    def route(self, router_logits: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """(tokens, E) logits -> expert indices (tokens, k) int64, weights (tokens, k) fp32."""
        vals, idx = torch.topk(router_logits.float(), self.top_k, dim=-1)
        w = F.softmax(vals, dim=-1)
        if self.norm_topk_prob:
            w = w / w.sum(dim=-1, keepdim=True)
        return idx, w

    def get_num_experts(self) -> int:
        return self.num_experts

    def get_top_k(self) -> int:
        return self.top_k


class GGUFExpertGroup:
    """The experts [e0, e0 + n) of a layer, weights in the TILED layout.

    ``experts[i] = (qtype, gate_packed, up_packed, down_packed)``: packed GGUF
    payloads, gate/up [ffn, hidden], down [hidden, ffn].
    """

    def __init__(self, experts: Sequence[Tuple[int, np.ndarray, np.ndarray, np.ndarray]], hidden: int, ffn: int,
                 device: torch.device, e0: int = 0) -> None:
        self.hidden, self.ffn, self.device, self.e0 = hidden, ffn, device, e0
        self.w = []  # per local expert: (qtype, gate, up, down) TILED tensors
        for qt, g, u, d in experts:
            def tiled(p, n, k, qt=qt):
                return G.repack(qt, torch.from_numpy(np.ascontiguousarray(p).reshape(-1)).to(device), n, k)
            self.w.append((qt, tiled(g, ffn, hidden), tiled(u, ffn, hidden), tiled(d, hidden, ffn)))
        self.w_ptrs = [(qt, a.data_ptr(), b.data_ptr(), c.data_ptr()) for qt, a, b, c in self.w]
        self.status = torch.zeros(1, dtype=torch.int32, device=device)

    @property
    def n_local(self) -> int:
        return len(self.w)

    def run(self, x: torch.Tensor, counts: Sequence[int]) -> torch.Tensor:
        """x: (rows, hidden) bf16 grouped by local expert (counts[i] rows for
        expert i, in order) -> (rows, hidden) bf16 expert outputs."""
        rows = x.shape[0]
        out = torch.empty((rows, self.hidden), dtype=torch.bfloat16, device=self.device)
        if rows == 0:
            return out
        if x.dtype != torch.bfloat16 or not x.is_contiguous():
            x = x.to(torch.bfloat16).contiguous()
        gate = torch.empty((rows, self.ffn), dtype=torch.bfloat16, device=self.device)
        up = torch.empty_like(gate)
        # each expert's rows are a block of x / gate / up / out: pass pointers
        # into the buffers rather than a tensor view per block
        H, Fn, bf = self.hidden, self.ffn, G.N.DTYPE_BF16
        px, pg, pu, po = x.data_ptr(), gate.data_ptr(), up.data_ptr(), out.data_ptr()
        gu, down, r0 = [], [], 0
        for i, c in enumerate(counts):
            if c:
                qt, wg, wu, wd = self.w_ptrs[i]
                xr, fr = px + 2 * r0 * H, 2 * r0 * Fn
                gu.append((qt, wg, xr, pg + fr, c, Fn, H, H, Fn, bf))
                gu.append((qt, wu, xr, pu + fr, c, Fn, H, H, Fn, bf))
                down.append((qt, wd, pg + fr, po + 2 * r0 * H, c, H, Fn, Fn, H, bf))
            r0 += c
        mx = G.N.GEMM_MAX_PROBLEMS
        for i in range(0, len(gu), mx):
            G.gemm_grouped_raw(gu[i:i + mx], self.device, self.status)
        G.swiglu_bf16(gate, up, out=gate)  # the SwiGLU product overwrites gate, the down input
        for i in range(0, len(down), mx):
            G.gemm_grouped_raw(down[i:i + mx], self.device, self.status)
        return out


class EPMoELayer:
    """Expert-parallel MoE FFN over `world` ranks (one process per GPU)."""

    def __init__(self, experts: Sequence, hidden: int, ffn: int, top_k: int, rank: int, world: int,
                 device: torch.device, group=None, expert_group_factory=None) -> None:
        """experts: per expert (qtype, gate, up, down) packed payloads, or whatever
        `expert_group_factory(experts_of_this_rank, hidden, ffn, device, e0)`
        takes (default: GGUFExpertGroup)."""
        n_exp = len(experts)
        if n_exp % world:
            raise ValueError(f"{n_exp} experts do not split evenly over {world} ranks")
        self.n_exp, self.hidden, self.ffn = n_exp, hidden, ffn
        self.rank, self.world, self.device = rank, world, device
        self.per_rank = n_exp // world
        self.group = group
        if world > 1 and group is None:
            import torch.distributed as dist

            self.group = dist.group.WORLD
        e0 = rank * self.per_rank
        self.router = TopKRouter(n_exp, top_k)
        factory = expert_group_factory or GGUFExpertGroup
        self.local = factory(experts[e0:e0 + self.per_rank], hidden, ffn, device, e0)

    def forward(self, x: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        """x (tokens, hidden) and router logits (tokens, E) of this rank's tokens
        -> (tokens, hidden) fp32 MoE output."""
        T = x.shape[0]
        idx, wts = self.router.route(router_logits)
        k = idx.shape[1]
        flat_e = idx.reshape(-1)
        flat_t = torch.arange(T, device=x.device).repeat_interleave(k)
        order = torch.argsort(flat_e, stable=True)  # by expert, hence by owner rank
        send_e = flat_e[order]
        send_t = flat_t[order]
        send_x = x.index_select(0, send_t)
        per_exp = torch.bincount(send_e, minlength=self.n_exp)
        if self.world == 1:
            y_rows = self.local.run(send_x, per_exp.tolist())
        else:
            import torch.distributed as dist

            send_counts = per_exp.view(self.world, self.per_rank).contiguous()  # [dest rank, local expert]
            recv_counts = torch.empty_like(send_counts)
            dist.all_to_all_single(recv_counts, send_counts, group=self.group)
            send_split = send_counts.sum(1).tolist()
            recv_split = recv_counts.sum(1).tolist()
            recv_x = torch.empty((sum(recv_split), self.hidden), dtype=x.dtype, device=x.device)
            dist.all_to_all_single(recv_x, send_x, recv_split, send_split, group=self.group)
            # rows arrive grouped by source rank, each block sorted by local
            # expert: regroup them by local expert for the grouped GEMM
            rc = recv_counts.tolist()
            src_off = np.concatenate([[0], np.cumsum(recv_split)])
            perm, counts = [], []
            for e in range(self.per_rank):
                c = 0
                for s in range(self.world):
                    start = int(src_off[s]) + sum(rc[s][:e])
                    perm.extend(range(start, start + rc[s][e]))
                    c += rc[s][e]
                counts.append(c)
            perm_t = torch.tensor(perm, dtype=torch.long, device=x.device)
            out_rows = self.local.run(recv_x.index_select(0, perm_t), counts)
            back = torch.empty_like(out_rows)
            back.index_copy_(0, perm_t, out_rows)  # source-rank order again
            y_rows = torch.empty((sum(send_split), self.hidden), dtype=out_rows.dtype, device=x.device)
            dist.all_to_all_single(y_rows, back, send_split, recv_split, group=self.group)
        w_rows = wts.reshape(-1)[order]
        out = torch.zeros((T, self.hidden), dtype=torch.float32, device=x.device)
        out.index_add_(0, send_t, y_rows.float() * w_rows[:, None])
        return out

    def check_status(self) -> int:
        st = getattr(self.local, "status", None)
        return int(st.item()) if st is not None else 0
