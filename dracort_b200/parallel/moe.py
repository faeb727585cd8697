"""Mixture-of-experts FFN with GGUF-quantized experts, expert-parallel across
ranks — the config-5 workload (Mixtral-8x7B-shaped layer).

Mirrors draco/models/moe:
* ``TopKRouter`` — router.py:55-120: top-k of the router logits, softmax over
  the k selected logits, renormalised (``norm_topk_prob``).
* ``GGUFExpertGroup`` — expert.py:16-129 (``Expert``: down(silu(gate(x)) *
  up(x)); ``ExpertGroup.forward``: every routed token's expert outputs summed
  with its routing weights) over TILED GGUF weights: the gate and up
  projections of all local experts go through one grouped tcgen05
  dequant-GEMM launch, the SwiGLU product through one kernel, the down
  projections through a second GEMM launch.
* ``EPMoELayer`` — the dispatch/combine of dispatch.py:17-79 made
  expert-parallel: rank r owns experts [r*E/W, (r+1)*E/W); each rank routes
  its own tokens, sends every (token, expert) copy to the expert's rank with
  one NCCL all-to-all, runs its experts on what it received, and returns the
  outputs with a second all-to-all; the source rank adds them with the
  routing weights.  At world size 1 there is no collective.

The step never waits for the host.  Routing positions and per-expert token
counts are computed on the device; tokens travel in fixed-capacity blocks
(an expert receives at most one row per token of each rank, so a block of
the rank's token count always suffices), every all-to-all has equal splits,
and the GEMM and SwiGLU kernels read the counts from device memory
(draco_gguf_gemm_rows, draco_swiglu_bf16_rows) and skip the empty rows.  The
layer can therefore be captured in a CUDA graph.  The combine sums each
token's k expert outputs in slot order: the result is deterministic.
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

    def run_padded(self, x: torch.Tensor, rows: torch.Tensor, cap: int) -> torch.Tensor:
        """x: [n_local, cap, hidden] bf16, expert i's tokens in the first rows[i]
        rows of block i; rows: CUDA int32 [n_local].  Returns [n_local, cap,
        hidden] bf16 expert outputs (rows past rows[i] hold no meaning)."""
        n, H, Fn, bf = self.n_local, self.hidden, self.ffn, G.N.DTYPE_BF16
        if x.dtype != torch.bfloat16 or not x.is_contiguous():
            x = x.to(torch.bfloat16).contiguous()
        gate = torch.empty((n, cap, Fn), dtype=torch.bfloat16, device=self.device)
        up = torch.empty_like(gate)
        out = torch.empty((n, cap, H), dtype=torch.bfloat16, device=self.device)
        px, pg, pu, po = x.data_ptr(), gate.data_ptr(), up.data_ptr(), out.data_ptr()
        gu, down = [], []
        for i, (qt, wg, wu, wd) in enumerate(self.w_ptrs):
            xr, fr = px + 2 * i * cap * H, 2 * i * cap * Fn
            gu.append((qt, wg, xr, pg + fr, cap, Fn, H, H, Fn, bf))
            gu.append((qt, wu, xr, pu + fr, cap, Fn, H, H, Fn, bf))
            down.append((qt, wd, pg + fr, po + 2 * i * cap * H, cap, H, Fn, Fn, H, bf))
        rows = rows.to(torch.int32).contiguous()
        rows2 = rows.repeat_interleave(2)  # gate and up of each expert
        mx = G.N.GEMM_MAX_PROBLEMS
        for i in range(0, len(gu), mx):
            G.gemm_rows_raw(gu[i:i + mx], rows2[i:i + mx], self.device, self.status)
        G.swiglu_bf16_rows(gate, up, gate, rows)  # the SwiGLU product overwrites gate, the down input
        for i in range(0, len(down), mx):
            G.gemm_rows_raw(down[i:i + mx], rows[i:i + mx], self.device, self.status)
        return out


class EPMoELayer:
    """Expert-parallel MoE FFN over `world` ranks (one process per GPU)."""

    def __init__(self, experts: Sequence, hidden: int, ffn: int, top_k: int, rank: int, world: int,
                 device: torch.device, group=None, expert_group_factory=None) -> None:
        """experts: per expert (qtype, gate, up, down) packed payloads, or whatever
        `expert_group_factory(experts_of_this_rank, hidden, ffn, device, e0)`
        takes (default: GGUFExpertGroup); the group's run_padded(x, rows, cap)
        computes its experts on fixed-capacity blocks."""
        n_exp = len(experts)
        if n_exp % world:
            raise ValueError(f"{n_exp} experts do not split evenly over {world} ranks")
        self.n_exp, self.hidden, self.ffn, self.top_k = n_exp, hidden, ffn, top_k
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

    def dispatch_plan(self, router_logits: torch.Tensor):
        """Device-side routing: expert index and weight of every (token, slot),
        its row in the [n_exp, cap] block layout (cap = tokens of this rank;
        rows of an expert in token order) and the per-expert counts."""
        T = router_logits.shape[0]
        idx, wts = self.router.route(router_logits)
        flat_e = idx.reshape(-1)
        # [expert, pair] running counts: a scan along the contiguous dimension
        # (a scan across rows costs ~150 us on the GPU for 512 x 8 values)
        csum = F.one_hot(flat_e, self.n_exp).to(torch.int32).t().contiguous().cumsum(1, dtype=torch.int32)
        pos = csum.gather(0, flat_e[None, :]).squeeze(0) - 1
        counts = csum[:, -1].contiguous() if T else torch.zeros(self.n_exp, dtype=torch.int32, device=flat_e.device)
        return flat_e * T + pos, wts, counts

    def forward(self, x: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        """x (tokens, hidden) and router logits (tokens, E) of this rank's tokens
        -> (tokens, hidden) fp32 MoE output."""
        T, H, k, E, W, El = x.shape[0], self.hidden, self.top_k, self.n_exp, self.world, self.per_rank
        dst, wts, counts = self.dispatch_plan(router_logits)
        cap = T
        send = x.new_empty((E * cap, H))
        send.index_copy_(0, dst, x.repeat_interleave(k, dim=0))
        if W == 1:
            back = self.local.run_padded(send.view(E, cap, H), counts, cap).view(E * cap, H)
        else:
            import torch.distributed as dist

            recv = torch.empty_like(send)  # [source rank][local expert][cap]
            dist.all_to_all_single(recv, send, group=self.group)
            rc = torch.empty_like(counts)
            dist.all_to_all_single(rc, counts, group=self.group)
            rc = rc.view(W, El)
            # regroup each local expert's rows from every source into one block
            # of capacity W * cap; unused rows of a source block go to a spare row
            cap2 = W * cap
            off = rc.cumsum(0) - rc
            i = torch.arange(cap, device=x.device)
            valid = i[None, None, :] < rc[:, :, None]
            el = torch.arange(El, device=x.device)
            dest = (el[None, :, None] * cap2 + off[:, :, None] + i[None, None, :]).to(torch.int64)
            dest = torch.where(valid, dest, torch.full_like(dest, El * cap2)).reshape(-1)
            xin = x.new_empty((El * cap2 + 1, H))
            xin.index_copy_(0, dest, recv)
            y = self.local.run_padded(xin[:El * cap2].view(El, cap2, H), rc.sum(0).to(torch.int32), cap2)
            y = torch.cat([y.view(El * cap2, H), y.new_zeros((1, H))])
            y_send = y.index_select(0, dest)  # back in [destination rank][local expert][cap] order
            back = torch.empty_like(y_send)
            dist.all_to_all_single(back, y_send, group=self.group)
        rows = back.index_select(0, dst).view(T, k, H).float()
        return (rows * wts[..., None]).sum(dim=1)

    def check_status(self) -> int:
        st = getattr(self.local, "status", None)
        return int(st.item()) if st is not None else 0
