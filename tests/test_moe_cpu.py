"""MoE routing and expert-parallel dispatch/combine on CPU ranks (gloo), no GPU.

The experts' GEMM is replaced by an fp32 restatement of the reference Expert
(down(silu(gate(x)) * up(x)), expert.py:47-49) on the oracle's dequantized
weights, injected through EPMoELayer's expert-group factory; the tests check
the router (router.py:106-111), the all-to-all token exchange and the
weighted combine against the single-rank result (ExpertGroup.forward,
expert.py:77-129).
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from dracort_b200.format import quantize as Q
from dracort_b200.parallel.moe import EPMoELayer, TopKRouter
from oracle import gguf_oracle as O

E, HIDDEN, FFN, TOP_K = 4, 256, 512, 2


class OracleExperts:
    """fp32 experts on the oracle's dequantized weights (same run() contract)."""

    def __init__(self, experts, hidden, ffn, device, e0):
        self.w = [tuple(torch.from_numpy(O.dequantize_matrix(qt, p, n, k)) for p, n, k in
                        ((g, ffn, hidden), (u, ffn, hidden), (d, hidden, ffn))) for qt, g, u, d in experts]

    def run_padded(self, x, rows, cap):
        out = torch.full((len(self.w), cap, x.shape[-1]), float("nan"))  # unused rows hold no meaning
        for e, ((wg, wu, wd), c) in enumerate(zip(self.w, rows.tolist())):
            xe = x[e, :c].float()
            out[e, :c] = (F.silu(xe @ wg.T) * (xe @ wu.T)) @ wd.T
        return out


def make_experts(seed):
    rng = np.random.default_rng(seed)
    return [(12, Q.encode(12, Q.random_weight(rng, FFN, HIDDEN)), Q.encode(12, Q.random_weight(rng, FFN, HIDDEN)),
             Q.encode(12, Q.random_weight(rng, HIDDEN, FFN))) for _ in range(E)]


def reference_moe(x, logits, experts):
    """ExpertGroup.forward semantics over all experts, one process."""
    idx, w = TopKRouter(E, TOP_K).route(logits)
    ex = OracleExperts(experts, HIDDEN, FFN, None, 0)
    out = torch.zeros((x.shape[0], HIDDEN))
    for e in range(E):
        mask = (idx == e).any(dim=-1)
        if not mask.any():
            continue
        t = mask.nonzero(as_tuple=True)[0]
        xe = torch.zeros((E, len(t), HIDDEN))
        xe[e] = x[t]
        ye = ex.run_padded(xe, torch.tensor([len(t) if j == e else 0 for j in range(E)], dtype=torch.int32),
                           len(t))[e]
        we = (w[t] * (idx[t] == e).float()).sum(dim=-1, keepdim=True)
        out.index_add_(0, t, ye * we)
    return out


def test_router_top2_softmax_renormalised():
    g = torch.Generator().manual_seed(3)
    logits = torch.randn((17, 8), generator=g)
    idx, w = TopKRouter(8, 2).route(logits)
    L = logits.numpy()
    for i in range(17):
        top = np.argsort(-L[i], kind="stable")[:2]
        assert set(idx[i].tolist()) == set(top.tolist())
        sel = L[i][idx[i].numpy()]
        e = np.exp(sel - sel.max())
        np.testing.assert_allclose(w[i].numpy(), e / e.sum(), rtol=1e-6)
    np.testing.assert_allclose(w.sum(-1).numpy(), 1.0, rtol=1e-6)
    with pytest.raises(ValueError):
        TopKRouter(4, 5)


def test_dispatch_plan_positions_and_counts():
    g = torch.Generator().manual_seed(8)
    logits = torch.randn((23, E), generator=g)
    layer = EPMoELayer(make_experts(2), HIDDEN, FFN, TOP_K, 0, 1, torch.device("cpu"),
                       expert_group_factory=OracleExperts)
    dst, w, counts = layer.dispatch_plan(logits)
    idx, _ = TopKRouter(E, TOP_K).route(logits)
    flat = idx.reshape(-1).tolist()
    assert counts.tolist() == [flat.count(e) for e in range(E)]
    seen = [0] * E
    for p, e in enumerate(flat):  # rows of an expert in token order, from row 0 of its block
        assert dst[p].item() == e * 23 + seen[e]
        seen[e] += 1
    assert len(set(dst.tolist())) == len(flat)


def test_ep_single_rank_matches_expert_group():
    experts = make_experts(1)
    g = torch.Generator().manual_seed(5)
    x = torch.randn((12, HIDDEN), generator=g)
    logits = torch.randn((12, E), generator=g)
    layer = EPMoELayer(experts, HIDDEN, FFN, TOP_K, 0, 1, torch.device("cpu"), expert_group_factory=OracleExperts)
    np.testing.assert_allclose(layer.forward(x, logits).numpy(), reference_moe(x, logits, experts).numpy(),
                               rtol=1e-5, atol=1e-6)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        experts = make_experts(1)
        g = torch.Generator().manual_seed(11)
        x_all = torch.randn((world * 9, HIDDEN), generator=g)
        logits_all = torch.randn((world * 9, E), generator=g)
        mine = slice(rank * 9, (rank + 1) * 9)
        layer = EPMoELayer(experts, HIDDEN, FFN, TOP_K, rank, world, torch.device("cpu"),
                           expert_group_factory=OracleExperts)
        y = layer.forward(x_all[mine], logits_all[mine])
        ref = reference_moe(x_all, logits_all, experts)[mine]
        result_q.put((rank, float((y - ref).abs().max())))
    finally:
        dist.destroy_process_group()


def test_ep_dispatch_combine_on_two_gloo_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err in res:
        assert err < 1e-4, (rank, err)
