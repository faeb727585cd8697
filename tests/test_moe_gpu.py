"""GPU parity of the MoE FFN with GGUF experts on the tcgen05 dequant-GEMM.

Reference: ExpertGroup.forward (expert.py:77-129) with TopKRouter
(router.py:106-111) on the oracle's fp32 dequantized weights.  The GPU path
runs bf16 activations (x, the SwiGLU product and the expert outputs are bf16
tensors), so the bar is the bf16 prefill one, 5e-3 relative L2.
"""

import numpy as np
import pytest

from oracle import gguf_oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

import torch.nn.functional as F  # noqa: E402

from dracort_b200.format import quantize as Q  # noqa: E402
from dracort_b200.parallel.moe import EPMoELayer, TopKRouter  # noqa: E402

PREFILL_TOL = 5e-3


def _experts(rng, n_exp, hidden, ffn, qtypes):
    out = []
    for e in range(n_exp):
        qt = qtypes[e % len(qtypes)]
        out.append((qt, Q.encode(qt, Q.random_weight(rng, ffn, hidden)), Q.encode(qt, Q.random_weight(rng, ffn, hidden)),
                    Q.encode(qt, Q.random_weight(rng, hidden, ffn))))
    return out


def _reference(x, logits, experts, hidden, ffn, top_k):
    idx, w = TopKRouter(len(experts), top_k).route(logits)
    out = torch.zeros((x.shape[0], hidden))
    for e, (qt, g, u, d) in enumerate(experts):
        mask = (idx == e).any(dim=-1)
        if not mask.any():
            continue
        t = mask.nonzero(as_tuple=True)[0]
        wg = torch.from_numpy(O.dequantize_matrix(qt, g, ffn, hidden))
        wu = torch.from_numpy(O.dequantize_matrix(qt, u, ffn, hidden))
        wd = torch.from_numpy(O.dequantize_matrix(qt, d, hidden, ffn))
        xe = x[t]
        ye = (F.silu(xe @ wg.T) * (xe @ wu.T)) @ wd.T
        we = (w[t] * (idx[t] == e).float()).sum(dim=-1, keepdim=True)
        out.index_add_(0, t, ye * we)
    return out


@pytest.mark.parametrize("qtypes", [(12,), (12, 14)])
def test_moe_layer_matches_expert_group(qtypes):
    rng = np.random.default_rng(7)
    n_exp, hidden, ffn, top_k, tokens = 8, 512, 1024, 2, 40
    experts = _experts(rng, n_exp, hidden, ffn, qtypes)
    x = torch.from_numpy(rng.standard_normal((tokens, hidden)).astype(np.float32)).to(torch.bfloat16)
    logits = torch.from_numpy(rng.standard_normal((tokens, n_exp)).astype(np.float32))
    layer = EPMoELayer(experts, hidden, ffn, top_k, 0, 1, torch.device("cuda"))
    y = layer.forward(x.cuda(), logits.cuda())
    torch.cuda.synchronize()
    assert layer.check_status() == 0
    ref = _reference(x.float(), logits, experts, hidden, ffn, top_k)
    assert O.rel_l2(y.cpu().numpy(), ref.numpy()) < PREFILL_TOL
    # no host synchronisation inside the step: it replays from a CUDA graph,
    # bit-identically
    xc, lc = x.cuda(), logits.cuda()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        yg = layer.forward(xc, lc)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(yg, y)


@pytest.mark.parametrize("n", [8 * 1000, 8 * 1000 + 5, 3])
def test_swiglu_bf16_matches_fp32_formula(n):
    from dracort_b200 import gguf_ops as G

    g = torch.Generator().manual_seed(n)
    gate = (3 * torch.randn(n, generator=g)).to(torch.bfloat16).cuda()
    up = torch.randn(n, generator=g).to(torch.bfloat16).cuda()
    out = G.swiglu_bf16(gate, up)
    ref = (F.silu(gate.float()) * up.float()).to(torch.bfloat16)
    diff = (out.float() - ref.float()).abs()
    # one bf16 rounding of an fp32 value; expf may differ from torch's by an ulp
    assert torch.all(diff <= 2 ** -7 * ref.float().abs() + 1e-30)
    inplace = gate.clone()
    G.swiglu_bf16(inplace, up, out=inplace)
    assert torch.equal(inplace, out)


def _numpy_route(logits, top_k):
    """TopKRouter.forward (router.py:81-120) restated in numpy, independent of
    the product's router: top-k of the logits, softmax over the k selected,
    renormalised (router.py:106-111)."""
    idx = np.argsort(-logits, axis=-1, kind="stable")[:, :top_k]
    sel = np.take_along_axis(logits, idx, axis=-1).astype(np.float64)
    w = np.exp(sel - sel.max(axis=-1, keepdims=True))
    w /= w.sum(axis=-1, keepdims=True)
    w /= w.sum(axis=-1, keepdims=True)
    return idx, w.astype(np.float32)


def test_moe_layer_at_config5_shapes_matches_expert_group_math():
    """Config 5 in full: 8 Q4_K experts (gate/up 14336x4096, down 4096x14336),
    256 bf16 tokens, top-2, against ExpertGroup.forward's math
    (expert.py:77-116: per expert down(silu(gate(x)) * up(x)), outputs added
    with the routing weights) on the oracle's fp32 weights, routed in numpy."""
    from dracort_b200.workloads import MOE_FFN, MOE_HIDDEN, MOE_TOKENS, MOE_TOP_K, moe_experts

    experts = moe_experts(2024)
    rng = np.random.default_rng(2025)
    x = torch.from_numpy(rng.standard_normal((MOE_TOKENS, MOE_HIDDEN)).astype(np.float32)).to(torch.bfloat16)
    logits = rng.standard_normal((MOE_TOKENS, len(experts))).astype(np.float32)
    layer = EPMoELayer(experts, MOE_HIDDEN, MOE_FFN, MOE_TOP_K, 0, 1, torch.device("cuda"))
    y = layer.forward(x.cuda(), torch.from_numpy(logits).cuda()).cpu().numpy()
    torch.cuda.synchronize()
    assert layer.check_status() == 0

    idx, w = _numpy_route(logits, MOE_TOP_K)
    xf = x.float().numpy()
    ref = np.zeros((MOE_TOKENS, MOE_HIDDEN), dtype=np.float32)
    for e, (qt, g, u, d) in enumerate(experts):
        rows, slot = np.nonzero(idx == e)
        if rows.size == 0:
            continue
        xe = xf[rows]
        h = xe @ O.dequantize_matrix(qt, g, MOE_FFN, MOE_HIDDEN).T
        h = h / (1.0 + np.exp(-h)) * (xe @ O.dequantize_matrix(qt, u, MOE_FFN, MOE_HIDDEN).T)
        ye = h @ O.dequantize_matrix(qt, d, MOE_HIDDEN, MOE_FFN).T
        np.add.at(ref, rows, ye * w[rows, slot][:, None])
    assert O.rel_l2(y, ref) < PREFILL_TOL
