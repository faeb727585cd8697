"""Layer-boundary fusions in the decode GEMV's activation read, against the oracle.

* RMSNorm before q/k/v and gate/up (draco/kernels/ops.py:29-50,
  fused_rms_norm): GEMV problems whose x is the hidden state before the norm;
  the kernel scales the activations by the norm weight as it reads them and
  the outputs by the row's rsqrt(mean(x^2) + eps).
* SwiGLU before down (draco/kernels/ops.py:114-137, fused_swiGLU): the down
  GEMV reads silu(gate) * up in place of a materialised product.
* The standalone RMSNorm kernel (draco_rmsnorm) with the reference signature.

The reference side is numpy: the norm / SwiGLU formula in fp32 in the
reference's order, then the oracle's linear layer (dequant + fp32 matmul);
the GEMV bar is 1e-3 relative L2.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from dracort_b200 import gguf_ops as G  # noqa: E402
from dracort_b200.format import quantize as Q  # noqa: E402
from oracle import gguf_oracle as O  # noqa: E402

GEMV_TOL = 1e-3


def rmsnorm_np(x, w, eps):
    var = (x * x).mean(-1, keepdims=True, dtype=np.float32)
    return (x * (np.float32(1.0) / np.sqrt(var + np.float32(eps))) * w).astype(np.float32)


def silu_np(g):
    return (g / (1.0 + np.exp(-g.astype(np.float64)))).astype(np.float32)


def _weight(rng, qt, n, k):
    p = Q.encode(qt, Q.random_weight(rng, n, k))
    return p, G.repack(qt, torch.from_numpy(p.reshape(-1)).cuda(), n, k)


@pytest.mark.parametrize("batch", [1, 3, 8, 32])
def test_rmsnorm_fused_into_grouped_gemv(batch):
    rng = np.random.default_rng(40 + batch)
    k = 2048
    x = (3.0 * rng.standard_normal((batch, k)) + 0.5).astype(np.float32)
    wn = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    xn = rmsnorm_np(x, wn, 1e-5)
    specs = [(12, 1024), (14, 512), (13, 256), (8, 768)]
    xt, wt = torch.from_numpy(x).cuda(), torch.from_numpy(wn).cuda()
    probs, refs = [], []
    for i, (qt, n) in enumerate(specs):
        p, t = _weight(rng, qt, n, k)
        bias = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda() if i == 0 else None
        probs.append(G.GemvProblem(qt, t, xt, torch.empty((batch, n), device="cuda"), n, k, bias,
                                   norm_weight=wt, norm_eps=1e-5))
        ref = O.linear(xn, qt, p, n, k)
        refs.append(ref + bias.cpu().numpy() if bias is not None else ref)
    plan = G.GemvPlan(probs)
    plan.run()
    first = [pr.y.clone() for pr in probs]
    plan.run()
    torch.cuda.synchronize()
    assert plan.status() == 0
    for pr, r, f in zip(probs, refs, first):
        assert O.rel_l2(pr.y.cpu().numpy(), r) < GEMV_TOL
        assert torch.equal(pr.y, f)  # deterministic


@pytest.mark.parametrize("batch", [1, 2, 5, 32])
def test_swiglu_fused_into_down_gemv(batch):
    rng = np.random.default_rng(50 + batch)
    f, h = 1536, 512
    g = (2.0 * rng.standard_normal((batch, f))).astype(np.float32)
    u = rng.standard_normal((batch, f)).astype(np.float32)
    for qt in (12, 14):
        p, t = _weight(rng, qt, h, f)
        y = torch.empty((batch, h), device="cuda")
        G.gemv_grouped([G.GemvProblem(qt, t, torch.from_numpy(g).cuda(), y, h, f, up=torch.from_numpy(u).cuda())])
        ref = O.linear(silu_np(g) * u, qt, p, h, f)
        assert O.rel_l2(y.cpu().numpy(), ref) < GEMV_TOL, qt


def test_plain_and_fused_problems_in_one_launch():
    rng = np.random.default_rng(61)
    k, batch = 1024, 4
    x = rng.standard_normal((batch, k)).astype(np.float32)
    g = rng.standard_normal((batch, k)).astype(np.float32)
    u = rng.standard_normal((batch, k)).astype(np.float32)
    wn = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    (p0, t0), (p1, t1), (p2, t2) = (_weight(rng, 12, 256, k) for _ in range(3))
    ys = [torch.empty((batch, 256), device="cuda") for _ in range(3)]
    G.gemv_grouped([G.GemvProblem(12, t0, torch.from_numpy(x).cuda(), ys[0], 256, k),
                    G.GemvProblem(12, t1, torch.from_numpy(x).cuda(), ys[1], 256, k,
                                  norm_weight=torch.from_numpy(wn).cuda(), norm_eps=1e-6),
                    G.GemvProblem(12, t2, torch.from_numpy(g).cuda(), ys[2], 256, k, up=torch.from_numpy(u).cuda())])
    refs = [O.linear(x, 12, p0, 256, k), O.linear(rmsnorm_np(x, wn, 1e-6), 12, p1, 256, k),
            O.linear(silu_np(g) * u, 12, p2, 256, k)]
    for y, r in zip(ys, refs):
        assert O.rel_l2(y.cpu().numpy(), r) < GEMV_TOL


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rms_norm_kernel_matches_reference_formula(dtype):
    from dracort_b200.kernels import fused_rms_norm

    gen = torch.Generator().manual_seed(3)
    x = (2 * torch.randn((5, 7, 4096), generator=gen)).to(dtype)
    w = 1 + 0.1 * torch.randn(4096, generator=gen)
    got = fused_rms_norm(x.cuda(), w.cuda(), 1e-6).float().cpu()
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    if dtype == torch.float32:
        assert torch.allclose(got, ref, rtol=2e-5, atol=2e-6)
    else:  # one bf16 rounding of the fp32 value
        assert torch.allclose(got, ref.to(torch.bfloat16).float(), rtol=2 ** -7, atol=1e-6)


def test_fused_rms_norm_linear_matches_oracle():
    from dracort_b200.kernels import fused_rms_norm_linear
    from dracort_b200.quantization import GGUFLinear

    rng = np.random.default_rng(70)
    k = 1024
    mods, packs = [], []
    for qt, n in ((12, 1024), (12, 256), (14, 256)):
        p = Q.encode(qt, Q.random_weight(rng, n, k))
        mods.append(GGUFLinear.from_packed(qt, p, k, n, device="cuda"))
        packs.append((qt, p, n))
    x = rng.standard_normal((2, k)).astype(np.float32)
    wn = (1 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    outs = fused_rms_norm_linear(torch.from_numpy(x).cuda(), torch.from_numpy(wn), 1e-5, mods)
    xn = rmsnorm_np(x, wn, 1e-5)
    for o, (qt, p, n) in zip(outs, packs):
        assert O.rel_l2(o.cpu().numpy(), O.linear(xn, qt, p, n, k)) < GEMV_TOL
