"""Kernel-level entry points with the reference's signatures.

* fused_swiGLU (draco/kernels/ops.py:114-137): for arbitrary callables it is
  the reference composition (CPU test); for GGUFLinear projections it runs
  the grouped GEMV or GEMM, the SwiGLU kernel and the down projection (GPU
  tests against the oracle's fp32 MLP on the dequantized weights).
* GGUFGemmKernel: the executor's kernel interface (CPUGemmKernel,
  draco/runtime/cpu/kernels/base.py:15-45) served by the GPU.
"""

from collections import namedtuple

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from dracort_b200.kernels import GGUFGemmKernel, fused_swiGLU
from oracle import gguf_oracle as O

Info = namedtuple("Info", "name ggml_type shape offset quantization")


def test_fused_swiglu_composes_arbitrary_callables_like_the_reference():
    g = torch.Generator().manual_seed(0)
    gate, up, down = torch.nn.Linear(16, 24), torch.nn.Linear(16, 24), torch.nn.Linear(24, 16)
    x = torch.randn((5, 16), generator=g)
    with torch.no_grad():
        assert torch.allclose(fused_swiGLU(x, gate, up, down), down(F.silu(gate(x)) * up(x)))


def test_gemm_kernel_interface():
    k = GGUFGemmKernel(device="cpu")
    assert k.tier == "b200" and "GGUF" in k.name
    assert k.supports(None) and k.supports("gguf_q4_k") and k.supports("gguf_q6_k") and k.supports("gguf_q8_0")
    assert not k.supports("int8_sym")
    w = np.random.default_rng(0).standard_normal((8, 12)).astype(np.float32)
    a = np.random.default_rng(1).standard_normal((3, 12)).astype(np.float32)
    np.testing.assert_allclose(k.matmul_f32(a, w), a @ w.T, rtol=1e-5, atol=1e-5)


gpu = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")


def _mlp(rng, qts, hidden=512, ffn=1024):
    from dracort_b200.format import quantize as Q
    from dracort_b200.quantization import GGUFLinear

    mods, dense = [], []
    for qt, (n, k) in zip(qts, ((ffn, hidden), (ffn, hidden), (hidden, ffn))):
        p = Q.encode(qt, Q.random_weight(rng, n, k))
        mods.append(GGUFLinear.from_packed(qt, p, k, n, device="cuda"))
        dense.append(torch.from_numpy(O.dequantize_matrix(qt, p, n, k)))
    return mods, dense


@gpu
@needs_cuda
@pytest.mark.parametrize("rows,dtype,tol", [(3, torch.float32, 1e-3), (40, torch.float32, 1e-3),
                                            (128, torch.bfloat16, 5e-3)])
def test_fused_swiglu_on_gguf_linear(rows, dtype, tol):
    rng = np.random.default_rng(rows)
    (gate, up, down), (wg, wu, wd) = _mlp(rng, (12, 12, 14))
    x = torch.from_numpy(rng.standard_normal((rows, 512)).astype(np.float32)).to(dtype)
    y = fused_swiGLU(x.cuda(), gate, up, down).float().cpu()
    xf = x.float()
    ref = (F.silu(xf @ wg.T) * (xf @ wu.T)) @ wd.T
    assert O.rel_l2(y.numpy(), ref.numpy()) < tol


@gpu
@needs_cuda
@pytest.mark.parametrize("n", [4 * 1000, 4 * 1000 + 3, 1])
def test_swiglu_f32_matches_formula(n):
    from dracort_b200 import gguf_ops as G

    g = torch.Generator().manual_seed(n)
    gate = (3 * torch.randn(n, generator=g)).cuda()
    up = torch.randn(n, generator=g).cuda()
    ref = F.silu(gate) * up
    out = G.swiglu(gate, up)
    # expf may differ from torch's exp by an ulp or two
    assert torch.allclose(out, ref, rtol=1e-5, atol=1e-6)
    G.swiglu(gate, up, out=gate)
    assert torch.equal(gate, out)


@gpu
@needs_cuda
@pytest.mark.parametrize("qtype,name", [(8, "gguf_q8_0"), (12, "gguf_q4_k"), (14, "gguf_q6_k")])
def test_gemm_kernel_matmul_matches_oracle(qtype, name):
    from dracort_b200.format import quantize as Q

    rng = np.random.default_rng(qtype)
    n, k = 272, 1024
    p = Q.encode(qtype, Q.random_weight(rng, n, k))
    a = rng.standard_normal((2, k)).astype(np.float32)
    kern = GGUFGemmKernel()
    for info in (Info("w", qtype, (n, k), 4096, None), Info(None, None, (n, k), None, name)):
        y = kern.matmul(a, info, p.tobytes())
        assert O.rel_l2(y, O.linear(a, qtype, p, n, k)) < 1e-3
    assert len(kern._cache) == 1  # the named tensor only


@gpu
@needs_cuda
def test_backend_cache_never_serves_a_freed_weight_at_a_reused_address():
    """quantized_linear keeps a TILED copy per weight.  A weight that is freed,
    followed by a new weight of the same size placed at the same address by
    the caching allocator, must be repacked, not served the old copy."""
    from dracort_b200.format import quantize as Q
    from dracort_b200.quantization import GGUFBackend

    be = GGUFBackend(12)
    rng = np.random.default_rng(5)
    n, k = 128, 512
    x = rng.standard_normal((2, k)).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    pa = Q.encode(12, Q.random_weight(rng, n, k))
    pb = Q.encode(12, Q.random_weight(rng, n, k))
    wa = torch.from_numpy(pa).cuda()
    ya = be.quantized_linear(xt, wa, None).cpu().numpy()
    assert O.rel_l2(ya, O.linear(x, 12, pa, n, k)) < 1e-3
    addr = wa.data_ptr()
    del wa
    wb = torch.empty(pb.shape, dtype=torch.uint8, device="cuda")
    assert wb.data_ptr() == addr  # the allocator reused the block (same size class)
    wb.copy_(torch.from_numpy(pb))
    yb = be.quantized_linear(xt, wb, None).cpu().numpy()
    assert O.rel_l2(yb, O.linear(x, 12, pb, n, k)) < 1e-3
    # an in-place rewrite of a live weight is seen as well
    wb.copy_(torch.from_numpy(pa))
    assert O.rel_l2(be.quantized_linear(xt, wb, None).cpu().numpy(), O.linear(x, 12, pa, n, k)) < 1e-3
