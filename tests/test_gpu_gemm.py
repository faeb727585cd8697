"""GPU parity of the tcgen05 prefill dequant-GEMM.

Bars: <= 5e-3 relative L2 against the oracle's fp32 matmul of the bf16-rounded
activations and the fp32 dequantized weights (the bf16 prefill rule), and a
much tighter check against an fp32 matmul of the same bf16 operands (the
tensor cores see bf16 X and bf16(dequant W) exactly; only the summation order
differs).
"""

import numpy as np
import pytest

from oracle import gguf_oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from dracort_b200 import gguf_ops as G  # noqa: E402
from dracort_b200.format import quantize as Q  # noqa: E402

PREFILL_TOL = 5e-3
ALL = [2, 3, 6, 7, 8, 12, 13, 14]


def _case(qtype, m, n, k, seed, ydtype=torch.float32):
    rng = np.random.default_rng(seed)
    packed = Q.encode(qtype, Q.random_weight(rng, n, k))
    x32 = rng.standard_normal((m, k)).astype(np.float32)
    xb = torch.from_numpy(x32).to(torch.bfloat16)
    tiled = G.repack(qtype, torch.from_numpy(packed.reshape(-1)).cuda(), n, k)
    y = G.gemm(qtype, tiled, xb.cuda(), n, k, out_dtype=ydtype)
    torch.cuda.synchronize()
    return packed, xb, tiled, y


def _check(qtype, packed, xb, tiled, y, n, k, tight=2e-5):
    xr = xb.float().numpy()
    ref = O.linear(xr, qtype, packed, n, k)  # oracle: bf16-rounded X, fp32 weights, fp32 matmul
    got = y.float().cpu().numpy()
    assert np.all(np.isfinite(got))
    assert O.rel_l2(got, ref) < PREFILL_TOL
    if y.dtype == torch.float32:
        wb = G.dequantize(qtype, tiled, n, k, layout="tiled", out_dtype=torch.bfloat16).float()
        exact = (xb.cuda().float() @ wb.T).cpu().numpy()
        assert O.rel_l2(got, exact) < tight


@pytest.mark.parametrize("qtype", ALL)
def test_gemm_one_tile(qtype):
    m, n, k = 256, 128, 256
    _check(qtype, *_case(qtype, m, n, k, seed=qtype), n, k)


@pytest.mark.parametrize("qtype", ALL)
@pytest.mark.parametrize("m,n,k", [(300, 200, 512), (1, 16, 256), (777, 384, 1024)])
def test_gemm_ragged(qtype, m, n, k):
    _check(qtype, *_case(qtype, m, n, k, seed=m + n + qtype), n, k)


def test_gemm_bf16_output():
    packed, xb, tiled, y = _case(12, 512, 256, 1024, seed=4, ydtype=torch.bfloat16)
    assert y.dtype == torch.bfloat16
    _check(12, packed, xb, tiled, y, 256, 1024)


def test_gemm_grouped_mixed_types():
    rng = np.random.default_rng(8)
    specs = [(12, 1024, 2048), (14, 512, 2048), (12, 256, 4096), (13, 384, 2048), (2, 256, 1024), (3, 128, 2048),
             (6, 384, 512), (7, 256, 1024), (8, 128, 768)]
    m = 600
    probs, refs = [], []
    for qt, n, k in specs:
        packed = Q.encode(qt, Q.random_weight(rng, n, k))
        xb = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).to(torch.bfloat16)
        tiled = G.repack(qt, torch.from_numpy(packed.reshape(-1)).cuda(), n, k)
        y = torch.empty((m, n), device="cuda")
        probs.append(G.GemmProblem(qt, tiled, xb.cuda(), y, n, k))
        refs.append(O.linear(xb.float().numpy(), qt, packed, n, k))
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    G.gemm_grouped(probs, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for p, r in zip(probs, refs):
        assert O.rel_l2(p.y.cpu().numpy(), r) < PREFILL_TOL


@pytest.mark.parametrize("qtype,n,k", [(12, 11008, 4096), (13, 11008, 4096), (14, 4096, 11008), (2, 11008, 4096),
                                        (7, 4096, 11008)])
def test_gemm_prefill_config_shapes(qtype, n, k):
    # config 3: M = 2048 tokens; gate/up N=11008 K=4096, down N=4096 K=11008
    m = 2048
    packed, xb, tiled, y = _case(qtype, m, n, k, seed=n + k)
    _check(qtype, packed, xb, tiled, y, n, k, tight=5e-5)


def test_gguf_linear_prefill_dispatch():
    # bf16 activations with >= PREFILL_MIN_ROWS rows take the tcgen05 GEMM; fp32
    # activations stay on the fp32 GEMV path (reference executor._linear semantics)
    from dracort_b200.quantization.gguf import PREFILL_MIN_ROWS, GGUFLinear

    rng = np.random.default_rng(21)
    n, k, m = 384, 1024, 200
    assert m >= PREFILL_MIN_ROWS
    packed = Q.encode(12, Q.random_weight(rng, n, k))
    lin = GGUFLinear.from_packed(12, torch.from_numpy(packed), k, n)
    x32 = rng.standard_normal((m, k)).astype(np.float32)
    xb = torch.from_numpy(x32).to(torch.bfloat16).cuda()
    yb = lin(xb)
    assert yb.dtype == torch.bfloat16 and yb.shape == (m, n)
    ref_b = O.linear(xb.float().cpu().numpy(), 12, packed, n, k)
    assert O.rel_l2(yb.float().cpu().numpy(), ref_b) < PREFILL_TOL
    y32 = lin(torch.from_numpy(x32).cuda())
    assert y32.dtype == torch.float32
    assert O.rel_l2(y32.cpu().numpy(), O.linear(x32, 12, packed, n, k)) < 1e-3


def test_gemm_grouped_balanced_schedule():
    # config-3 shapes at M=512: 102 pair tiles of two lengths (64 and 172 k-blocks)
    # on 74 SM pairs, where the launch uses its packed tile schedule instead of
    # the strided order; every output must still be complete and exact
    rng = np.random.default_rng(33)
    m = 512
    specs = [(12, 11008, 4096), (12, 11008, 4096), (14, 4096, 11008)]
    probs, packs, xs = [], [], []
    for qt, n, k in specs:
        packed = Q.encode(qt, Q.random_weight(rng, n, k))
        xb = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).to(torch.bfloat16).cuda()
        tiled = G.repack(qt, torch.from_numpy(packed.reshape(-1)).cuda(), n, k)
        y = torch.full((m, n), float("nan"), device="cuda")
        probs.append(G.GemmProblem(qt, tiled, xb, y, n, k))
        packs.append(packed)
        xs.append(xb)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    G.gemm_grouped(probs, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for (qt, n, k), p, packed, xb in zip(specs, probs, packs, xs):
        assert torch.isfinite(p.y).all()
        wb = G.dequantize(qt, p.w_tiled, n, k, layout="tiled", out_dtype=torch.bfloat16).float()
        exact = xb.float() @ wb.T
        err = (torch.linalg.norm(p.y - exact) / torch.linalg.norm(exact)).item()
        assert err < 5e-5
        ref = O.linear(xb[:64].float().cpu().numpy(), qt, packed, n, k)  # oracle on a token sample
        assert O.rel_l2(p.y[:64].cpu().numpy(), ref) < PREFILL_TOL
