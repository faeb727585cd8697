"""GPU parity of the CUDA kernels against the CPU oracle (pinned to the reference).

Bars (from the reference's parity rules):
* dequantized weights: bit-exact (fp16 scale x integer quant is exact in fp32);
* GEMV: <= 1e-3 relative L2 against the oracle's fp32 matmul.
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

GEMV_TOL = 1e-3
TYPES = [(2, "q4_0"), (3, "q4_1"), (6, "q5_0"), (7, "q5_1"), (8, "q8_0"), (12, "q4_k"), (13, "q5_k"), (14, "q6_k")]
ALL = [t for t, _ in TYPES]
SMALL_BLOCK = [2, 3, 6, 7, 8]  # 32-element blocks: k need not be a multiple of 256


def dev_bytes(a: np.ndarray) -> "torch.Tensor":
    return torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1)).cuda()


def bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("qtype,name", TYPES)
def test_dequant_gguf_layout_matches_reference_golden(golden, qtype, name):
    n, k = (int(v) for v in golden[f"{name}_shape"])
    got = G.dequantize(qtype, dev_bytes(golden[f"{name}_packed"]), n, k).cpu().numpy()
    assert bits_equal(got, golden[f"{name}_expected"])


def test_dequant_q6k_dlast_matches_llamacpp_decoder(golden):
    n, k = (int(v) for v in golden["q6_k_shape"])
    got = G.dequantize(14, dev_bytes(golden["q6_k_dlast_packed"]), n, k, layout="gguf_dlast").cpu().numpy()
    assert bits_equal(got, golden["q6_k_dlast_expected"])


@pytest.mark.parametrize("qtype,name", TYPES)
def test_repack_then_tiled_dequant_is_bit_exact(golden, qtype, name):
    n, k = (int(v) for v in golden[f"{name}_shape"])
    t = G.repack(qtype, dev_bytes(golden[f"{name}_packed"]), n, k)
    assert t.numel() == G.tiled_nbytes(qtype, n, k)
    got = G.dequantize(qtype, t, n, k, layout="tiled").cpu().numpy()
    assert bits_equal(got, golden[f"{name}_expected"])


@pytest.mark.parametrize("qtype", ALL)
@pytest.mark.parametrize("shape", [(1, 256), (17, 512), (130, 768), (300, 2304)])
def test_dequant_random_shapes(qtype, shape):
    n, k = shape
    rng = np.random.default_rng(n * 7 + k + qtype)
    w = Q.random_weight(rng, n, k)
    packed = Q.encode(qtype, w)
    exp = O.dequantize_matrix(qtype, packed, n, k)
    d = dev_bytes(packed)
    assert bits_equal(G.dequantize(qtype, d, n, k).cpu().numpy(), exp)
    t = G.repack(qtype, d, n, k)
    assert bits_equal(G.dequantize(qtype, t, n, k, layout="tiled").cpu().numpy(), exp)
    bf = G.dequantize(qtype, d, n, k, out_dtype=torch.bfloat16).float().cpu().numpy()
    assert np.array_equal(bf, torch.from_numpy(exp).bfloat16().float().numpy())


@pytest.mark.parametrize("qtype", SMALL_BLOCK)
@pytest.mark.parametrize("batch", [1, 3])
def test_row_length_not_multiple_of_256(qtype, batch):
    n, k = 40, 32 * 13
    rng = np.random.default_rng(5 + qtype)
    packed = Q.encode(qtype, Q.random_weight(rng, n, k))
    exp = O.dequantize_matrix(qtype, packed, n, k)
    t = G.repack(qtype, dev_bytes(packed), n, k)
    assert bits_equal(G.dequantize(qtype, t, n, k, layout="tiled").cpu().numpy(), exp)
    x = rng.standard_normal((batch, k)).astype(np.float32)
    y = G.gemv(qtype, t, torch.from_numpy(x).cuda(), n, k).cpu().numpy()
    assert O.rel_l2(y, O.matmul_f32(x, exp)) < GEMV_TOL


def _gemv_case(qtype, n, k, batch, seed, bias=False, xscale=1.0):
    rng = np.random.default_rng(seed)
    w = Q.random_weight(rng, n, k)
    packed = Q.encode(qtype, w)
    x = (rng.standard_normal((batch, k)) * xscale).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32) if bias else None
    t = G.repack(qtype, dev_bytes(packed), n, k)
    y = G.gemv(qtype, t, torch.from_numpy(x).cuda(), n, k,
               bias=None if b is None else torch.from_numpy(b).cuda()).cpu().numpy()
    ref = O.linear(x, qtype, packed, n, k, bias=b)
    return y, ref, O.linear_f64(x, qtype, packed, n, k, bias=b)


@pytest.mark.parametrize("qtype", ALL)
@pytest.mark.parametrize("batch", [1, 2, 3, 4, 5, 8, 16, 32])
def test_gemv_small_batches(qtype, batch):
    y, ref, ref64 = _gemv_case(qtype, 272, 1024, batch, seed=batch * 31 + qtype)
    assert O.rel_l2(y, ref) < GEMV_TOL
    # int8-digit activations (warp-MMA kernel): ~6.5e-5 for Gaussian x; fp16
    # activations (tensor-memory kernel, K-quants from batch 17): ~2e-4
    tc = batch >= 17 and qtype in (12, 13, 14)
    assert O.rel_l2(y, ref64) < (6e-4 if tc else 3e-4)


@pytest.mark.parametrize("qtype", ALL)
def test_gemv_bias_and_ragged_rows(qtype):
    y, ref, _ = _gemv_case(qtype, 1000, 768, 2, seed=77 + qtype, bias=True)
    assert O.rel_l2(y, ref) < GEMV_TOL


@pytest.mark.parametrize("xscale", [1e-30, 1e-3, 1e4, 1e30])
def test_gemv_activation_range(xscale):
    y, ref, _ = _gemv_case(12, 256, 512, 2, seed=3, xscale=xscale)
    assert np.all(np.isfinite(y))
    assert O.rel_l2(y, ref) < GEMV_TOL


@pytest.mark.parametrize("qtype,n,k", [(12, 4096, 4096), (12, 4096, 11008), (13, 4096, 11008), (14, 4096, 11008),
                                        (8, 4096, 4096), (2, 4096, 4096), (3, 11008, 4096), (6, 4096, 11008),
                                        (7, 4096, 4096)])
def test_gemv_llama_shapes(qtype, n, k):
    # full-size shapes exercise row groups split between CTAs (stream-K fixup)
    y, ref, _ = _gemv_case(qtype, n, k, 1, seed=n + k + qtype)
    assert O.rel_l2(y, ref) < GEMV_TOL


def test_gemv_grouped_mixed_types_is_deterministic():
    rng = np.random.default_rng(9)
    specs = [(12, 4096, 4096), (12, 1024, 4096), (14, 1024, 4096), (12, 4096, 4096),
             (12, 11008, 4096), (12, 11008, 4096), (14, 4096, 11008), (13, 1024, 4096),
             (2, 1024, 4096), (3, 512, 2048), (6, 768, 4096), (7, 1024, 1024), (8, 256, 4096)]
    batch = 4
    probs, refs = [], []
    for qt, n, k in specs:
        packed = Q.encode(qt, Q.random_weight(rng, n, k))
        x = rng.standard_normal((batch, k)).astype(np.float32)
        t = G.repack(qt, dev_bytes(packed), n, k)
        probs.append(G.GemvProblem(qt, t, torch.from_numpy(x).cuda(),
                                   torch.empty((batch, n), device="cuda"), n, k))
        refs.append(O.linear(x, qt, packed, n, k))
    G.gemv_grouped(probs)
    first = [p.y.clone() for p in probs]
    for p, r in zip(probs, refs):
        assert O.rel_l2(p.y.cpu().numpy(), r) < GEMV_TOL
    for _ in range(3):
        G.gemv_grouped(probs)
        for p, f in zip(probs, first):
            assert torch.equal(p.y, f)
    assert G.workspace_status() == 0
