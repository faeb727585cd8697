"""GPU parity of the tensor-memory decode GEMV (gemv_tc.cu): batches of 17..32
rows over Q4_K / Q5_K / Q6_K weights take the tcgen05 kernel.

Bars: <= 1e-3 relative L2 against the oracle's fp32 matmul (the decode rule).
The kernel carries activations as fp16 scaled per super-block (11 significant
bits) and Q6_K's sc * (q - 32) rounded to fp16: about 2e-4 relative L2 for
Gaussian activations, checked against the float64 oracle at 6e-4.
"""

import os
import subprocess
import sys

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
F64_TOL = 6e-4


def dev_bytes(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1)).cuda()


def _case(qtype, n, k, batch, seed, bias=False, xscale=1.0):
    rng = np.random.default_rng(seed)
    packed = Q.encode(qtype, Q.random_weight(rng, n, k))
    x = (rng.standard_normal((batch, k)) * xscale).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32) if bias else None
    t = G.repack(qtype, dev_bytes(packed), n, k)
    y = G.gemv(qtype, t, torch.from_numpy(x).cuda(), n, k,
               bias=None if b is None else torch.from_numpy(b).cuda()).cpu().numpy()
    return y, O.linear(x, qtype, packed, n, k, bias=b), O.linear_f64(x, qtype, packed, n, k, bias=b)


@pytest.mark.parametrize("qtype", [12, 13, 14])
@pytest.mark.parametrize("batch", [17, 20, 24, 31, 32])
def test_tc_gemv_batches(qtype, batch):
    y, ref, ref64 = _case(qtype, 272, 1024, batch, seed=batch * 13 + qtype)
    assert np.all(np.isfinite(y))
    assert O.rel_l2(y, ref) < GEMV_TOL
    assert O.rel_l2(y, ref64) < F64_TOL


@pytest.mark.parametrize("qtype", [12, 13, 14])
def test_tc_gemv_bias_and_ragged_rows(qtype):
    # 1000 rows: a ragged last row tile and a ragged last row group
    y, ref, _ = _case(qtype, 1000, 768, 20, seed=5 + qtype, bias=True)
    assert O.rel_l2(y, ref) < GEMV_TOL


@pytest.mark.parametrize("qtype,n,k", [(12, 4096, 4096), (14, 4096, 11008), (13, 11008, 4096), (12, 11008, 4096)])
def test_tc_gemv_llama_shapes(qtype, n, k):
    # full-size shapes: row groups split between CTAs (partials in CTA order)
    y, ref, ref64 = _case(qtype, n, k, 32, seed=n + k + qtype)
    assert O.rel_l2(y, ref) < GEMV_TOL
    assert O.rel_l2(y, ref64) < F64_TOL


@pytest.mark.parametrize("xscale", [1e-30, 1e-3, 1e4, 1e30])
def test_tc_gemv_activation_range(xscale):
    y, ref, _ = _case(12, 256, 512, 20, seed=3, xscale=xscale)
    assert np.all(np.isfinite(y))
    assert O.rel_l2(y, ref) < GEMV_TOL


def test_tc_gemv_outlier_and_zero_rows():
    # one batch row all zero, one with a single large outlier per super-block
    rng = np.random.default_rng(11)
    n, k, batch = 384, 1024, 20
    packed = Q.encode(12, Q.random_weight(rng, n, k))
    x = rng.standard_normal((batch, k)).astype(np.float32)
    x[3] = 0.0
    x[5, ::256] = 3e3
    t = G.repack(12, dev_bytes(packed), n, k)
    y = G.gemv(12, t, torch.from_numpy(x).cuda(), n, k).cpu().numpy()
    ref = O.linear(x, 12, packed, n, k)
    assert np.all(y[3] == 0.0)
    for b in range(batch):
        if b != 3:
            assert O.rel_l2(y[b], ref[b]) < GEMV_TOL


def test_tc_gemv_grouped_mixed_types_is_deterministic():
    rng = np.random.default_rng(21)
    specs = [(12, 4096, 4096), (14, 1024, 4096), (13, 1536, 4096), (12, 11008, 4096), (14, 4096, 11008)]
    batch = 32
    probs, refs = [], []
    for qt, n, k in specs:
        packed = Q.encode(qt, Q.random_weight(rng, n, k))
        x = rng.standard_normal((batch, k)).astype(np.float32)
        t = G.repack(qt, dev_bytes(packed), n, k)
        probs.append(G.GemvProblem(qt, t, torch.from_numpy(x).cuda(), torch.empty((batch, n), device="cuda"), n, k))
        refs.append(O.linear(x, qt, packed, n, k))
    G.gemv_grouped(probs)
    first = [p.y.clone() for p in probs]
    for _ in range(3):
        G.gemv_grouped(probs)
        for p, f in zip(probs, first):
            assert torch.equal(p.y, f)  # partials of split row groups are added in CTA order
    for p, r in zip(probs, refs):
        assert O.rel_l2(p.y.cpu().numpy(), r) < GEMV_TOL
    assert G.workspace_status() == 0


@pytest.mark.parametrize("mode", ["rmsnorm", "swiglu"])
def test_tc_gemv_fused_inputs(mode):
    rng = np.random.default_rng(31)
    n, k, batch, eps = 512, 2048, 24, 1e-5
    packed = Q.encode(12, Q.random_weight(rng, n, k))
    x = rng.standard_normal((batch, k)).astype(np.float32)
    t = G.repack(12, dev_bytes(packed), n, k)
    y = torch.empty((batch, n), device="cuda")
    if mode == "rmsnorm":
        w = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
        xin = x / np.sqrt((x.astype(np.float64) ** 2).mean(axis=1, keepdims=True) + eps) * w
        prob = G.GemvProblem(12, t, torch.from_numpy(x).cuda(), y, n, k, norm_weight=torch.from_numpy(w).cuda(),
                             norm_eps=eps)
    else:
        up = rng.standard_normal((batch, k)).astype(np.float32)
        xin = x / (1.0 + np.exp(-x.astype(np.float64))) * up
        prob = G.GemvProblem(12, t, torch.from_numpy(x).cuda(), y, n, k, up=torch.from_numpy(up).cuda())
    G.gemv_grouped([prob])
    ref = O.linear(xin.astype(np.float32), 12, packed, n, k)
    assert O.rel_l2(y.cpu().numpy(), ref) < GEMV_TOL


def test_tc_and_warp_mma_kernels_agree_with_the_oracle():
    """The same batch-32 launch through both kernels (the warp-MMA one forced by
    DRACO_GEMV_TC_MIN_BATCH=33 in a child process) is within tolerance of the
    oracle either way."""
    code = (
        "import numpy as np, torch, sys\n"
        "from dracort_b200 import gguf_ops as G\n"
        "from dracort_b200.format import quantize as Q\n"
        "rng = np.random.default_rng(4)\n"
        "p = Q.encode(12, Q.random_weight(rng, 2048, 4096))\n"
        "x = rng.standard_normal((32, 4096)).astype(np.float32)\n"
        "t = G.repack(12, torch.from_numpy(p.reshape(-1)).cuda(), 2048, 4096)\n"
        "y = G.gemv(12, t, torch.from_numpy(x).cuda(), 2048, 4096).cpu().numpy()\n"
        "np.save(sys.argv[1], y)\n"
    )
    outs = []
    for env_val, name in (("33", "mma"), ("17", "tc")):
        path = f"/tmp/draco_tc_ab_{name}_{os.getpid()}.npy"
        env = dict(os.environ, DRACO_GEMV_TC_MIN_BATCH=env_val)
        subprocess.run([sys.executable, "-c", code, path], check=True, env=env, timeout=300)
        outs.append(np.load(path))
        os.remove(path)
    rng = np.random.default_rng(4)
    p = Q.encode(12, Q.random_weight(rng, 2048, 4096))
    x = rng.standard_normal((32, 4096)).astype(np.float32)
    ref = O.linear(x, 12, p, 2048, 4096)
    for y in outs:
        assert O.rel_l2(y, ref) < GEMV_TOL
    assert not np.array_equal(outs[0], outs[1])  # two different kernels ran


def test_launch_count_query():
    """draco_gguf_gemv_launch_count matches the kernels each path launches."""
    rng = np.random.default_rng(2)

    def plan(specs, batch):
        probs = []
        for qt, n, k in specs:
            t = G.repack(qt, dev_bytes(Q.encode(qt, Q.random_weight(rng, n, k))), n, k)
            probs.append(G.GemvProblem(qt, t, torch.randn((batch, k), device="cuda"),
                                       torch.empty((batch, n), device="cuda"), n, k))
        return G.GemvPlan(probs)

    assert plan([(12, 512, 1024)], 1).launches == 1          # warp-MMA kernel alone
    # batch 1 with an RMSNorm input: the converter warps compute the row scale, no extra kernel
    t = G.repack(12, dev_bytes(Q.encode(12, Q.random_weight(rng, 512, 1024))), 512, 1024)
    normed = G.GemvPlan([G.GemvProblem(12, t, torch.randn((1, 1024), device="cuda"),
                                       torch.empty((1, 512), device="cuda"), 512, 1024,
                                       norm_weight=torch.ones(1024, device="cuda"))])
    assert normed.launches == 1
    normed.run()
    assert normed.status() == 0
    assert plan([(12, 512, 1024)], 4).launches == 2          # + activation conversion
    assert plan([(12, 512, 1024), (8, 256, 1024)], 32).launches == 2  # Q8_0 keeps the warp-MMA kernel
    big = plan([(12, 4096, 4096), (14, 4096, 11008)], 32)   # row groups split between CTAs
    assert big.launches == 3
    big.run()
    assert big.status() == 0


@pytest.mark.parametrize("batch", [1, 4, 32])
def test_accumulate_flag_adds_into_y(batch):
    """DRACO_GEMV_ACCUMULATE: y += x @ W^T + bias (the residual add of a layer),
    on the warp-MMA kernel (batch 1, 4) and the tensor-memory one (batch 32),
    including row groups split between CTAs."""
    from dracort_b200 import _native as N

    rng = np.random.default_rng(40 + batch)
    probs, refs = [], []
    for qt, n, k in [(12, 4096, 4096), (14, 1000, 768), (2, 512, 1024)]:
        packed = Q.encode(qt, Q.random_weight(rng, n, k))
        x = rng.standard_normal((batch, k)).astype(np.float32)
        y0 = rng.standard_normal((batch, n)).astype(np.float32)
        b = rng.standard_normal(n).astype(np.float32)
        t = G.repack(qt, dev_bytes(packed), n, k)
        probs.append(G.GemvProblem(qt, t, torch.from_numpy(x).cuda(), torch.from_numpy(y0).cuda(), n, k,
                                   bias=torch.from_numpy(b).cuda(), accumulate=True))
        refs.append((y0, O.linear(x, qt, packed, n, k, bias=b)))
    G.gemv_grouped(probs)
    for p, (y0, lin) in zip(probs, refs):
        assert O.rel_l2(p.y.cpu().numpy() - y0, lin) < GEMV_TOL
    # unknown flag bits and flags on the tensor-parallel entry are rejected
    s = G._to_struct(probs[0])
    s.flags = 2
    arr = (N.GemvProblem * 1)(s)
    assert N.load().draco_gguf_gemv_workspace_bytes(arr, 1, batch) == 0
    assert "flags" in N.last_error()
    s.flags = N.GEMV_ACCUMULATE
    arr = (N.GemvProblem * 1)(s)
    assert N.load().draco_gguf_gemv_grouped_tp(arr, 1, batch, None, None, 0, None) == N.DRACO_ERR_ARG
    assert "flags" in N.last_error()
