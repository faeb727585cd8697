"""GEMV parity at full layer sizes, where every CTA's slab range is several
times longer than its shared-memory stage ring, so the ring wraps many times.

The stage count follows from the stage size: 6 for Q6_K and 8 for Q4_K
weights at batch 1-4, 5 for Q8_0 at batch 1 (each stage 8 x 4352 B of
weights), 5 for a Q6_K set at batch 9-16 and 3 at batch 17-32.  With an odd
count a stage alternates between the even-slab and odd-slab consumer warps;
these cases cover that schedule, the mixed Q4_K / Q6_K grouped launch of a
Llama-7B Q4_K_M layer (config 4) and every batch-size class of the kernel.
Bar: 1e-3 relative L2 against the oracle's fp32 matmul (generic.py:32-33) on
its dequantized weights (gguf.py:272-497).
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
from dracort_b200.workloads import encode_specs, layer_specs  # noqa: E402

GEMV_TOL = 1e-3


@pytest.fixture(scope="module")
def q4_k_m_layer():
    specs = layer_specs("q4_k_m")
    packed = encode_specs(specs, 21)
    tiled = [G.repack(s.qtype, torch.from_numpy(p.reshape(-1)).cuda(), s.n_rows, s.k) for s, p in zip(specs, packed)]
    dense = [O.dequantize_matrix(s.qtype, p, s.n_rows, s.k) for s, p in zip(specs, packed)]
    return specs, tiled, dense


@pytest.mark.parametrize("batch", [1, 2, 3, 8, 16, 32])
def test_grouped_q4_k_m_layer_set(q4_k_m_layer, batch):
    specs, tiled, dense = q4_k_m_layer
    rng = np.random.default_rng(batch)
    xs = [rng.standard_normal((batch, s.k)).astype(np.float32) for s in specs]
    probs = [G.GemvProblem(s.qtype, t, torch.from_numpy(x).cuda(), torch.empty((batch, s.n_rows), device="cuda"),
                           s.n_rows, s.k) for s, t, x in zip(specs, tiled, xs)]
    plan = G.GemvPlan(probs)
    plan.run()
    assert plan.status() == 0
    first = [p.y.clone() for p in probs]
    for s, p, x, w in zip(specs, probs, xs, dense):
        assert O.rel_l2(p.y.cpu().numpy(), O.matmul_f32(x, w)) < GEMV_TOL, s.name
    for _ in range(3):  # back-to-back launches (programmatic dependent launch)
        plan.run()
    assert plan.status() == 0
    for p, f in zip(probs, first):
        assert torch.equal(p.y, f)


@pytest.mark.parametrize("batch", [1, 32])
def test_q8_0_odd_stage_ring(batch):
    n, k = 4096, 11008
    rng = np.random.default_rng(5 + batch)
    packed = Q.encode(8, Q.random_weight(rng, n, k))
    x = rng.standard_normal((batch, k)).astype(np.float32)
    t = G.repack(8, torch.from_numpy(packed.reshape(-1)).cuda(), n, k)
    y = G.gemv(8, t, torch.from_numpy(x).cuda(), n, k).cpu().numpy()
    assert G.workspace_status() == 0
    assert O.rel_l2(y, O.matmul_f32(x, O.dequantize_matrix(8, packed, n, k))) < GEMV_TOL
