"""The allocation-free GEMV entry point against the workspace entry point.

draco_gguf_gemv_grouped_noalloc serves callers that cannot allocate device
memory themselves (a host whose device memory belongs to another allocator,
a plain C / FFI host, a decode loop that cannot afford cudaMalloc's implicit
synchronisation): its scratch lives in a fixed array inside the library.
This test calls it through the C ABI twice in a row and compares each result
with draco_gguf_gemv_grouped given a caller-allocated workspace and with the
CPU oracle's fp32 linear layer, and reads the call's device status through
draco_gguf_gemv_noalloc_status.  Batch 3 is the case with a padded batch slot
in the in-kernel activation conversion, which only this entry point runs.
Its file name makes pytest collect it last, and it needs no state from other
tests.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from dracort_b200 import _native as N  # noqa: E402
from dracort_b200 import gguf_ops as G  # noqa: E402
from dracort_b200.format import quantize as Q  # noqa: E402
from oracle import gguf_oracle as O  # noqa: E402

GEMV_TOL = 1e-3  # relative L2, the bar every GEMV test uses


def _problems(batch, seed, with_packed=False):
    rng = np.random.default_rng(seed)
    specs = [(12, 1024, 4096), (14, 512, 4096), (8, 256, 1024), (12, 4096, 11008)]
    tensors, packs = [], []
    for qt, n, k in specs:
        packed = Q.encode(qt, Q.random_weight(rng, n, k))
        tiled = G.repack(qt, torch.from_numpy(packed.reshape(-1)).cuda(), n, k)
        x = torch.from_numpy(rng.standard_normal((batch, k)).astype(np.float32)).cuda()
        y_ref = torch.empty((batch, n), device="cuda")
        y_new = torch.empty((batch, n), device="cuda")
        tensors.append((qt, n, k, tiled, x, y_ref, y_new))
        packs.append(packed)
    return (tensors, packs) if with_packed else tensors


def _status(lib, stream):
    st = ctypes.c_int(-1)
    N.check(lib.draco_gguf_gemv_noalloc_status(ctypes.byref(st), stream))
    return st.value


def _struct(qt, n, k, tiled, x, y):
    s = N.GemvProblem()
    s.qtype, s.w, s.x, s.y, s.bias = qt, tiled.data_ptr(), x.data_ptr(), y.data_ptr(), None
    s.n_rows, s.k, s.ldx, s.ldy = n, k, x.stride(0), y.stride(0)
    return s


@pytest.mark.parametrize("batch", [1, 2, 3, 4])
def test_noalloc_matches_workspace_entry_point_twice(batch):
    lib = N.load()
    items, packs = _problems(batch, seed=100 + batch, with_packed=True)
    oracle = [O.linear(x.cpu().numpy(), qt, p, n, k) for (qt, n, k, _, x, _, _), p in zip(items, packs)]
    ref = (N.GemvProblem * len(items))(*[_struct(q, n, k, t, x, yr) for q, n, k, t, x, yr, _ in items])
    new = (N.GemvProblem * len(items))(*[_struct(q, n, k, t, x, yn) for q, n, k, t, x, _, yn in items])
    stream = torch.cuda.current_stream().cuda_stream

    ws_bytes = lib.draco_gguf_gemv_workspace_bytes(ref, len(items), batch)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    N.check(lib.draco_gguf_gemv_grouped(ref, len(items), batch, ws.data_ptr(), ws_bytes, stream))

    for _call in range(2):  # the shared array keeps the previous call's contents
        for it in items:
            it[6].fill_(float("nan"))
        N.check(lib.draco_gguf_gemv_grouped_noalloc(new, len(items), batch, stream))
        assert _status(lib, stream) == 0
        torch.cuda.synchronize()
        for (qt, n, k, tiled, x, y_ref, y_new), want in zip(items, oracle):
            got = y_new.cpu().numpy()
            assert np.isfinite(got).all()
            assert O.rel_l2(got, y_ref.cpu().numpy()) < GEMV_TOL
            assert O.rel_l2(got, want) < GEMV_TOL


def test_noalloc_rejects_batches_beyond_the_fixed_scratch():
    lib = N.load()
    items = _problems(5, seed=7)[:1]
    arr = (N.GemvProblem * 1)(_struct(*items[0][:5], items[0][6]))
    rc = lib.draco_gguf_gemv_grouped_noalloc(arr, 1, 5, torch.cuda.current_stream().cuda_stream)
    assert rc == N.DRACO_ERR_WORKSPACE
    assert "scratch" in N.last_error()
