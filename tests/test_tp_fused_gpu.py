"""Tensor-parallel GEMV with the in-kernel NVLink exchange.

* One GPU, two emulated ranks: rank 0's and rank 1's tensor-parallel GEMVs
  (draco_gguf_gemv_grouped_tp) run one after the other on one stream, each
  storing into both exchange buffers, then rank 0's draco_tp_finish gathers
  the column outputs and sums the row partials.  Nothing waits on another
  kernel of the GPU: the GEMVs never wait and the finish only reads flags
  that are already set.  Checked against the CPU oracle's fp32 linear layer
  of the unsharded weights, for several steps so both parity blocks are used.
* One GPU, a peer that never signals: the finish kernel's bounded wait runs
  out and reports DRACO_ERR_TIMEOUT (no GPU fault, no hang).
* Two GPUs (skipped on one): TPDecodeLayer(fused=True) over NCCL-free
  exchange against the CPU oracle's linear layers of the unsharded layer set.

Reference boundary: ColumnParallelLinear / RowParallelLinear
(draco/parallel/tp.py:120-183), whose all-reduce the reference leaves as a
comment (tp.py:182-183).
"""

import ctypes
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from dracort_b200 import _native as N  # noqa: E402
from dracort_b200 import gguf_ops as G  # noqa: E402
from dracort_b200.format import quantize as Q  # noqa: E402
from dracort_b200.parallel.tp import shard_k, shard_rows  # noqa: E402
from oracle import gguf_oracle as O  # noqa: E402

GEMV_TOL = 1e-3  # relative L2 against the oracle, the bar of every GEMV test

FLAGS_OFF, COUNTER_OFF, GATHER_OFF = 0, 128, 256


def _buffer(lib, nbytes):
    p = ctypes.c_void_p()
    N.check(lib.draco_tp_buffer_alloc(nbytes, ctypes.byref(p)))
    return int(p.value)


class _Emulated:
    """Two ranks' exchange buffers and problems on one GPU (layout as TPDecodeLayer's)."""

    def __init__(self, batch, seed):
        rng = np.random.default_rng(seed)
        self.lib = N.load()
        self.batch = B = batch
        # one column-parallel Q4_K weight and one row-parallel Q6_K weight
        self.nc, self.kc = 512, 1024
        self.nr, self.kr = 256, 2048
        self.wcol = Q.encode(12, Q.random_weight(rng, self.nc, self.kc))
        self.wrow = Q.encode(14, Q.random_weight(rng, self.nr, self.kr))
        self.xc = torch.from_numpy(rng.standard_normal((B, self.kc)).astype(np.float32)).cuda()
        self.xr = torch.from_numpy(rng.standard_normal((B, self.kr)).astype(np.float32)).cuda()
        self.wc = self.nc // 2  # column shard width per rank
        self.wr = self.nr      # row-parallel partials cover all rows
        self.g_stride = 2 * B * self.wc * 4
        self.r_off = (GATHER_OFF + 2 * self.g_stride + 255) // 256 * 256
        self.r_stride = 2 * B * self.wr * 4
        nbytes = (self.r_off + 2 * self.r_stride + 255) // 256 * 256
        self.bufs = [_buffer(self.lib, nbytes), _buffer(self.lib, nbytes)]
        self.keep = []
        self.ranks = [self._rank(r) for r in range(2)]

    def _rank(self, r):
        B = self.batch
        cs, _, _ = shard_rows(self.wcol, 12, self.nc, self.kc, r, 2)
        rs, k0, k1 = shard_k(self.wrow, 14, self.nr, self.kr, r, 2)
        tc = G.repack(12, torch.from_numpy(cs.reshape(-1)).cuda(), self.wc, self.kc)
        tr = G.repack(14, torch.from_numpy(rs.reshape(-1)).cuda(), self.nr, k1 - k0)
        xr = self.xr[:, k0:k1].contiguous()
        self.keep += [tc, tr, xr]
        arr = (N.GemvProblem * 2)()
        arr[0] = N.GemvProblem(12, 0, tc.data_ptr(), self.xc.data_ptr(), None, None, self.wc, self.kc, self.kc,
                               self.wc)
        arr[1] = N.GemvProblem(14, 0, tr.data_ptr(), xr.data_ptr(), None, None, self.nr, k1 - k0, k1 - k0, self.wr)
        ex = N.TpExchange()
        ex.world, ex.rank = 2, r
        # rank r sees its own buffer at [r]: the two buffers keep their rank slots
        ex.buffers[0], ex.buffers[1] = self.bufs[0], self.bufs[1]
        ex.flags_off, ex.counter_off = FLAGS_OFF, COUNTER_OFF
        ex.y_off[0] = GATHER_OFF + r * B * self.wc * 4
        ex.parity_stride[0] = self.g_stride
        ex.y_off[1] = self.r_off + r * B * self.wr * 4
        ex.parity_stride[1] = self.r_stride
        need = self.lib.draco_gguf_gemv_workspace_bytes(arr, 2, B)
        assert need > 0
        ws = torch.zeros(int(need), dtype=torch.uint8, device="cuda")
        return arr, ex, ws

    def gemv(self, r):
        arr, ex, ws = self.ranks[r]
        N.check(self.lib.draco_gguf_gemv_grouped_tp(arr, 2, self.batch, ctypes.byref(ex), ws.data_ptr(),
                                                      ws.numel(), torch.cuda.current_stream().cuda_stream))

    def finish(self, r, status):
        _, ex, _ = self.ranks[r]
        gout = torch.empty((2 * self.batch, self.wc), device="cuda")
        rout = torch.empty((self.batch, self.wr), device="cuda")
        N.check(self.lib.draco_tp_finish(ctypes.byref(ex), self.batch, GATHER_OFF, self.g_stride, self.wc,
                                         gout.data_ptr(), self.r_off, self.r_stride, self.wr, rout.data_ptr(),
                                         status.data_ptr(), torch.cuda.current_stream().cuda_stream))
        return gout, rout

    def references(self):
        """The oracle's fp32 linear layers of the unsharded weights (numpy)."""
        return (O.linear(self.xc.cpu().numpy(), 12, self.wcol, self.nc, self.kc),
                O.linear(self.xr.cpu().numpy(), 14, self.wrow, self.nr, self.kr))

    def close(self):
        torch.cuda.synchronize()
        for b in self.bufs:
            N.check(self.lib.draco_tp_buffer_free(b))


@pytest.mark.parametrize("batch", [1, 3, 8])  # 8: activations converted once per launch
def test_emulated_two_rank_exchange_matches_oracle(batch):
    em = _Emulated(batch, seed=batch)
    try:
        yc, yr = em.references()
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        for step in range(4):  # both parities, twice
            em.gemv(0)
            em.gemv(1)
            gout, rout = em.finish(0, status)
            torch.cuda.synchronize()
            assert int(status.item()) == 0, step
            g = gout.view(2, batch, em.wc)
            cols = torch.cat([g[0], g[1]], dim=1).cpu().numpy()
            assert O.rel_l2(cols, yc) < GEMV_TOL, step
            assert O.rel_l2(rout.cpu().numpy(), yr) < GEMV_TOL, step
            for _, _, ws in em.ranks:
                assert int(ws[:4].view(torch.int32).item()) == 0
    finally:
        em.close()


def test_finish_reports_timeout_when_a_peer_never_signals():
    em = _Emulated(1, seed=11)
    try:
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        em.gemv(0)  # rank 1 never runs: its flag stays unset
        em.finish(0, status)
        torch.cuda.synchronize()
        assert int(status.item()) == N.DRACO_ERR_TIMEOUT
    finally:
        em.close()


# ---------------------------------------------------------------------------
# two GPUs: the real layer over NVLink
# ---------------------------------------------------------------------------
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from dracort_b200.parallel.decode import TPDecodeLayer
    from dracort_b200.workloads import encode_specs, layer_specs

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        specs = layer_specs("q4_k_m")
        packed = encode_specs(specs, 78)
        layer = TPDecodeLayer(specs, packed, rank, world, 1, dev, seed=4, min_copies=2, l2_bytes=0, fused=True)
        steps = []
        for step in range(5):
            layer.step(step)
            torch.cuda.synchronize()
            steps.append({k: v.cpu().numpy() for k, v in layer.outputs().items()})
        xs = {k: v.cpu().numpy() for k, v in layer.x_full.items()}
        q.put((rank, steps, xs, layer.status()))
        layer.close()
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 CUDA GPUs")
def test_tp2_fused_exchange_matches_oracle():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    from dracort_b200.workloads import encode_specs, layer_specs

    specs = layer_specs("q4_k_m")
    packed = encode_specs(specs, 78)
    _, _, xs0, _ = res[0]
    want = {s.name: O.linear(xs0[s.name], s.qtype, p, s.n_rows, s.k) for s, p in zip(specs, packed)}
    for rank, steps, xs, st in res:
        assert st == 0, (rank, st)
        for step, outs in enumerate(steps):
            for name, ref in want.items():
                assert np.array_equal(xs[name], xs0[name])  # every rank holds the same activations
                assert O.rel_l2(outs[name], ref) < GEMV_TOL, (rank, step, name)
