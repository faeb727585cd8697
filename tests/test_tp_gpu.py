"""Tensor-parallel decode on 2 GPUs (NCCL): sharded GEMV + all-gather / all-reduce
must reproduce the CPU oracle's fp32 linear layers of the unsharded layer set
(the GEMV bar, 1e-3 relative L2)."""

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available() or torch.cuda.device_count() < 2:  # pragma: no cover
    pytest.skip("needs 2 CUDA GPUs", allow_module_level=True)


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
        packed = encode_specs(specs, 77)
        layer = TPDecodeLayer(specs, packed, rank, world, 2, dev, seed=3, min_copies=1, l2_bytes=0)
        layer.step(0)
        torch.cuda.synchronize()
        outs = {k: v.cpu().numpy() for k, v in layer.outputs().items()}
        q.put((rank, outs, {k: v.cpu().numpy() for k, v in layer.x_full.items()}))
        layer.close()
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_tp2_decode_layer_matches_oracle():
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
    from oracle import gguf_oracle as O

    specs = layer_specs("q4_k_m")
    packed = encode_specs(specs, 77)
    _, _, xs0 = res[0]
    for rank, outs, xs in res:
        for s, p in zip(specs, packed):
            assert np.array_equal(xs[s.name], xs0[s.name])
            want = O.linear(xs[s.name], s.qtype, p, s.n_rows, s.k)
            assert O.rel_l2(outs[s.name], want) < 1e-3, (rank, s.name)
