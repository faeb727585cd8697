"""Tensor-parallel decode on 2 GPUs (NCCL): sharded GEMV + all-gather / all-reduce
must reproduce the single-GPU GEMV of the unsharded layer set."""

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

    from dracort_b200 import gguf_ops as G
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
        outs = layer.outputs()
        errs = {}
        for s, p in zip(specs, packed):
            t = G.repack(s.qtype, torch.from_numpy(p.reshape(-1)).to(dev), s.n_rows, s.k)
            ref = G.gemv(s.qtype, t, layer.x_full[s.name], s.n_rows, s.k)
            got = outs[s.name]
            errs[s.name] = float((got - ref).norm() / ref.norm())
        q.put((rank, errs))
        layer.close()
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_tp2_decode_layer_matches_single_gpu():
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
    for rank, errs in res:
        for name, e in errs.items():
            # sharding changes only the k ranges of the activation groups and the
            # summation order: both results are within the GEMV error budget
            assert e < 5e-4, (rank, name, e)
