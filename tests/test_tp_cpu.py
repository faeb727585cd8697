"""Tensor-parallel sharding and collectives on CPU ranks (gloo), no GPU.

The GPU GEMV is replaced by the oracle's dequantize + matmul through the
layers' `local_matmul` hook, so these tests check the shard arithmetic
(packed-row and super-block splits, uneven ranges) and the all-gather /
all-reduce composition against the unsharded reference linear.
"""

import os
import socket

import numpy as np
import pytest
import torch

from dracort_b200.format import quantize as Q
from dracort_b200.parallel.tp import (
    ColumnParallelGGUFLinear,
    RowParallelGGUFLinear,
    TensorParallelConfig,
    even_split,
    partition_parameters,
    shard_k,
    shard_rows,
    split_tensor,
)
from oracle import gguf_oracle as O


def oracle_local(x, qtype, packed, n, k):
    w = torch.from_numpy(O.dequantize_matrix(qtype, packed, n, k))
    return x.float() @ w.T


def test_even_split_down_projection_super_blocks():
    # down: K = 11008 = 43 super-blocks (43 is prime: uneven at every TP size)
    assert [b - a for a, b in even_split(11008, 2, 256)] == [22 * 256, 21 * 256]
    assert [(b - a) // 256 for a, b in even_split(11008, 4, 256)] == [11, 11, 11, 10]
    assert [(b - a) // 256 for a, b in even_split(11008, 8, 256)] == [6, 6, 6, 5, 5, 5, 5, 5]
    assert [b - a for a, b in even_split(11008, 8, 16)] == [1376] * 8


@pytest.mark.parametrize("qtype", [8, 12, 14])
def test_shards_dequantize_to_slices_of_the_full_weight(qtype):
    rng = np.random.default_rng(qtype)
    n, k = 48, 256 * 5
    packed = Q.encode(qtype, Q.random_weight(rng, n, k))
    full = O.dequantize_matrix(qtype, packed, n, k)
    for world in (2, 3):
        rows = []
        for r in range(world):
            sh, r0, r1 = shard_rows(packed, qtype, n, k, r, world)
            np.testing.assert_array_equal(O.dequantize_matrix(qtype, sh, r1 - r0, k), full[r0:r1])
            rows.append((r0, r1))
            shk, k0, k1 = shard_k(packed, qtype, n, k, r, world)
            np.testing.assert_array_equal(O.dequantize_matrix(qtype, shk, n, k1 - k0), full[:, k0:k1])
        assert rows[0][0] == 0 and rows[-1][1] == n
    assert len(split_tensor(packed, qtype, n, k, 4, dim=1)) == 4


def test_partition_plan_follows_reference_rules():
    m = torch.nn.ModuleDict({"q_proj": torch.nn.Linear(4, 4), "o_proj": torch.nn.Linear(4, 4),
                             "down_proj": torch.nn.Linear(4, 4)})
    plan = partition_parameters(m, TensorParallelConfig())
    assert plan["q_proj.weight"] == ("column", 0)
    assert plan["o_proj.weight"] == ("row", 1)
    assert plan["down_proj.weight"] == ("row", 1)
    assert plan["q_proj.bias"] == ("replicate", -1)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(5)
        cfg = TensorParallelConfig(world_size=world, rank=rank, device="cpu")
        # gate-like (column) and down-like (row, 43 super-blocks: uneven shards)
        n_c, k_c = 96, 512
        n_r, k_r = 64, 11008
        pc = Q.encode(12, Q.random_weight(rng, n_c, k_c))
        pr = Q.encode(14, Q.random_weight(rng, n_r, k_r))
        bias = torch.from_numpy(rng.standard_normal(n_r).astype(np.float32))
        xc = torch.from_numpy(rng.standard_normal((3, k_c)).astype(np.float32))
        xr = torch.from_numpy(rng.standard_normal((3, k_r)).astype(np.float32))
        col = ColumnParallelGGUFLinear(12, pc, k_c, n_c, cfg, local_matmul=oracle_local)
        row = RowParallelGGUFLinear(14, pr, k_r, n_r, cfg, bias=bias, local_matmul=oracle_local)
        yc = col(xc).numpy()
        yr = row(xr).numpy()
        ref_c = O.linear(xc.numpy(), 12, pc, n_c, k_c)
        ref_r = O.linear(xr.numpy(), 14, pr, n_r, k_r, bias=bias.numpy())
        result_q.put((rank, O.rel_l2(yc, ref_c), O.rel_l2(yr, ref_r), row.k1 - row.k0))
    finally:
        dist.destroy_process_group()


def test_column_and_row_parallel_on_two_gloo_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    widths = sorted(w for _, _, _, w in res)
    assert widths == [21 * 256, 22 * 256]
    for _, ec, er, _ in res:
        assert ec < 1e-6 and er < 1e-6
