"""NVLink exchange buffers for the tensor-parallel decode step.

Every rank allocates one device buffer of the same size through the library
(cudaMalloc, zero-filled), exports it as a CUDA IPC handle, and maps every
other rank's buffer.  The handles travel once over the process group
(``all_gather_object``); after that the GEMV kernels store into the peers'
buffers directly and no host collective is involved.  This is the transport
behind the shard-boundary exchanges of draco/parallel/tp.py
(ColumnParallelLinear / RowParallelLinear, tp.py:120-183) on one box.
"""

from __future__ import annotations

import ctypes
from typing import List

from dracort_b200 import _native as N


class ExchangeBuffer:
    """This rank's exchange buffer and every peer's, mapped into this process."""

    def __init__(self, nbytes: int, rank: int, world: int, group=None) -> None:
        import torch.distributed as dist

        if not 2 <= world <= N.TP_MAX_WORLD:
            raise ValueError(f"exchange needs 2..{N.TP_MAX_WORLD} ranks, got {world}")
        self.rank, self.world, self.nbytes = rank, world, int(nbytes)
        self.group = group
        self._lib = N.load()
        own = ctypes.c_void_p()
        N.check(self._lib.draco_tp_buffer_alloc(self.nbytes, ctypes.byref(own)), "tp buffer")
        self.own = int(own.value)
        handle = (ctypes.c_char * N.IPC_HANDLE_BYTES)()
        N.check(self._lib.draco_ipc_get_handle(self.own, ctypes.cast(handle, ctypes.c_void_p)), "ipc handle")
        handles: List = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.ptrs: List[int] = []
        for q, h in enumerate(handles):
            if q == rank:
                self.ptrs.append(self.own)
                continue
            peer = ctypes.c_void_p()
            buf = (ctypes.c_char * N.IPC_HANDLE_BYTES).from_buffer_copy(h)
            N.check(self._lib.draco_ipc_open(ctypes.cast(buf, ctypes.c_void_p), ctypes.byref(peer)),
                    f"ipc open of rank {q}")
            self.ptrs.append(int(peer.value))
        self.closed = False

    def close(self) -> None:
        """Unmap the peers, wait until every rank has, then free the own buffer.
        Call it on every rank, with no kernel using the buffers in flight."""
        import torch
        import torch.distributed as dist

        if self.closed:
            return
        torch.cuda.synchronize()
        for q, p in enumerate(self.ptrs):
            if q != self.rank:
                N.check(self._lib.draco_ipc_close(p), "ipc close")
        dist.barrier(group=self.group)
        N.check(self._lib.draco_tp_buffer_free(self.own), "tp buffer free")
        self.closed = True
