"""Process-group plumbing and peer-mapped device buffers.

One process per GPU; ``torch.distributed`` (NCCL on GPUs, gloo on CPU) is used
for bootstrap and small control messages only.  Bulk data moves through buffers
that every rank maps into its address space with CUDA IPC, so kernels can load
and store a peer's HBM directly over NVLink 5 / NVSwitch.
"""
import datetime
import os

import torch
import torch.distributed as dist

from grappa_b200 import _native


def init_distributed(backend=None, timeout_s=600):
    """Initialise torch.distributed from the torchrun environment (no-op for one process)."""
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29511")
        if backend == "nccl":
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
    return rank, world


class Comm:
    """Rank/world of the job plus helpers for small host-side exchanges."""

    def __init__(self, group=None):
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.rank = dist.get_rank(group)
            self.world = dist.get_world_size(group)
        else:
            self.rank, self.world = 0, 1

    def all_gather_object(self, obj):
        if self.world == 1:
            return [obj]
        out = [None] * self.world
        dist.all_gather_object(out, obj, group=self.group)
        return out

    def barrier(self):
        if self.world > 1:
            dist.barrier(group=self.group)

    def all_reduce_max(self, values):
        return self._all_reduce(values, dist.ReduceOp.MAX)

    def all_reduce_sum(self, values):
        return self._all_reduce(values, dist.ReduceOp.SUM)

    def _all_reduce(self, values, op):
        t = torch.tensor(values, dtype=torch.float64)
        if self.world > 1:
            if dist.get_backend(self.group) == "nccl":
                t = t.cuda()
            dist.all_reduce(t, op=op, group=self.group)
        return [float(x) for x in t.cpu().tolist()]


class PeerBuffer:
    """A device buffer allocated on every rank and mapped into every other rank.

    ``ptrs[p]`` is the address of rank p's buffer in this process (its own
    allocation for p == rank, a CUDA IPC mapping otherwise).  Collective: every
    rank must create the same buffers in the same order; sizes may differ.
    """

    def __init__(self, comm, nbytes):
        self.comm = comm
        self.nbytes = int(nbytes)
        cu = _native.cuda()
        self.local = cu.peer_alloc(self.nbytes)
        handle = cu.ipc_handle(self.local) if comm.world > 1 else b""
        handles = comm.all_gather_object(bytes(handle))
        self.sizes = comm.all_gather_object(self.nbytes)
        self.ptrs = []
        for p, h in enumerate(handles):
            self.ptrs.append(self.local if p == comm.rank else cu.ipc_open(h))
        self._open = True

    def tensor(self, dtype, shape, offset_bytes=0, rank=None):
        """A tensor view of (a peer's) buffer; peers' views are for kernel arguments only."""
        rank = self.comm.rank if rank is None else rank
        dev = torch.cuda.current_device()
        return _native.cuda().tensor_from_ptr(self.ptrs[rank] + offset_bytes, list(shape), dtype, dev)

    def close(self):
        if not self._open:
            return
        cu = _native.cuda()
        torch.cuda.synchronize()
        self.comm.barrier()
        for p, ptr in enumerate(self.ptrs):
            if p != self.comm.rank:
                cu.ipc_close(ptr)
        cu.peer_free(self.local)
        self._open = False
