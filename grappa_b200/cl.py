"""Control-plane collectives (reference: t10n/cl.py:19-126).

Ragged exchanges of id lists and feature rows between ranks: counts first, then
payloads.  On GPUs they run on NCCL; on CPU ranks on gloo.  The training data
plane does not use them (it moves bytes with the peer-memory kernels); they
serve the CPU path, offline chunking and cross-partition inference on CPU ranks.
"""
import torch
import torch.distributed as dist


def _dev_for_backend(device):
    if dist.get_backend() == "nccl":
        return device if device is not None and torch.device(device).type == "cuda" else torch.device("cuda")
    return torch.device("cpu")


def total_mb(list_of_count_th, ele_size):
    """MiB carried by messages whose element counts are the first entries of
    ``list_of_count_th`` (reference: t10n/cl.py:11-16)."""
    return sum(float(c.reshape(-1)[0]) * ele_size for c in list_of_count_th) / 2**20


def t10n_gather_gloo(in_tensor, rank, world_size, dst_rank):
    """Gather ragged 1-D/2-D tensors to ``dst_rank`` (pad to the max length, then trim)."""
    assert torch.is_tensor(in_tensor) and in_tensor.dim() in (1, 2)

    def zeros(n):
        shape = (n,) if in_tensor.dim() == 1 else (n, in_tensor.shape[1])
        return torch.zeros(shape, dtype=in_tensor.dtype)

    mx = torch.tensor(in_tensor.shape[0], dtype=torch.int64)
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    ln = torch.tensor(in_tensor.shape[0], dtype=torch.int64)
    lens = [torch.tensor(0, dtype=torch.int64) for _ in range(world_size)] if rank == dst_rank else None
    dist.gather(ln, gather_list=lens, dst=dst_rank)
    padded = zeros(int(mx))
    padded[: in_tensor.shape[0]] = in_tensor
    bufs = [zeros(int(mx)) for _ in range(world_size)] if rank == dst_rank else None
    dist.gather(padded, gather_list=bufs, dst=dst_rank)
    out = None
    if rank == dst_rank:
        out = torch.cat([b[: int(l)] for b, l in zip(bufs, lens)])
    dist.barrier()
    return out


def _all_to_all(outs, ins):
    if dist.get_backend() == "gloo":
        # gloo has no all_to_all: emulate with point-to-point exchanges
        rank, world = dist.get_rank(), dist.get_world_size()
        reqs = []
        for p in range(world):
            if p == rank:
                outs[p].copy_(ins[p])
                continue
            reqs.append(dist.isend(ins[p].contiguous(), p))
            reqs.append(dist.irecv(outs[p], p))
        for r in reqs:
            r.wait()
    else:
        dist.all_to_all(outs, [t.contiguous() for t in ins])


def t10n_all_to_all_1d_int64_nccl(list_of_th_tensor, rank, world_size, device):
    """Exchange ragged int64 id lists: list_of_th_tensor[p] goes to rank p."""
    dev = _dev_for_backend(device)
    counts = [torch.tensor([t.shape[0]], dtype=torch.int64, device=dev) for t in list_of_th_tensor]
    got = [torch.zeros(1, dtype=torch.int64, device=dev) for _ in range(world_size)]
    _all_to_all(got, counts)
    outs = [torch.zeros(int(c.item()), dtype=torch.int64, device=dev) for c in got]
    _all_to_all(outs, [t.to(dev, torch.int64) for t in list_of_th_tensor])
    return outs


def t10n_all_to_all_2d_float32_nccl(list_of_th_tensor, rank, world_size, device, dim_2nd):
    """Exchange ragged fp32 row blocks [n_p, dim_2nd]."""
    dev = _dev_for_backend(device)
    ins = [t.reshape(-1, dim_2nd).to(dev, torch.float32) if t.numel() else
           torch.zeros((0, dim_2nd), dtype=torch.float32, device=dev) for t in list_of_th_tensor]
    counts = [torch.tensor([t.shape[0]], dtype=torch.int64, device=dev) for t in ins]
    got = [torch.zeros(1, dtype=torch.int64, device=dev) for _ in range(world_size)]
    _all_to_all(got, counts)
    outs = [torch.zeros((int(c.item()), dim_2nd), dtype=torch.float32, device=dev) for c in got]
    _all_to_all(outs, ins)
    return outs


# gloo names of the reference (stubs there); the implementations above handle both backends
t10n_all_to_all_1d_int64_gloo = t10n_all_to_all_1d_int64_nccl
t10n_all_to_all_2d_float32_gloo = t10n_all_to_all_2d_float32_nccl


class PeerAllToAll:
    """Ragged all-to-all of device tensors through NVLink peer memory (the GPU form of
    the exchanges above, t10n/cl.py:62-117): every rank copies its outgoing blocks into
    its peer-mapped send buffer and publishes its per-destination byte counts, a device
    barrier (grappa_b200/csrc/cuda/peer.cu, peer_barrier) makes them visible, and every
    rank pulls its incoming segments from the senders' buffers with one a2a_pull
    launch; a second barrier lets the senders reuse their buffers.  No NCCL call is on
    this path.  Collective: every rank calls ``exchange`` the same number of times."""

    def __init__(self, comm, device, timeout_s=30.0):
        from grappa_b200.parallel.comm import PeerBuffer

        self.comm = comm
        self.W, self.rank = comm.world, comm.rank
        self.device = torch.device(device)
        W = self.W
        # control page: barrier flags [W] u32 (256 B), then this rank's W outgoing byte counts
        # (int64 each, padded to 16 B so that every count is one a2a segment)
        self._ctl = PeerBuffer(comm, 256 + 16 * W)
        self._counts = self._ctl.tensor(torch.int64, [2 * W], offset_bytes=256)
        self._epoch = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.timeout_ns = int(timeout_s * 1e9)
        self._send = None
        self._cap = 0

    def _barrier(self):
        from grappa_b200 import _native

        _native.cuda().peer_barrier(self.rank, self.W, self._ctl.local, list(self._ctl.ptrs), self._epoch,
                                    self.timeout_ns, self.err)

    def _ensure(self, nbytes):
        from grappa_b200.parallel.comm import PeerBuffer

        need = int(self.comm.all_reduce_max([nbytes])[0])
        if need > self._cap or self._send is None:
            if self._send is not None:
                self._send.close()
            self._cap = max(4096, (need * 3 // 2 + 255) // 256 * 256)
            self._send = PeerBuffer(self.comm, self._cap)

    def exchange(self, parts):
        """parts[p] (a CUDA tensor; same dtype and trailing shape for every p) goes to rank
        p; returns the W received tensors (received[p] came from rank p)."""
        from grappa_b200 import _native

        cu = _native.cuda()
        W, r = self.W, self.rank
        ref = parts[0]
        tail = tuple(ref.shape[1:])
        row_bytes = ref.element_size() * int(torch.tensor(tail).prod().item()) if tail else ref.element_size()
        sizes = [int(t.numel()) * t.element_size() for t in parts]
        padded = [(s + 15) // 16 * 16 for s in sizes]
        offs = [0]
        for s in padded:
            offs.append(offs[-1] + s)
        self._ensure(offs[-1])
        send = self._send.tensor(torch.uint8, [self._cap])
        for p, t in enumerate(parts):
            if sizes[p]:
                send[offs[p]:offs[p] + sizes[p]].copy_(t.contiguous().view(-1).view(torch.uint8))
        self._counts.copy_(torch.tensor([[pd, sz] for pd, sz in zip(padded, sizes)], dtype=torch.int64).view(-1))
        self._barrier()
        # every sender's count row: 16 bytes per destination, the whole row of each peer
        rows = torch.empty((W, W, 2), dtype=torch.int64, device=self.device)
        cu.a2a_pull([self._ctl.ptrs[p] + 256 for p in range(W)], [0] * W, [16 * W] * W,
                    [16 * W * p for p in range(W)], rows.data_ptr(), (r + 1) % W)
        rows = rows.cpu()
        mat = rows[:, :, 0]  # mat[p][q]: padded bytes p sends to q
        true_bytes = [int(rows[p, r, 1]) for p in range(W)]
        src_off = [int(mat[p, :r].sum()) for p in range(W)]
        lens = [int(mat[p, r]) for p in range(W)]
        dst_off = [0]
        for ln in lens:
            dst_off.append(dst_off[-1] + ln)
        recv = torch.empty(max(16, dst_off[-1]), dtype=torch.uint8, device=self.device)
        cu.a2a_pull(list(self._send.ptrs), src_off, lens, dst_off[:-1], recv.data_ptr(), (r + 1) % W)
        self._barrier()
        if int(self.err.item()):
            raise RuntimeError("peer all-to-all: a device barrier timed out")
        out = []
        for p in range(W):
            n_rows = true_bytes[p] // row_bytes
            blk = recv[dst_off[p]:dst_off[p] + n_rows * row_bytes]
            out.append(blk.view(ref.dtype).view((n_rows,) + tail))
        return out

    def close(self):
        if self._send is not None:
            self._send.close()
            self._send = None
        self._ctl.close()
