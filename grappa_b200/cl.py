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
