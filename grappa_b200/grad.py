"""Coverage-corrected gradient aggregation.

``weighted_grad_hook`` is the reference's DDP communication hook
(t10n/grad.py:6-24): every rank scales its gradient bucket by its coverage
weight c_r (the mean coverage ratio of the batch's seeds) and by 1/W, then the
buckets are summed with an all-reduce: g = sum_r c_r g_r / W.  It is kept as the
NCCL/gloo path (CPU training, and the baseline the fused kernel is compared with).

On GPUs the product path is the fused kernel of grappa_b200/csrc/cuda/allreduce.cu
(``grappa_b200.parallel.allreduce.FusedAllReduceAdam``), which does the scaling, the
all-reduce over NVLink peer memory and Adam in one launch per gradient bucket.
"""
from typing import Tuple, cast

import torch
import torch.distributed as dist


def weighted_grad_hook(state, bucket):
    group = dist.group.WORLD
    world = group.size()
    buf = cast(Tuple[torch.Tensor, ...], bucket)[0] if isinstance(bucket, tuple) else bucket.buffer()
    buf.mul_(float(state["coarse_count"])).div_(float(world))
    fut = dist.all_reduce(buf, async_op=True).get_future()
    return fut.then(lambda f: f.value()[0])


def coverage_all_reduce(params, coverage, world=None):
    """Apply the same aggregation to plain parameter gradients (no DDP wrapper)."""
    world = world or (dist.get_world_size() if dist.is_initialized() else 1)
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1) for g in grads])
    flat.mul_(float(coverage) / world)
    if world > 1:
        dist.all_reduce(flat)
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off:off + n].view_as(g))
        off += n
