"""The memory-lean per-partition builder gives the same graph, features, splits and
(up to bf16 rounding of the teacher) labels as the global builder."""
import pytest
import torch

from grappa_b200.dataset import synthetic as S
from grappa_b200.graph_store import partition_from_global


def _check(device):
    spec = S.SPECS["tiny"]
    g = S.build(spec, device)
    ref = partition_from_global(g, 1, 0, device, part_seed=spec.seed)  # world 1: ids unchanged
    for world in (1, 3):
        prefix = S.lean_prefix(spec.n_nodes, world)
        for rank in range(world):
            p = S.build_partition(spec, world, rank, device)
            lo, hi = prefix[rank], prefix[rank + 1]
            assert p.prefix == prefix and p.n_nodes == hi - lo
            e0, e1 = int(ref.indptr[lo]), int(ref.indptr[hi])
            assert torch.equal(p.indptr.cpu(), (ref.indptr[lo:hi + 1] - e0).cpu())
            assert torch.equal(p.indices.cpu(), ref.indices[e0:e1].cpu())
            assert torch.equal(p.gideg.cpu(), ref.gideg[lo:hi].cpu())
            assert torch.equal(p.feat.cpu(), ref.feat[lo:hi].cpu())
            for a, b in ((p.train_mask, ref.train_mask), (p.val_mask, ref.val_mask), (p.test_mask, ref.test_mask)):
                assert torch.equal(a.cpu(), b[lo:hi].cpu())
            agree = (p.label.cpu() == ref.label[lo:hi].cpu()).float().mean().item()
            assert agree > 0.95, agree
            ext = p.indices[(p.indices < lo) | (p.indices >= hi)]
            assert torch.equal(p.ext_src.cpu(), torch.unique(ext).to(torch.int32).cpu())


def test_lean_partition_matches_global_cpu():
    _check(torch.device("cpu"))


@pytest.mark.gpu
def test_lean_partition_matches_global_gpu():
    _check(torch.device("cuda", 0))
