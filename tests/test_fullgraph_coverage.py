"""Coverage weight of isolated full-graph training (CPU): with three partitions an own
node loses the in-edges whose sources lie in the third partition, so the partition's
c_r drops below 1; it must equal the mean per-node ratio recomputed from the global
edge list (the mini-batch path's formula, reference csrc/graph/sampling_h.h:97-116)."""
import torch

from grappa_b200 import _native
from grappa_b200.dataset import synthetic as S
from grappa_b200.graph_store import partition_from_global, working_graph_host
from grappa_b200.trainer import full_graph_blocks


def test_full_graph_coverage_three_partitions():
    W, seed = 3, 7
    g = S.build(S.SPECS["tiny"], "cpu")
    parts = [partition_from_global(g, W, r, "cpu", part_seed=seed) for r in range(W)]
    rank, nbr = 0, 1
    w = working_graph_host(parts, rank, nbr)
    fb = full_graph_blocks(w, 3, parts[rank])
    c_sum, c_n = fb.cov.tolist()
    # recomputation from the global graph: relabel as partition_from_global does
    n = g.n_nodes
    pid = torch.from_numpy(_native.host().c_dist.random_assign_pid(n, W, seed))
    order = torch.argsort(pid * n + torch.arange(n))
    new_id = torch.empty(n, dtype=torch.int64)
    new_id[order] = torch.arange(n)
    u, v = new_id[g.u], new_id[g.v]
    prefix = parts[0].prefix
    owner = torch.bucketize(u, torch.tensor(prefix[1:]), right=True)
    lo, hi = prefix[rank], prefix[rank + 1]
    gideg = torch.bincount(v, minlength=n)
    kept = torch.bincount(v[(owner == rank) | (owner == nbr)], minlength=n)
    train = parts[rank].train_mask.bool()
    ids = torch.arange(lo, hi)[train]
    r = ((kept[ids].float() + 1.0) / (gideg[ids].float() + 1.0)).clamp(max=1.0)
    assert c_n == float(train.sum())
    assert abs(c_sum - float(r.sum())) < 1e-3 * max(1.0, c_sum)
    assert c_sum / c_n < 0.95  # edges into the third partition are missing
    # with two partitions every in-edge of the own nodes is kept: c_r == 1
    parts2 = [partition_from_global(g, 2, r_, "cpu", part_seed=seed) for r_ in range(2)]
    fb2 = full_graph_blocks(working_graph_host(parts2, 0, 1), 3, parts2[0])
    s2, n2 = fb2.cov.tolist()
    assert abs(s2 - n2) < 1e-3


def test_full_graph_blocks_refill_in_place():
    """A repartition refills the block source in place when the new working graph fits
    its capacities: every buffer keeps its address (a captured step graph stays valid)
    and the live part equals a freshly built block source; the device counters carry
    the new sizes and the rows past them read as empty."""
    W, seed = 3, 7
    g = S.build(S.SPECS["tiny"], "cpu")
    parts = [partition_from_global(g, W, r, "cpu", part_seed=seed) for r in range(W)]
    cap_n = parts[0].n_nodes + max(p.n_nodes for p in parts)
    cap_e = parts[0].n_edges + max(p.n_edges for p in parts)
    fb = full_graph_blocks(working_graph_host(parts, 0, 1), 2, parts[0], cap_n, cap_e)
    ptrs = [t.data_ptr() for t in (fb.indptr[0], fb.indices[0], fb.labels, fb.row_mask, fb.cov, fb.cnt)]
    w2 = working_graph_host(parts, 0, 2)
    out = full_graph_blocks(w2, 2, parts[0], cap_n, cap_e, into=fb)
    assert out is fb
    assert ptrs == [t.data_ptr() for t in (fb.indptr[0], fb.indices[0], fb.labels, fb.row_mask, fb.cov, fb.cnt)]
    ref = full_graph_blocks(w2, 2, parts[0])
    n, E = ref.n, int(ref.cnt[1])
    assert fb.n == n and fb.cnt.tolist() == ref.cnt.tolist()
    assert torch.equal(fb.indptr[0][: n + 1], ref.indptr[0][: n + 1])
    assert torch.all(fb.indptr[0][n + 1:] == E)
    assert torch.equal(fb.indices[0][:E], ref.indices[0][:E])
    assert torch.equal(fb.labels[:n], ref.labels[:n]) and int(fb.row_mask[n:].sum()) == 0
    assert torch.equal(fb.row_mask[:n], ref.row_mask[:n]) and int(fb.n_sel) == int(ref.n_sel)
    assert torch.allclose(fb.cov, ref.cov)
    # a graph larger than the capacities gets a new block source
    small = full_graph_blocks(working_graph_host(parts, 0, 1), 2, parts[0])
    assert full_graph_blocks(working_graph_host(parts, 0, 2), 2, parts[0], into=small) is not small or \
        ref.n <= small.cap_dst[0]
