"""Multilevel k-way partitioner (the ``metis`` method of the chunkers): balanced in node
count and training nodes, a lower edge cut than the hash partition, deterministic for a
seed, and usable by the sequential chunk builder."""
import numpy as np
import pytest

from grappa_b200 import _native
from grappa_b200.dataset import synthetic as S


@pytest.fixture(scope="module")
def graph():
    g = S.build(S.SPECS["rmat16k"], "cpu")
    return g, g.u.numpy().astype(np.int64), g.v.numpy().astype(np.int64), g.train_mask.numpy().astype(np.int8)


@pytest.mark.parametrize("k", [2, 4, 8])
def test_multilevel_partition_balance_and_cut(graph, k):
    g, u, v, tr = graph
    h = _native.host()
    n = g.n_nodes
    p = h.c_seq.multilevel_partition(n, u, v, k, tr, 3, 0.03)
    assert p.shape == (n,) and p.min() >= 0 and p.max() < k
    sizes = np.bincount(p, minlength=k)
    train = np.bincount(p, weights=tr, minlength=k)
    assert sizes.max() <= 1.03 * n / k + 1
    assert train.max() <= 1.03 * tr.sum() / k + 1
    cut = h.c_seq.edge_cut(n, u, v, p)
    hash_cut = h.c_seq.edge_cut(n, u, v, h.c_dist.random_assign_pid(n, k, 3))
    assert cut < (0.5 if k == 2 else 0.9) * hash_cut, (cut, hash_cut)
    assert np.array_equal(p, h.c_seq.multilevel_partition(n, u, v, k, tr, 3, 0.03))


def test_chunk_builder_metis(tmp_path):
    from grappa_b200.dataset.chunk_seq import build_chunks_seq

    g = S.build("tiny")
    S.to_t10n_layout(g, str(tmp_path / "src"))
    out, _ = build_chunks_seq(str(tmp_path), "tiny", str(tmp_path / "src"), "metis", 2)
    n = [np.fromfile(f"{out}/p{i}.train.bin", dtype=np.int8).size for i in range(2)]
    assert sum(n) == g.n_nodes and max(n) <= 1.03 * g.n_nodes / 2 + 1
