"""The reference's native module API under ``t10n._C`` (csrc/python/pybind11.cc:59-130):
signatures and results over the engine, on the reference's own toy graph
(csrc/test/test_build_graph.cc:11-20)."""
import numpy as np
import pytest
import torch

import t10n  # noqa: F401  (installs the alias)
from t10n._C import c_dist, c_seq, graph, xborder

U = np.array([1, 2, 3, 4, 5, 100, 101, 101], dtype=np.int64)
V = np.array([10, 12, 200, 24, 200, 120, 200, 300], dtype=np.int64)


def test_host_graph_signatures():
    g2 = graph.HostGraph(U, V)
    g3 = graph.HostGraph(U, V, 0)  # third argument: the NUMA node, not a node count
    for g in (g2, g3):
        assert g.n_nodes == 301 and g.n_edges == 8
    assert np.array_equal(g2.indptr(), g3.indptr()) and np.array_equal(g2.indices(), g3.indices())
    gg = graph.GpuGraph(g2, device="cpu")
    assert torch.equal(gg.indptr, torch.from_numpy(g2.indptr())) and gg.n_nodes == 301


def test_host_sampler_batch_object():
    g = graph.HostGraph(U, V)
    seeds = np.array([200, 300, 10, 12, 24], dtype=np.int64)
    s = graph.HostSampler(g, [2, 2], False, True)  # (graph, fanouts, repeated, count_resampling)
    s.c_reinit_with_gideg_from(seeds, np.full(5, 3, dtype=np.int64), 5, -1)
    b = s.c_next_batch()
    assert isinstance(b, graph.Batch)
    layers, inputs = b.get_layers(), b.get_input_nodes()
    assert len(layers) == 4 and len(inputs) == 2
    u0, v0 = np.array(layers[0]), np.array(layers[1])
    assert set(v0.tolist()) <= set(seeds.tolist()) and len(u0) == len(v0)
    for a, bb in zip(u0, v0):  # every sampled edge is an edge of the graph
        assert ((U == a) & (V == bb)).any()
    assert inputs[0] == sorted(set(u0.tolist()))
    assert b.resampling.shape == (2,) and b.resampling[1] == 5
    with pytest.raises(StopIteration):
        s.c_next_batch()


def test_neighbor_sampler_and_fixture():
    g = graph.HostGraph(U, V)
    for repeated in (False, True):
        (u, v), cnt = graph.HostNeighborSampler(g, repeated).c_next_batch_py(np.array([200, 300], dtype=np.int64), 2)
        assert set(v.tolist()) == {200, 300} and cnt.size == 0
        if repeated:  # with replacement: exactly the fan-out per seed (300 has one in-neighbour)
            assert len(u) == 4 and u[v == 300].tolist() == [101, 101]
        else:  # without: min(degree, fan-out) distinct neighbours
            assert len(u) == 3 and len(set(zip(u.tolist(), v.tolist()))) == 3
    b = graph.py_test_batch()
    assert b.get_layers() == [[0, 1, 2], [0, 1, 2, 3, 4], [0, 1, 2], [0, 1, 2, 3, 4]]
    assert b.get_input_nodes() == [[0], [0, 1]]


def test_random_assign_pid_forms():
    whole = c_dist.random_assign_pid(30, 4)  # the engine's form
    for rank in range(3):
        sl = np.zeros(10, dtype=np.int32)
        assert c_dist.random_assign_pid(rank, sl, 4) is None  # the reference's in-place form
        assert np.array_equal(sl, whole[rank * 10:(rank + 1) * 10])
    with pytest.raises(ValueError):
        c_dist.random_assign_pid(10, 0)
    assert callable(c_seq.build) and callable(c_seq.split_node_feat)


def test_xborder_fill_v2():
    xb = xborder.XBorder(0, 2, [0, 3, 6])
    xb.set_nbr_idx(1)
    f0 = np.arange(6, dtype=np.float32).reshape(3, 2)
    f1 = 10 + np.arange(6, dtype=np.float32).reshape(3, 2)
    out = np.zeros((4, 2), dtype=np.float32)
    ids = np.array([4, 0, 2], dtype=np.int64)
    xb.ad_hoc_fill_batch_feat_v2(out, [f0, f1], ids, np.array([3, 0, 1], dtype=np.int64))
    assert np.array_equal(out[3], f1[1]) and np.array_equal(out[0], f0[0]) and np.array_equal(out[1], f0[2])
    assert not out[2].any()
