"""CPU tests of the C++ host engine (grappa_b200._C): CSC build, sampling rule,
coverage counter, compaction order, pipelined sampler, XBorder, chunk writer."""
import os

import numpy as np
import pytest

from grappa_b200 import host

G = host().graph


def small_graph(n=500, m=6000, seed=0, hubs=True):
    rng = np.random.default_rng(seed)
    u = rng.integers(0, n, m)
    v = rng.integers(0, n, m)
    if hubs:
        v[: m // 4] = rng.integers(0, 5, m // 4)  # a few high-degree destinations
    u2 = np.concatenate([u, v, np.arange(n)])
    v2 = np.concatenate([v, u, np.arange(n)])
    return u2, v2, n


def test_build_csc_dedups_and_sorts():
    u = np.array([1, 2, 3, 1, 1, 0, 2], dtype=np.int64)
    v = np.array([0, 0, 0, 0, 2, 2, 2], dtype=np.int64)
    g = G.HostGraph(u, v, 4)
    assert g.indptr().tolist() == [0, 3, 3, 6, 6]
    assert g.indices().tolist() == [1, 2, 3, 0, 1, 2]


def test_pick_offsets_distinct_and_uniform():
    d, k = 40, 15
    counts = np.zeros(d)
    for nid in range(4000):
        o = G.pick_offsets(123, nid, d, k)
        assert len(set(o.tolist())) == k
        assert o.min() >= 0 and o.max() < d
        counts[o] += 1
    expected = 4000 * k / d
    assert np.all(np.abs(counts - expected) < 6 * np.sqrt(expected))


def test_pick_offsets_near_full():
    for nid in range(200):
        o = G.pick_offsets(7, nid, 17, 16)
        assert len(set(o.tolist())) == 16


def test_sample_batch_semantics():
    u, v, n = small_graph()
    g = G.HostGraph(u, v, n)
    ip, ix = g.indptr(), g.indices()
    seeds = np.arange(0, 300, 3, dtype=np.int64)
    gideg = np.full(len(seeds), 40, dtype=np.int64)
    blocks, cov_sum, cov_n = G.sample_batch(g, [15, 10, 5], seeds, gideg, 11, 2, 3, False)
    assert cov_n == len(seeds)
    exp = sum(G.coverage_ratio(int(ip[s + 1] - ip[s]), 40) for s in seeds)
    assert abs(cov_sum - exp) < 1e-3
    fan = [5, 10, 15]
    dst = seeds
    front = None
    for h, b in enumerate(blocks):
        assert b["n_dst"] == len(dst)
        assert np.array_equal(b["src_nid"][: b["n_dst"]], dst)
        src = b["src_nid"]
        assert len(set(src.tolist())) == len(src)
        for i in range(b["n_dst"]):
            deg = ip[dst[i] + 1] - ip[dst[i]]
            picked = b["indptr"][i + 1] - b["indptr"][i]
            want = 0 if (front is not None and not front[i]) else min(deg, fan[h])
            assert picked == want
            nb = set(ix[ip[dst[i]]:ip[dst[i] + 1]].tolist())
            got = src[b["indices"][b["indptr"][i]:b["indptr"][i + 1]]]
            assert set(got.tolist()) <= nb and len(set(got.tolist())) == picked
        # new sources appear in order of first appearance
        seen, order = set(dst.tolist()), []
        for e in range(len(b["indices"])):
            x = src[b["indices"][e]]
            if x not in seen:
                seen.add(x)
                order.append(x)
        assert order == src[b["n_dst"]:].tolist()
        marked = np.zeros(b["n_src"], dtype=bool)
        marked[b["indices"]] = True
        assert np.array_equal(marked, b["src_sampled"].astype(bool))
        dst, front = src, b["src_sampled"]


def test_host_sampler_pipeline_matches_direct():
    u, v, n = small_graph(seed=3)
    g = G.HostGraph(u, v, n)
    targets = np.arange(100, dtype=np.int64)
    gideg = np.full(100, 10, dtype=np.int64)
    s = G.HostSampler(g, [10, 5], False, True, 5)
    s.reinit(targets, gideg, 32, -1, 4)
    for step in range(4):
        seeds, blocks, cs, cn = s.next_batch()
        lo = step * 32
        ref_blocks, rcs, rcn = G.sample_batch(g, [10, 5], targets[lo:lo + 32], gideg[lo:lo + 32], 5, 4, step, False)
        assert np.array_equal(seeds, targets[lo:lo + 32])
        for a, b in zip(blocks, ref_blocks):
            assert np.array_equal(a["indices"], b["indices"]) and np.array_equal(a["src_nid"], b["src_nid"])
        assert abs(cs - rcs) < 1e-6 and cn == rcn
    with pytest.raises(StopIteration):
        s.next_batch()


def test_host_sampler_restart_mid_epoch():
    """A reinit while the worker still has batches queued ends that epoch; the new one
    starts from its own first batch (the epoch number keys the draws)."""
    u, v, n = small_graph(seed=5)
    g = G.HostGraph(u, v, n)
    targets = np.arange(200, dtype=np.int64)
    s = G.HostSampler(g, [6, 3], False, False, 9)
    s.reinit(targets, None, 20, -1, 0)
    s.next_batch()
    s.reinit(targets[::-1].copy(), None, 20, -1, 7)
    assert s.epoch == 7
    seeds, blocks, _, _ = s.next_batch()
    assert np.array_equal(seeds, targets[::-1][:20])
    ref_blocks, _, _ = G.sample_batch(g, [6, 3], targets[::-1][:20].copy(), None, 9, 7, 0, False)
    for a, b in zip(blocks, ref_blocks):
        assert np.array_equal(a["indices"], b["indices"])
    for _ in range(9):
        s.next_batch()
    with pytest.raises(StopIteration):
        s.next_batch()
    s.reinit(targets, None, 50, 2, -1)  # epoch -1: the next epoch number
    assert s.epoch == 8
    assert len(s.next_batch()[0]) == 50 and len(s.next_batch()[0]) == 50
    with pytest.raises(StopIteration):
        s.next_batch()
    with pytest.raises(ValueError):
        s.reinit(targets, None, 0, -1, 0)


def test_reference_style_coo_output():
    u, v, n = small_graph(seed=4)
    g = G.HostGraph(u, v, n)
    s = G.HostSampler(g, [4, 3], False, True, 1)
    s.c_reinit_with_gideg_from(np.arange(20, dtype=np.int64), np.full(20, 5, dtype=np.int64), 10, 2)
    layers, correct = s.c_next_batch_py()
    assert len(layers) == 4 and len(correct) == 2 and correct[1] == 10


def test_with_replacement():
    u, v, n = small_graph(seed=5)
    g = G.HostGraph(u, v, n)
    blocks, _, _ = G.sample_batch(g, [8], np.arange(50, dtype=np.int64), None, 1, 0, 0, True)
    b = blocks[0]
    ip = g.indptr()
    for i in range(50):
        deg = ip[i + 1] - ip[i]
        assert b["indptr"][i + 1] - b["indptr"][i] == (0 if deg == 0 else 8)


def test_xborder_group_and_fill():
    X = host().xborder.XBorder
    prefix = [0, 10, 25, 40, 50]
    xb = X(1, 4, prefix)
    ids = np.array([3, 12, 27, 45, 11, 30, 0], dtype=np.int64)
    mask = np.zeros((4, len(ids)), dtype=np.int8)
    groups = xb.group_by_partition(ids, mask)
    assert [g.tolist() for g in groups] == [[3, 0], [12, 11], [27, 30], [45]]
    assert mask.sum() == len(ids) and mask[1, 1] == 1
    xb.set_nbr_idx(2)
    xb.ad_hoc_build_id_mapping(0, np.array([0, 3], dtype=np.int64))
    xb.ad_hoc_build_id_mapping(3, np.array([45], dtype=np.int64))
    tables = [np.array([[100.0], [103.0]], dtype=np.float32),
              np.arange(15, dtype=np.float32).reshape(15, 1) + 10,
              np.arange(15, dtype=np.float32).reshape(15, 1) + 25,
              np.array([[45.0]], dtype=np.float32)]
    out = np.zeros((len(ids), 1), dtype=np.float32)
    xb.ad_hoc_fill_batch_feat(out, tables, ids)
    assert out[:, 0].tolist() == [103.0, 12.0, 27.0, 45.0, 11.0, 30.0, 100.0]


def test_chunk_layout_roundtrip(tmp_path):
    u, v, n = small_graph(n=200, m=1500, seed=6, hubs=False)
    keep = u != v
    u, v = u[keep], v[keep]
    n_part = 3
    pid = host().c_dist.random_assign_pid(n, n_part, 9)
    st = host().c_seq.build(str(tmp_path), n, len(u), 8, n_part, u, v, pid)
    feat = np.random.default_rng(0).standard_normal((n, 8)).astype(np.float32)
    host().c_seq.split_node_feat(str(tmp_path), n, 8, n_part, feat)
    lab = np.arange(n, dtype=np.float32)
    msk = (np.arange(n) % 2).astype(np.int8)
    host().c_seq.split_node_data(str(tmp_path), n, n_part, lab, msk, 1 - msk, msk)
    total_nodes, intra, bridge = 0, 0, 0
    for p in range(n_part):
        oid = np.fromfile(os.path.join(tmp_path, f"p{p}.oid.bin"), dtype=np.int64)
        assert np.all(pid[oid] == p) and np.all(np.diff(oid) > 0)
        total_nodes += len(oid)
        pu = np.fromfile(os.path.join(tmp_path, f"p{p}.u.bin"), dtype=np.int64)
        assert np.array_equal(pu[-len(oid):], np.arange(len(oid)))  # appended self-loops
        intra += len(pu) - len(oid)
        f = np.fromfile(os.path.join(tmp_path, f"p{p}.nfeat.bin"), dtype=np.float32).reshape(-1, 8)
        assert np.allclose(f, feat[oid])
        lb = np.fromfile(os.path.join(tmp_path, f"p{p}.label.bin"), dtype=np.float32)
        assert np.array_equal(lb, oid.astype(np.float32))
        tr = np.fromfile(os.path.join(tmp_path, f"p{p}.train.bin"), dtype=np.int8)
        assert len(tr) == len(oid)
        ideg = np.fromfile(os.path.join(tmp_path, f"p{p}.ideg.bin"), dtype=np.int64)
        assert np.array_equal(ideg, np.bincount(v, minlength=n)[oid])
        for q in range(n_part):
            if q == p:
                continue
            fu = os.path.join(tmp_path, f"b{p}_{q}.u.bin")
            if os.path.isfile(fu):
                bridge += len(np.fromfile(fu, dtype=np.int64))
    assert total_nodes == n
    assert intra + bridge == len(u)
    assert sum(st["part_nodes"]) == n


def test_dropout_mask_rate():
    m = host().dropout_mask(1, 2, 3, 0, 64, 256, 256, 0.5)
    assert abs(m.mean() - 0.5) < 0.02
    m2 = host().dropout_mask(1, 2, 3, 0, 64, 256, 256, 0.5)
    assert np.array_equal(m, m2)


def test_rmat_candidates_deterministic():
    a = G.rmat_candidates(1000, 10, 0.57, 0.19, 0.19, 3, 0, 5000)
    b = G.rmat_candidates(1000, 10, 0.57, 0.19, 0.19, 3, 100, 5000)
    assert np.array_equal(a[100:], b[:4900])
    valid = a[a >= 0]
    assert len(valid) > 2000 and np.all(valid // 1000 < valid % 1000)


def test_dropout_mask_byte_resolution():
    """Byte-resolution masks: the probability is quantised to 1/256 (p and p + 1/1024 give
    the same mask), the keep rate follows the quantised p, and element (r, c) of a
    buffer with row stride ld is the element r * ld + c of the flat mask (so the mask of
    a row does not depend on where the 16-element draw groups start)."""
    import numpy as np

    a = np.asarray(host().dropout_mask(5, 1, 2, 3, 40, 100, 104, 0.2))
    b = np.asarray(host().dropout_mask(5, 1, 2, 3, 40, 100, 104, 0.2 + 1.0 / 1024))
    assert np.array_equal(a, b)
    q = round(0.2 * 256) / 256
    assert abs(a.mean() - (1 - q)) < 0.02
    flat = np.asarray(host().dropout_mask(5, 1, 2, 3, 1, 40 * 104, 40 * 104, 0.2)).reshape(40, 104)[:, :100]
    assert np.array_equal(a.reshape(40, 100), flat)
    assert abs(np.asarray(host().dropout_mask(5, 1, 2, 3, 64, 256, 256, 0.5)).mean() - 0.5) < 0.01
