"""Dataset conversion with the reference's function names, on small directories in the
downloaded layouts: OGB (csv.gz and the papers100M npz form), DGL's Reddit files and
the IGB release (linked arrays, row-pair edges), then chunked by both chunkers."""
import gzip
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from grappa_b200.dataset import dgl_to_t10n as cv
from grappa_b200.dataset import partition
from grappa_b200.dataset.io_dist import DatasetIO, pfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
N, M, D = 300, 2000, 8


def _graph(seed=0):
    rng = np.random.default_rng(seed)
    src = rng.integers(0, N, M)
    dst = rng.integers(0, N, M)
    src[:5] = dst[:5]  # a few self-loops, replaced by one per node in the layout
    feat = rng.standard_normal((N, D)).astype(np.float32)
    label = rng.integers(0, 5, N).astype(np.float32)
    return src, dst, feat, label


def _csv_gz(path, arr):
    with gzip.open(path, "wt") as f:
        for row in np.atleast_2d(arr.T).T if arr.ndim == 2 else arr.reshape(-1, 1):
            f.write(",".join(str(x) for x in np.atleast_1d(row)) + "\n")


def _splits(d, scheme):
    os.makedirs(os.path.join(d, "split", scheme), exist_ok=True)
    for name, idx in (("train", np.arange(0, 150)), ("valid", np.arange(150, 200)), ("test", np.arange(200, N))):
        _csv_gz(os.path.join(d, "split", scheme, f"{name}.csv.gz"), idx)


def _check_layout(cfg_path, src, dst, feat, label, augmented=True):
    cfg = json.load(open(cfg_path))
    io = DatasetIO(os.path.dirname(cfg_path), os.path.dirname(cfg_path))
    u, v = (t.numpy() for t in io.read_edge(0, io.num_edges()))
    if augmented:
        keep = src != dst
        want = set(zip(src[keep].tolist(), dst[keep].tolist())) | {(i, i) for i in range(N)}
        assert set(zip(u.tolist(), v.tolist())) == want
        assert int((u == v).sum()) == N
    else:
        assert np.array_equal(u, src) and np.array_equal(v, dst)
    assert np.array_equal(io.read("node_feats_file_bin", 0, N).numpy(), feat)
    assert np.array_equal(io.read("node_label_file", 0, N).numpy(), label)
    assert cfg["num_nodes"] == N and cfg["feat_dim"] == D and cfg["num_labels"] == len(np.unique(label))
    return cfg


def test_ogb_csv_through_graph_arrays(tmp_path):
    src, dst, feat, label = _graph(1)
    d = tmp_path / "dl" / "ogbn_products"
    os.makedirs(d / "raw")
    _csv_gz(str(d / "raw" / "edge.csv.gz"), np.stack([src, dst], 1))
    _csv_gz(str(d / "raw" / "node-feat.csv.gz"), feat)
    _csv_gz(str(d / "raw" / "node-label.csv.gz"), label.astype(np.int64))
    _splits(str(d), "sales_ranking")
    g = cv.load_as_dgl_g(str(tmp_path / "dl"), "ogbpr")
    assert g.num_nodes() == N and g.num_edges() == M and int(g.ndata["train_mask"].sum()) == 150
    aug = cv.augmentation_dgl_g(g)
    au, av = (t.numpy() for t in aug.edges())
    assert int((au == av).sum()) == N
    cfg_path = cv.to_t10n_from_dgl_g(str(tmp_path / "t10n"), "ogbpr", g)
    cfg = _check_layout(cfg_path, src, dst, feat.astype(np.float32), label)
    assert cfg["num_train_nodes"] == 150
    assert cv.get_num_labels(np.array([0, 1, np.nan, 1, 4])) == 3


def test_papers100m_npz_form(tmp_path):
    src, dst, feat, label = _graph(2)
    d = tmp_path / "dl" / "ogbn_papers100M"
    os.makedirs(d / "raw")
    np.savez(d / "raw" / "data.npz", edge_index=np.stack([src, dst]), node_feat=feat, num_nodes_list=np.array([N]),
             num_edges_list=np.array([M]))
    np.savez(d / "raw" / "node-label.npz", node_label=label.reshape(-1, 1))
    _splits(str(d), "time")
    cfg_path = cv.to_t10n_from_downloaded_ds(str(tmp_path / "t10n"), "ogbpa", str(tmp_path / "dl"))
    _check_layout(cfg_path, src, dst, feat, label)
    assert cv.to_t10n_from_downloaded_ds(str(tmp_path / "t10n"), "ogbpa", str(tmp_path / "dl")) == cfg_path


def test_reddit_dgl_files(tmp_path):
    import scipy.sparse as sp

    src, dst, feat, label = _graph(3)
    keep = src != dst
    d = tmp_path / "dl" / "reddit"
    os.makedirs(d)
    types = np.full(N, 3)
    types[:150], types[150:200] = 1, 2
    np.savez(d / "reddit_data.npz", feature=feat, label=label.astype(np.int64), node_types=types)
    sp.save_npz(d / "reddit_graph.npz", sp.coo_matrix((np.ones(keep.sum()), (src[keep], dst[keep])), shape=(N, N)))
    g = cv.load_as_dgl_g(str(tmp_path / "dl"), "reddit")
    assert int(g.ndata["val_mask"].sum()) == 50
    cfg_path = cv.to_t10n_from_dgl_g(str(tmp_path / "t10n"), "reddit", g)
    _check_layout(cfg_path, src[keep], dst[keep], feat, label)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_igb_linked_and_chunked(tmp_path):
    """IGB arrays are linked (row-pair edges, a raw feature file, an .npy label file);
    both chunkers read them and agree."""
    from grappa_b200.dataset.meta import name_to_meta

    meta = name_to_meta("igb260m")
    src, dst, _, label = _graph(4)
    keep = src != dst  # the release has no self-loops
    src, dst = src[keep], dst[keep]
    base = tmp_path / "dl" / meta.origin_path  # where the registry says the release puts its arrays
    os.makedirs(base / "paper")
    os.makedirs(base / "paper__cites__paper")
    np.save(base / "paper__cites__paper" / "edge_index.npy", np.stack([src, dst], 1))
    feat_w = np.random.default_rng(5).standard_normal((N, meta.n_dim)).astype(np.float32)
    feat_w.tofile(base / "paper" / "node_feat.npy")  # raw, no header: the width comes from the file size
    np.save(base / "paper" / "node_label_19.npy", label)
    cfg_path = cv.to_t10n_from_downloaded_ds(str(tmp_path / "t10n"), "igb260m", str(tmp_path / "dl"))
    cfg = json.load(open(cfg_path))
    assert cfg["num_edges"] == len(src) and cfg["feat_dim"] == meta.n_dim and not cfg["add_reverse_edge"]
    assert os.path.islink(cfg["edge_file_bin"]) and os.path.islink(cfg["node_feats_file_bin"])
    io = DatasetIO(os.path.dirname(cfg_path), "")
    u, v = (t.numpy() for t in io.read_edge(0, io.num_edges()))
    assert np.array_equal(u, src) and np.array_equal(v, dst)
    assert np.array_equal(io.read("node_feats_file_bin", 0, N).numpy(), feat_w)
    # both chunkers on the linked layout
    t10n_dir = os.path.dirname(cfg_path)
    assert partition.main(["seq", "--src_path", t10n_dir, "--dest_path", str(tmp_path / "seq"), "--graph_name",
                           "igb260m", "--n_part", "2"]) == 0
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(_free_port()), "-m", "grappa_b200.dataset.partition", "dist",
           "--src_path", t10n_dir, "--dest_path", str(tmp_path / "dist"), "--graph_name", "igb260m",
           "--pg_timeout", "120"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    for i in range(2):
        for ext, dt in (("oid", np.int64), ("ideg", np.int64), ("nfeat", np.float32), ("label", np.float32)):
            a = np.fromfile(pfile(str(tmp_path / "seq" / "chunking_igb260m_hash_002"), i, ext), dtype=dt)
            b = np.fromfile(pfile(str(tmp_path / "dist" / "chunking_igb260m_hash_002"), i, ext), dtype=dt)
            assert np.array_equal(a, b), ext


def test_unsupported_names():
    with pytest.raises(ValueError):
        cv.to_t10n_from_downloaded_ds("/nonexistent", "ogbpr", "/nonexistent")
    with pytest.raises(NotImplementedError):
        cv.load_as_dgl_g("/nonexistent", "cora")
