"""The offline dataset pipeline from its command line: generate a seeded graph in the
pre-partition layout, chunk it in one process (hash and metis) and with gloo ranks, and
check the chunk sets against each other and against the source graph."""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from grappa_b200.dataset import partition
from grappa_b200.dataset.io_dist import bfile, pfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def src(tmp_path_factory):
    d = tmp_path_factory.mktemp("ds")
    out = str(d / "t10n" / "tiny")
    assert partition.main(["generate", "--graph_name", "tiny", "--out", out]) == 0
    return d, out


def _edges(path, k):
    """Global (u, v) pairs of a chunk set (self-loops dropped), sorted."""
    oid = [np.fromfile(pfile(path, i, "oid"), dtype=np.int64) for i in range(k)]
    us, vs = [], []
    for i in range(k):
        u = np.fromfile(pfile(path, i, "u"), dtype=np.int64)
        v = np.fromfile(pfile(path, i, "v"), dtype=np.int64)
        us.append(oid[i][u])
        vs.append(oid[i][v])
        for j in range(k):
            if j != i and os.path.exists(bfile(path, i, j, "u")):
                us.append(oid[i][np.fromfile(bfile(path, i, j, "u"), dtype=np.int64)])
                vs.append(oid[j][np.fromfile(bfile(path, i, j, "v"), dtype=np.int64)])
    u, v = np.concatenate(us), np.concatenate(vs)
    keep = u != v
    pairs = np.stack([u[keep], v[keep]], 1)
    return pairs[np.lexsort((pairs[:, 1], pairs[:, 0]))]


def _source_edges(src_dir):
    cfg = json.load(open(os.path.join(src_dir, "t10n.json")))
    e = np.load(cfg["edge_file_bin"])
    m = cfg["num_edges"]
    u, v = e[:m], e[m:]
    keep = u != v
    pairs = np.unique(np.stack([u[keep], v[keep]], 1), axis=0)
    return cfg, pairs


@pytest.mark.parametrize("method", ["hash", "metis"])
def test_seq_chunks_hold_the_graph(src, method, capsys):
    d, s = src
    assert partition.main(["seq", "--src_path", s, "--dest_path", str(d), "--graph_name", "tiny",
                           "--part_method", method, "--n_part", "4"]) == 0
    path = str(d / f"chunking_tiny_{method}_004")
    summary, rows = partition.chunk_info(path)
    cfg, pairs = _source_edges(s)
    assert summary["n_part"] == 4 and summary["nodes"] == cfg["num_nodes"]
    assert summary["edges"] == len(pairs)
    assert sum(r["train"] for r in rows) == cfg["num_train_nodes"]
    for r in rows:  # the halo: distinct sources of the edges that enter the partition from others
        i = r["part"]
        oid = [np.fromfile(pfile(path, j, "oid"), dtype=np.int64) for j in range(4)]
        mine = set(oid[i].tolist())
        want = {int(a) for a, b in pairs if int(b) in mine and int(a) not in mine}
        assert r["halo_in"] == len(want)
    assert np.array_equal(_edges(path, 4), pairs)
    oid = np.concatenate([np.fromfile(pfile(path, i, "oid"), dtype=np.int64) for i in range(4)])
    assert np.array_equal(np.sort(oid), np.arange(cfg["num_nodes"]))
    if method == "metis":  # balanced by nodes and by training nodes, fewer cut edges than hashing
        assert summary["node_imbalance"] <= 1.04 and summary["train_imbalance"] <= 1.04
        hashed = partition.chunk_info(str(d / "chunking_tiny_hash_004"))[0] if os.path.isdir(
            str(d / "chunking_tiny_hash_004")) else None
        if hashed:
            assert summary["cut_fraction"] < hashed["cut_fraction"]
    assert partition.main(["info", "--path", path, "--json"]) == 0
    info = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert info["summary"]["n_part"] == 4 and len(info["parts"]) == 4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("n_part", [2, 4])
def test_dist_chunks_match_seq_hash(src, n_part):
    """Two gloo ranks (one or two partitions each) write the same hash partition as the
    one-process chunker: the same nodes, in-degrees, features, labels and masks per
    partition and the same edges."""
    d, s = src
    dest = str(d / f"dist{n_part}")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), "-m", "grappa_b200.dataset.partition",
           "dist", "--src_path", s, "--dest_path", dest, "--graph_name", "tiny", "--n_part", str(n_part),
           "--pg_timeout", "120"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    seq_dest = str(d / f"seq{n_part}")
    assert partition.main(["seq", "--src_path", s, "--dest_path", seq_dest, "--graph_name", "tiny",
                           "--part_method", "hash", "--n_part", str(n_part)]) == 0
    name = f"chunking_tiny_hash_{n_part:03}"
    pd, ps = os.path.join(dest, name), os.path.join(seq_dest, name)
    for i in range(n_part):
        oid_d = np.fromfile(pfile(pd, i, "oid"), dtype=np.int64)
        oid_s = np.fromfile(pfile(ps, i, "oid"), dtype=np.int64)
        assert np.array_equal(oid_d, oid_s)
        for ext, dt in (("ideg", np.int64), ("label", np.float32), ("train", np.int8), ("valid", np.int8),
                        ("test", np.int8), ("nfeat", np.float32), ("u", np.int64), ("v", np.int64)):
            a = np.fromfile(pfile(pd, i, ext), dtype=dt)
            b = np.fromfile(pfile(ps, i, ext), dtype=dt)
            if ext in ("u", "v"):
                assert a.shape == b.shape
            else:
                assert np.array_equal(a, b), ext
    assert np.array_equal(_edges(pd, n_part), _edges(ps, n_part))
    _, pairs = _source_edges(s)
    assert np.array_equal(_edges(pd, n_part), pairs)


def test_info_rejects_a_directory_without_chunks(tmp_path):
    with pytest.raises(FileNotFoundError):
        partition.chunk_info(str(tmp_path))


def test_sweep_builds_missing_chunk_sets_first(tmp_path, capsys):
    """launch --partition plans generation (once per graph), chunking of each missing
    (method, graph) set, then training; sets already on disk are skipped."""
    from grappa_b200 import launch

    data = tmp_path / "data"
    argv = ["--partition", "--dry_run", "--data_path", str(data), "--graphs", "tiny,rmat16k", "--parts",
            "hash,metis", "--nproc", "2", "--num_gpus", "-1", "--log_dir", str(tmp_path / "log")]
    assert launch.main(argv) == 0
    lines = capsys.readouterr().out.strip().splitlines()
    gens = [l for l in lines if "dataset.partition generate" in l]
    chunks = [l for l in lines if "dataset.partition seq" in l]
    trains = [l for l in lines if "grappa_b200.train.t10n_train" in l]
    assert len(gens) == 2 and len(chunks) == 4 and len(trains) == 4
    assert lines.index(chunks[-1]) < lines.index(trains[0])
    assert any("--part_method metis --n_part 2" in l and "--graph_name tiny" in l for l in chunks)
    (data / "chunking_tiny_hash_002").mkdir(parents=True)
    (data / "t10n" / "tiny").mkdir(parents=True)
    (data / "t10n" / "tiny" / "t10n.json").write_text("{}")
    assert launch.main(argv) == 0
    lines = capsys.readouterr().out.strip().splitlines()
    assert sum("dataset.partition generate" in l for l in lines) == 1  # rmat16k only
    chunks = [l for l in lines if "dataset.partition seq" in l]
    assert len(chunks) == 3 and not any("--part_method hash" in l and "--graph_name tiny" in l for l in chunks)


def test_dataset_io_layouts_and_strides(tmp_path):
    """DatasetIO reads flat and row-pair edge files and raw mmap.npy node arrays; the
    per-rank split covers every row exactly once."""
    from grappa_b200.dataset import io_dist

    n, m = 10, 7
    u = np.arange(m, dtype=np.int64)
    v = (np.arange(m, dtype=np.int64) * 3) % n
    np.save(tmp_path / "flat.bin.npy", np.concatenate([u, v]))
    np.save(tmp_path / "pairs.bin.npy", np.stack([u, v], 1))
    feat = np.arange(n * 4, dtype=np.float32).reshape(n, 4)
    feat.tofile(tmp_path / "feat_mmap.npy")
    cfg = {"num_nodes": n, "num_edges": m, "feat_dim": 4, "edge_file_bin": str(tmp_path / "flat.bin.npy"),
           "node_feats_file_bin": str(tmp_path / "feat_mmap.npy")}
    (tmp_path / "t10n.json").write_text(json.dumps(cfg))
    for cls, edge_file in ((io_dist.OgbprIO, "flat"), (io_dist.DatasetIO, "flat"), (io_dist.Igb260mIO, "pairs"),
                           (io_dist.DatasetIO, "pairs")):
        cfg["edge_file_bin"] = str(tmp_path / f"{edge_file}.bin.npy")
        (tmp_path / "t10n.json").write_text(json.dumps(cfg))
        io = cls(str(tmp_path), str(tmp_path))
        eu, ev = io.read_edge(2, 5)
        assert eu.tolist() == u[2:5].tolist() and ev.tolist() == v[2:5].tolist()
    rows = io.read("node_feats_file_bin", 3, 6)
    assert np.array_equal(rows.numpy(), feat[3:6])
    assert np.array_equal(io.read_rows("node_feats_file_bin", [1, 7]).numpy(), feat[[1, 7]])
    assert io.zero("node_feats_file_bin", 5).shape == (5, 4)
    io.write("node_feats_file_bin", 2, rows)
    assert np.array_equal(np.fromfile(tmp_path / "p2.nfeat.bin", dtype=np.float32).reshape(-1, 4), feat[3:6])
    with pytest.raises(TypeError):
        io.write("train_mask_file_bin", 0, rows)  # float rows for an int8 key
    assert isinstance(io_dist.get_dataset_io(str(tmp_path), str(tmp_path), "igb260m"), io_dist.Igb260mIO)
    for total in (0, 1, 9, 10, 11, 1000003):
        for world in (1, 3, 4, 8):
            counts = [io_dist.per_rank_local_num(world, r, total) for r in range(world)]
            stride = io_dist.per_rank_stride(world, 0, total)
            assert sum(counts) == total and all(c <= stride for c in counts)
            assert io_dist.per_rank_padding(world, 0, total) % world == 0
            assert io_dist.per_rank_padding(world, 0, total) >= total
