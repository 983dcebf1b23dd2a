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


def test_dist_chunks_match_seq_hash(src):
    """Two gloo ranks write the same hash partition as the one-process chunker: the same
    nodes, in-degrees, features, labels and masks per partition and the same edges."""
    d, s = src
    dest = str(d / "dist")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), "-m", "grappa_b200.dataset.partition",
           "dist", "--src_path", s, "--dest_path", dest, "--graph_name", "tiny", "--pg_timeout", "120"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert partition.main(["seq", "--src_path", s, "--dest_path", str(d / "seq2"), "--graph_name", "tiny",
                           "--part_method", "hash", "--n_part", "2"]) == 0
    pd, ps = os.path.join(dest, "chunking_tiny_hash_002"), str(d / "seq2" / "chunking_tiny_hash_002")
    for i in range(2):
        oid_d = np.fromfile(pfile(pd, i, "oid"), dtype=np.int64)
        oid_s = np.fromfile(pfile(ps, i, "oid"), dtype=np.int64)
        assert np.array_equal(oid_d, oid_s)
        for ext, dt in (("ideg", np.int64), ("label", np.float32), ("train", np.int8), ("valid", np.int8),
                        ("test", np.int8), ("nfeat", np.float32)):
            assert np.array_equal(np.fromfile(pfile(pd, i, ext), dtype=dt), np.fromfile(pfile(ps, i, ext), dtype=dt))
    assert np.array_equal(_edges(pd, 2), _edges(ps, 2))
    _, pairs = _source_edges(s)
    assert np.array_equal(_edges(pd, 2), pairs)


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
