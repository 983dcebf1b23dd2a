"""Sequential (single-process) chunk builder (reference: t10n/dataset/chunk_seq.py:27-150).

Reads a dataset in the pre-partition layout (``t10n.json`` + ``*.bin.npy``, see
grappa_b200.dataset.synthetic.to_t10n_layout), assigns nodes to partitions and
writes the partition chunks with the C++ writer (grappa_b200._C.c_seq).

Partition methods: ``hash`` / ``random`` (seeded hash of the node id), ``metis``
(multilevel k-way edge-cut partition balanced by node count and by training nodes,
grappa_b200/csrc/host/mlpart.cc: the role of the reference's
dgl.metis_partition_assignment with the train mask as a balance type,
t10n/dataset/chunk_seq.py:47-50) and ``lp`` (label-propagation refinement of the
hash assignment under a size cap).
"""
import os
import pathlib

import numpy as np
import torch

from grappa_b200 import _native
from grappa_b200.dataset.meta import t10n_chunk_path


def assign_partitions(u, v, n, n_part, method="hash", seed=0, rounds=4, train_mask=None):
    if n_part == 1:
        return np.zeros(n, dtype=np.int64)
    if method == "metis":
        tr = None if train_mask is None else np.ascontiguousarray(train_mask, dtype=np.int8)
        return _native.host().c_seq.multilevel_partition(n, np.ascontiguousarray(u, dtype=np.int64),
                                                        np.ascontiguousarray(v, dtype=np.int64), n_part, tr,
                                                        seed, 0.03)
    pid = _native.host().c_dist.random_assign_pid(n, n_part, seed)
    if method in ("hash", "random"):
        return pid
    if method != "lp":
        raise ValueError(f"unknown partition method {method}")
    return label_propagation(u, v, n, n_part, pid, rounds)


def label_propagation(u, v, n, n_part, pid, rounds=4, slack=1.05):
    """Move nodes to the partition most of their neighbours are in, subject to a size cap."""
    pid = torch.from_numpy(pid.copy())
    uu, vv = torch.from_numpy(u), torch.from_numpy(v)
    cap = int(slack * n / n_part) + 1
    for _ in range(rounds):
        votes = torch.zeros((n, n_part), dtype=torch.int32)
        votes.index_put_((vv, pid[uu]), torch.ones(vv.numel(), dtype=torch.int32), accumulate=True)
        best = votes.argmax(1)
        gain = votes.gather(1, best.unsqueeze(1)).squeeze(1) - votes.gather(1, pid.unsqueeze(1)).squeeze(1)
        order = torch.argsort(gain, descending=True)
        sizes = torch.bincount(pid, minlength=n_part)
        moved = 0
        for node in order[gain[order] > 0].tolist():
            a, b = int(pid[node]), int(best[node])
            if sizes[b] < cap:
                sizes[a] -= 1
                sizes[b] += 1
                pid[node] = b
                moved += 1
        if moved == 0:
            break
    return pid.numpy()


def get_u_v_nid2pid(cfg_json, part_method, n_parts, seed=0):
    """(u, v, nid2pid) of a pre-partition dataset given its t10n.json dict (reference:
    t10n/dataset/chunk_seq.py:27-82): its edges and the partition of every node
    (int64) by ``part_method`` (metis balances the training mask)."""
    from grappa_b200.dataset.io_dist import DatasetIO

    io = DatasetIO(os.path.dirname(cfg_json["edge_file_bin"]), None, ds_cfg=cfg_json)
    n = int(cfg_json["num_nodes"])
    u, v = (t.numpy() for t in io.read_edge(0, io.num_edges()))
    train = io.read("train_mask_file_bin", 0, n).numpy() if part_method == "metis" else None
    return u, v, np.asarray(assign_partitions(u, v, n, n_parts, part_method, seed, train_mask=train), dtype=np.int64)


def build_chunks_seq(dest_path, dataset_name, src_path, part_method, n_part, seed=0):
    """Chunk ``src_path`` (a t10n.json directory) into
    ``dest_path/chunking_{dataset}_{part_method}_{n_part:03}`` in this process (reference:
    t10n/dataset/chunk_seq.py:110-150).  Inputs are read through the dataset IO (flat or
    row-pair edge files, .npy or raw memory-mapped node arrays).  Returns the output
    directory and the writer's statistics."""
    from grappa_b200.dataset.io_dist import get_dataset_io

    out = os.path.join(dest_path, t10n_chunk_path(dataset_name, part_method, n_part))
    if os.path.exists(out):
        raise FileExistsError(f"please delete {out} first")
    io = get_dataset_io(src_path, out, dataset_name)
    cfg = io.ds_cfg
    n, dim = int(cfg["num_nodes"]), int(cfg["feat_dim"])
    pathlib.Path(out).mkdir(parents=True)
    u, v = (t.numpy() for t in io.read_edge(0, io.num_edges()))
    m = int(u.shape[0])

    def node(key):
        return io.read(key, 0, n).numpy()

    train = node("train_mask_file_bin")
    pid = assign_partitions(u, v, n, n_part, part_method, seed, train_mask=train if part_method == "metis" else None)
    c = _native.host().c_seq
    stats = c.build(out, n, m, dim, n_part, u, v, pid)
    c.split_node_feat(out, n, dim, n_part, node("node_feats_file_bin"))
    c.split_node_data(out, n, n_part, node("node_label_file"), train, node("val_mask_file_bin"),
                      node("test_mask_file_bin"))
    return out, stats


def build_chunks_from_graph(graph, dest_path, n_part, part_method="hash", seed=0):
    """Write the chunk layout of an in-memory SyntheticGraph (no intermediate files)."""
    name = graph.spec.name
    out = os.path.join(dest_path, t10n_chunk_path(name, part_method, n_part))
    pathlib.Path(out).mkdir(parents=True, exist_ok=True)
    n = graph.n_nodes
    u = graph.u.cpu().numpy().astype(np.int64)
    v = graph.v.cpu().numpy().astype(np.int64)
    pid = assign_partitions(u, v, n, n_part, part_method, seed, train_mask=graph.train_mask.cpu().numpy())
    c = _native.host().c_seq
    stats = c.build(out, n, len(u), graph.spec.feat_dim, n_part, u, v, pid)
    c.split_node_feat(out, n, graph.spec.feat_dim, n_part, graph.feat.cpu().numpy().astype(np.float32))
    c.split_node_data(out, n, n_part, graph.label.cpu().numpy().astype(np.float32),
                      graph.train_mask.cpu().numpy(), graph.val_mask.cpu().numpy(), graph.test_mask.cpu().numpy())
    return out, stats
