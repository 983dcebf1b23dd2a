"""Distributed chunk builder (reference: t10n/dataset/chunk_dist.py:19-318).

Every rank of a (gloo) process group reads one slice of the edge list, splits it
into intra-partition and bridge edges, and sends each list to the rank that owns
the partition; every rank then writes the files of its own partition (one
partition per rank).  The partition assignment is a seeded hash of the node id,
so every rank computes it locally (the reference all-gathers random ids,
t10n/dataset/chunk_dist.py:30-31).  Output layout: grappa_b200.dataset.io_dist.
"""
import json
import os
import pathlib

import numpy as np
import torch
import torch.distributed as dist

from grappa_b200 import _native
from grappa_b200.cl import t10n_gather_gloo
from grappa_b200.dataset.meta import t10n_chunk_path


def _write(path, arr):
    np.ascontiguousarray(arr).tofile(path)


def build_chunks_dist(dest_path, dataset_name, src_path, seed=0):
    rank, world = dist.get_rank(), dist.get_world_size()
    with open(os.path.join(src_path, "t10n.json")) as f:
        cfg = json.load(f)
    n, m = int(cfg["num_nodes"]), int(cfg["num_edges"])
    out = os.path.join(dest_path, t10n_chunk_path(dataset_name, "hash", world))
    pathlib.Path(out).mkdir(parents=True, exist_ok=True)
    pid = _native.host().c_dist.random_assign_pid(n, world, seed)
    counts = np.bincount(pid, minlength=world)
    order = np.argsort(pid * n + np.arange(n), kind="stable")
    lid = np.empty(n, dtype=np.int64)
    for p in range(world):  # local id = rank of the node within its partition (original-id order)
        start = counts[:p].sum()
        lid[order[start:start + counts[p]]] = np.arange(counts[p])
    edges = np.load(cfg["edge_file_bin"], mmap_mode="r")
    lo, hi = rank * m // world, (rank + 1) * m // world
    u = np.asarray(edges[lo:hi], dtype=np.int64)
    v = np.asarray(edges[m + lo:m + hi], dtype=np.int64)
    ideg = torch.from_numpy(np.bincount(v, minlength=n).astype(np.int64))
    dist.all_reduce(ideg)
    keep = u != v
    u, v = u[keep], v[keep]
    pu, pv = pid[u], pid[v]
    for owner in range(world):
        # intra edges of partition `owner`
        sel = (pu == owner) & (pv == owner)
        uu = t10n_gather_gloo(torch.from_numpy(lid[u[sel]]), rank, world, owner)
        vv = t10n_gather_gloo(torch.from_numpy(lid[v[sel]]), rank, world, owner)
        if rank == owner:
            loops = np.arange(counts[owner], dtype=np.int64)
            _write(os.path.join(out, f"p{owner}.u.bin"), np.concatenate([uu.numpy(), loops]))
            _write(os.path.join(out, f"p{owner}.v.bin"), np.concatenate([vv.numpy(), loops]))
        # bridges b{owner}_{q}: u in `owner`, v in q (written by the owner of u)
        for q in range(world):
            if q == owner:
                continue
            sel = (pu == owner) & (pv == q)
            bu = t10n_gather_gloo(torch.from_numpy(lid[u[sel]]), rank, world, owner)
            bv = t10n_gather_gloo(torch.from_numpy(lid[v[sel]]), rank, world, owner)
            if rank == owner and bu.numel():
                _write(os.path.join(out, f"b{owner}_{q}.u.bin"), bu.numpy())
                _write(os.path.join(out, f"b{owner}_{q}.v.bin"), bv.numpy())
    oid = order[counts[:rank].sum():counts[:rank].sum() + counts[rank]]
    _write(os.path.join(out, f"p{rank}.oid.bin"), oid)
    _write(os.path.join(out, f"p{rank}.ideg.bin"), ideg.numpy()[oid])
    feat = np.load(cfg["node_feats_file_bin"], mmap_mode="r")
    _write(os.path.join(out, f"p{rank}.nfeat.bin"), np.asarray(feat[oid], dtype=np.float32))
    lab = np.load(cfg["node_label_file"], mmap_mode="r")
    _write(os.path.join(out, f"p{rank}.label.bin"), np.asarray(lab[oid], dtype=np.float32))
    for name, key in (("train", "train_mask_file_bin"), ("valid", "val_mask_file_bin"), ("test", "test_mask_file_bin")):
        mk = np.load(cfg[key], mmap_mode="r")
        _write(os.path.join(out, f"p{rank}.{name}.bin"), np.asarray(mk[oid], dtype=np.int8))
    dist.barrier()
    return out
