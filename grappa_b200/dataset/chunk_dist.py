"""Distributed chunk builder (reference: t10n/dataset/chunk_dist.py:19-318).

One gloo process group chunks a graph in the pre-partition layout into ``num_part``
partitions, a multiple of its size: rank r writes partitions [r k, (r + 1) k) with
k = num_part / world_size.  The steps keep the reference's names:

  random_assign_pid_for_nid   partition of every node: a seeded hash of its id, the
                              same assignment as the one-process chunker's ``hash``
                              method, computed by every rank locally (the reference
                              draws random ids per slice and all-gathers them)
  relabel_nid                 local id = rank of the node among its partition's nodes
                              in original-id order; nodes per partition
  split_edges                 every rank reads one stride of the edge file and sends
                              each partition's intra edges and each (i, j) bridge list
                              to the rank that writes partition i (local ids)
  split_ideg                  global in-degrees: per-stride counts summed by an
                              all-reduce, each owner writes its partitions' slice
  split_node_data             node arrays (labels, masks, features): each owner reads
                              its partitions' rows straight from the source arrays
                              (all ranks see the same files), in ascending id order
                              (the reference reads strides and gathers them)

The self-loop of every node is appended to its partition's intra edges, as the
one-process chunker writes them; p{i}.oid.bin records the original ids.  Output
layout: grappa_b200.dataset.io_dist.
"""
import os
import pathlib

import numpy as np
import torch
import torch.distributed as dist

from grappa_b200 import _native
from grappa_b200.cl import t10n_gather_gloo
from grappa_b200.dataset.io_dist import (DatasetIO, SplitConfig, get_dataset_io, per_rank_local_num,
                                         per_rank_stride)
from grappa_b200.dataset.meta import name_to_meta, t10n_chunk_path


def random_assign_pid_for_nid(world_size, rank, nid2pid, num_part, seed=0):
    """Fill int32 ``nid2pid`` (one entry per node, any padding beyond n is left alone)
    with each node's partition."""
    if nid2pid.dtype != torch.int32:
        raise TypeError("nid2pid must be int32")
    n = nid2pid.shape[0]
    pid = _native.host().c_dist.random_assign_pid(n, num_part, seed)
    nid2pid.copy_(torch.from_numpy(pid.astype(np.int32)))
    return nid2pid


def relabel_nid(world_size, rank, nid2lid, nid2pid, num_part):
    """Fill ``nid2lid`` with each node's rank within its partition (original-id order);
    returns the node count of every partition."""
    pid = nid2pid.to(torch.int64)
    counts = torch.bincount(pid, minlength=num_part)
    order = torch.argsort(pid * nid2pid.shape[0] + torch.arange(nid2pid.shape[0]), stable=True)
    starts = torch.cumsum(counts, 0) - counts
    nid2lid[order] = torch.arange(nid2pid.shape[0]) - torch.repeat_interleave(starts, counts)
    return counts.tolist()


def _my_edges(sc, ds_io):
    m = ds_io.num_edges()
    stride = per_rank_stride(sc.world_size, sc.rank, m)
    lo = sc.rank * stride
    return ds_io.read_edge(lo, lo + per_rank_local_num(sc.world_size, sc.rank, m))


def split_edges(sc: SplitConfig, ds_io: DatasetIO):
    """Intra edges p{i}.u/v (with one self-loop per node) and bridges b{i}_{j}.u/v in
    local ids, written by the owner of partition i."""
    u, v = _my_edges(sc, ds_io)
    keep = u != v  # self-loops of the source are replaced by exactly one per node
    u, v = u[keep], v[keep]
    pu, pv = sc.nid2pid[u].to(torch.int64), sc.nid2pid[v].to(torch.int64)
    for i in range(sc.num_part):
        owner = sc.owner(i)
        in_i = pu == i
        # every rank takes part in every gather, in the same order
        lists = [(i, in_i & (pv == i))] + [(j, in_i & (pv == j)) for j in range(sc.num_part) if j != i]
        for j, sel in lists:
            gu = t10n_gather_gloo(sc.nid2lid[u[sel]], sc.rank, sc.world_size, owner)
            gv = t10n_gather_gloo(sc.nid2lid[v[sel]], sc.rank, sc.world_size, owner)
            if sc.rank != owner:
                continue
            if j == i:
                loops = torch.arange(sc.nodes_per_part[i], dtype=torch.int64)
                ds_io.write_primary(i, torch.cat([gu, loops]), torch.cat([gv, loops]))
            elif gu.numel():
                ds_io.write_bridge(i, gu, j, gv)


def split_ideg(sc: SplitConfig, ds_io: DatasetIO):
    """p{i}.ideg.bin: in-degree of every node over the source's edge list (its
    self-loops included, as the one-process chunker counts them), in local-id order."""
    _, v = _my_edges(sc, ds_io)
    ideg = torch.bincount(v, minlength=sc.nid2pid.shape[0]).to(torch.int64)
    dist.all_reduce(ideg)
    for i in sc.my_parts():
        oid = _part_oids(sc, i)
        ds_io.write("ideg", i, ideg[oid].contiguous())


def _part_oids(sc, i):
    return torch.nonzero(sc.nid2pid == i).flatten()  # ascending = local-id order


def split_node_data(sc: SplitConfig, ds_io: DatasetIO, key: str):
    """Per-partition file of node array ``key``, rows in local-id order."""
    for i in sc.my_parts():
        oid = _part_oids(sc, i)
        ds_io.write(key, i, ds_io.read_rows(key, oid.numpy()))


def split_1d(sc: SplitConfig, ds_io: DatasetIO, key: str):
    split_node_data(sc, ds_io, key)


def split_2d(sc: SplitConfig, ds_io: DatasetIO, key: str):
    split_node_data(sc, ds_io, key)


def build_chunks_dist(world_size, rank, dest_path, graph_name, src_path, part_method="hash", num_part=None,
                      seed=0):
    """Chunk ``src_path`` (a t10n.json directory) into
    ``dest_path/chunking_{graph}_{part_method}_{num_part:03}`` with this process group
    (reference signature: t10n/dataset/chunk_dist.py:278-318).  ``part_method`` names
    the directory; the assignment is the seeded hash (``hash`` / ``random``).  Returns
    the output directory."""
    if part_method not in ("hash", "random"):
        raise ValueError(f"the distributed chunker assigns by hash; {part_method} needs the one-process chunker")
    num_part = world_size if num_part is None else int(num_part)
    if num_part % world_size:
        raise ValueError(f"num_part {num_part} is not a multiple of the world size {world_size}")
    out = os.path.join(dest_path, t10n_chunk_path(graph_name, part_method, num_part))
    exists = torch.tensor([int(os.path.exists(out) and rank == 0)])
    dist.all_reduce(exists)
    if int(exists):
        raise FileExistsError(f"please delete {out} first")
    dist.barrier()
    pathlib.Path(out).mkdir(parents=True, exist_ok=True)
    dist.barrier()
    io = get_dataset_io(src_path, out, graph_name)
    n = int(io.ds_cfg["num_nodes"])
    try:
        meta = name_to_meta(graph_name)
    except AssertionError:
        meta = None  # a graph outside the registry: t10n.json carries its sizes
    nid2pid = random_assign_pid_for_nid(world_size, rank, torch.zeros(n, dtype=torch.int32), num_part, seed)
    nid2lid = torch.zeros(n, dtype=torch.int64)
    nodes_per_part = relabel_nid(world_size, rank, nid2lid, nid2pid, num_part)
    sc = SplitConfig(world_size, rank, nid2pid, nid2lid, num_part, meta, nodes_per_part)
    split_edges(sc, io)
    split_ideg(sc, io)
    for i in sc.my_parts():
        io.write_oid(i, _part_oids(sc, i).numpy())
    for key in ("node_label_file", "train_mask_file_bin", "val_mask_file_bin", "test_mask_file_bin"):
        split_1d(sc, io, key)
    split_2d(sc, io, "node_feats_file_bin")
    dist.barrier()
    return out
