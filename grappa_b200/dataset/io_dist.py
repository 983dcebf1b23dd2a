"""Dataset IO of the chunkers and the loaders (reference: t10n/dataset/io_dist.py:10-283).

``DatasetIO`` reads row ranges and edge ranges of a graph in the pre-partition layout
(``t10n.json`` naming one ``.bin.npy`` or raw ``mmap.npy`` array per key) and writes the
per-partition files; ``ChunkIO`` reads a partitioned dataset back.  ``per_rank_*`` split
a count over ranks (ceil-sized strides, the last rank takes the rest) and
``SplitConfig`` carries one distributed chunking run's node maps.

The on-disk layout of a partitioned dataset, directory
``{data_path}/chunking_{graph}_{method}_{NNN}/``:

  p{i}.u.bin / p{i}.v.bin      int64  intra-partition edges (local ids) + one self-loop per node
  p{i}.oid.bin                 int64  original id of each local node
  p{i}.ideg.bin                int64  global in-degree
  p{i}.nfeat.bin               float32 [n_i, dim]
  p{i}.label.bin               float32
  p{i}.train/.valid/.test.bin  int8
  b{i}_{j}.u.bin / .v.bin      int64  bridge edges i -> j (absent when empty)
"""
import json
import os

import numpy as np
import torch

DTYPES = {"u": np.int64, "v": np.int64, "oid": np.int64, "ideg": np.int64, "nfeat": np.float32,
          "label": np.float32, "train": np.int8, "valid": np.int8, "test": np.int8}


def pfile(path, i, ext):
    return os.path.join(path, f"p{i}.{ext}.bin")


def bfile(path, i, j, ext):
    return os.path.join(path, f"b{i}_{j}.{ext}.bin")


def read_part(path, i, ext, dim=None, mmap=False):
    f = pfile(path, i, ext)
    if not os.path.isfile(f):
        return None
    a = np.memmap(f, dtype=DTYPES[ext], mode="r") if mmap else np.fromfile(f, dtype=DTYPES[ext])
    if ext == "nfeat" and dim:
        a = a.reshape(-1, dim)
    return a


def read_bridge(path, i, j):
    fu, fv = bfile(path, i, j, "u"), bfile(path, i, j, "v")
    if not os.path.isfile(fu):
        return None, None
    return np.fromfile(fu, dtype=np.int64), np.fromfile(fv, dtype=np.int64)


def part_num_nodes(path, n_part):
    """Nodes per partition, from the size of p{i}.train.bin (t10n/dataloader.py:242-247)."""
    return [os.path.getsize(pfile(path, i, "train")) for i in range(n_part)]


def prefix_sum(counts):
    out = [0]
    for c in counts:
        out.append(out[-1] + c)
    return out


class ChunkIO:
    """Reader of one partitioned dataset directory."""

    def __init__(self, path, n_part, dim):
        self.path, self.n_part, self.dim = path, n_part, dim
        self.counts = part_num_nodes(path, n_part)
        self.prefix = prefix_sum(self.counts)

    def part(self, i, ext, mmap=False):
        return read_part(self.path, i, ext, self.dim, mmap)

    def bridge(self, i, j):
        return read_bridge(self.path, i, j)


def per_rank_stride(world_size, rank, total_num):
    """Rows per rank when total_num rows are split in ceil-sized strides."""
    return -(-total_num // world_size)


def per_rank_local_num(world_size, rank, total_num):
    """Rows of ``rank`` under that split (the last rank holds the remainder)."""
    stride = per_rank_stride(world_size, rank, total_num)
    return max(0, min(stride, total_num - rank * stride))


def per_rank_padding(world_size, rank, total_num):
    """total_num rounded up to a multiple of world_size."""
    return per_rank_stride(world_size, rank, total_num) * world_size


class SplitConfig:
    """One distributed chunking run: this rank among world_size, the node maps
    (nid2pid int32, nid2lid int64), partition count (a multiple of world_size; rank r
    writes partitions [r k, (r + 1) k), k = num_part / world_size) and their sizes."""

    def __init__(self, world_size, rank, nid2pid, nid2lid, num_part, ds_meta, nodes_per_part):
        if len(nodes_per_part) != num_part:
            raise ValueError("nodes_per_part needs one count per partition")
        if num_part % world_size:
            raise ValueError("num_part must be a multiple of the world size")
        self.world_size, self.rank = world_size, rank
        self.nid2pid, self.nid2lid = nid2pid, nid2lid
        self.num_part, self.ds_meta = num_part, ds_meta
        self.nodes_per_part = list(nodes_per_part)

    @property
    def parts_per_rank(self):
        return self.num_part // self.world_size

    def owner(self, pid):
        return pid // self.parts_per_rank

    def my_parts(self):
        k = self.parts_per_rank
        return range(self.rank * k, (self.rank + 1) * k)


# key of t10n.json -> (numpy dtype, per-partition file extension; None for edges)
_KEYS = {
    "node_label_file": (np.float32, "label"),
    "node_feats_file_bin": (np.float32, "nfeat"),
    "train_mask_file_bin": (np.int8, "train"),
    "val_mask_file_bin": (np.int8, "valid"),
    "test_mask_file_bin": (np.int8, "test"),
    "edge_file_bin": (np.int64, None),
    "ideg": (np.int64, "ideg"),
}


class DatasetIO:
    """Reader of a pre-partition dataset (``src_path/t10n.json``) and writer of the
    per-partition files under ``dest_path``.

    Node arrays are ``.npy`` files (np.load, memory-mapped) or raw ``mmap.npy`` arrays
    (no header) of the key's dtype and the shape t10n.json implies.  The edge file is either
    flat, all sources then all destinations (``edge_layout = "flat"``, the t10n layout),
    or one (u, v) row per edge (``"pairs"``, the IGB release's layout); ``"auto"`` tells
    them apart by the array's shape."""

    edge_layout = "auto"
    allowed_keys = list(_KEYS)

    def __init__(self, src_path, dest_path, ds_cfg=None):
        if ds_cfg is None:
            with open(os.path.join(src_path, "t10n.json")) as f:
                ds_cfg = json.load(f)
        self.ds_cfg = ds_cfg
        self.src_path, self.dest_path = src_path, dest_path

    # tables
    def get_npy_dtype(self, key):
        self._check_key(key)
        return _KEYS[key][0]

    def get_th_dtype(self, key):
        return torch.from_numpy(np.zeros(0, dtype=self.get_npy_dtype(key))).dtype

    def get_npy_shape(self, key):
        self._check_key(key)
        if key == "edge_file_bin":
            raise ValueError("edges are read with read_edge")
        n = int(self.ds_cfg["num_nodes"])
        return (n, int(self.ds_cfg["feat_dim"])) if key == "node_feats_file_bin" else (n,)

    def get_node_data_fname(self, key, pidx):
        self._check_key(key)
        if _KEYS[key][1] is None:
            raise ValueError("edges are written with write_primary / write_bridge")
        return f"p{pidx}.{_KEYS[key][1]}.bin"

    def check_npy_dtype(self, key, arr):
        if arr.dtype != self.get_npy_dtype(key):
            raise TypeError(f"{key}: dtype {arr.dtype}, expected {np.dtype(self.get_npy_dtype(key))}")

    def _check_key(self, key):
        if key not in _KEYS:
            raise KeyError(f"unknown dataset key {key}")

    def _array(self, key):
        path = self.ds_cfg[key]
        if not os.path.isabs(path) and not os.path.exists(path):
            path = os.path.join(self.src_path, path)
        with open(path, "rb") as f:
            has_header = f.read(6) == b"\x93NUMPY"
        if path.endswith("mmap.npy") and not has_header:
            shape = None if key == "edge_file_bin" else self.get_npy_shape(key)
            a = np.memmap(path, dtype=self.get_npy_dtype(key), mode="r", shape=shape)
        else:
            a = np.load(path, mmap_mode="r")
        return a

    # reads
    def read(self, key, oid_start, oid_end):
        """Rows [oid_start, oid_end) of a node array, as a tensor of the key's dtype."""
        a = self._array(key)
        if tuple(a.shape) != self.get_npy_shape(key):
            raise ValueError(f"{key}: shape {a.shape}, t10n.json implies {self.get_npy_shape(key)}")
        self.check_npy_dtype(key, a)
        return torch.from_numpy(np.array(a[oid_start:oid_end]))  # a copy: the source is read-only

    def read_rows(self, key, oids):
        """Rows ``oids`` (ascending for a sequential read) of a node array."""
        a = self._array(key)
        self.check_npy_dtype(key, a)
        return torch.from_numpy(np.ascontiguousarray(a[np.asarray(oids)]))

    def zero(self, key, num_node):
        shape = self.get_npy_shape(key)
        return torch.zeros((num_node,) + tuple(shape[1:]), dtype=self.get_th_dtype(key))

    def num_edges(self):
        return int(self.ds_cfg["num_edges"])

    def read_edge(self, off_start, off_end):
        """Edges [off_start, off_end) as int64 (u, v) tensors."""
        a = self._array("edge_file_bin")
        m = self.num_edges()
        layout = self.edge_layout
        if layout == "auto":
            layout = "pairs" if a.ndim == 2 and a.shape[1] == 2 else "flat"
        if layout == "pairs":
            if a.shape[0] != m:
                raise ValueError(f"edge file holds {a.shape[0]} rows, t10n.json says {m}")
            part = np.asarray(a[off_start:off_end])
            u, v = part[:, 0], part[:, 1]
        else:
            if a.reshape(-1).shape[0] != 2 * m:
                raise ValueError(f"edge file holds {a.size} ids, t10n.json says 2 x {m}")
            flat = a.reshape(-1)
            u, v = flat[off_start:off_end], flat[m + off_start:m + off_end]
        return torch.from_numpy(np.array(u, dtype=np.int64)), torch.from_numpy(np.array(v, dtype=np.int64))

    # writes
    def write(self, key, pidx, data_tensor):
        arr = data_tensor.numpy() if torch.is_tensor(data_tensor) else np.asarray(data_tensor)
        self.check_npy_dtype(key, arr)
        np.ascontiguousarray(arr).tofile(os.path.join(self.dest_path, self.get_node_data_fname(key, pidx)))

    def write_primary(self, pidx, p_u, p_v):
        for ext, t in (("u", p_u), ("v", p_v)):
            np.ascontiguousarray(np.asarray(t, dtype=np.int64)).tofile(pfile(self.dest_path, pidx, ext))

    def write_bridge(self, pidx, b_u, pjdx, b_v):
        for ext, t in (("u", b_u), ("v", b_v)):
            np.ascontiguousarray(np.asarray(t, dtype=np.int64)).tofile(bfile(self.dest_path, pidx, pjdx, ext))

    def write_oid(self, pidx, oids):
        np.ascontiguousarray(np.asarray(oids, dtype=np.int64)).tofile(pfile(self.dest_path, pidx, "oid"))


class OgbprIO(DatasetIO):
    """Flat edge file (all sources, then all destinations)."""
    edge_layout = "flat"


class Igb260mIO(DatasetIO):
    """One (u, v) row per edge, as the IGB release ships it."""
    edge_layout = "pairs"


def get_dataset_io(src_path, dest_path, graph_name):
    """The DatasetIO of a graph: IGB's row-pair edges for igb*, else auto-detected."""
    if graph_name.startswith("igb"):
        return Igb260mIO(src_path, dest_path)
    if graph_name in ("ogbpr", "ogbpa"):
        return OgbprIO(src_path, dest_path)
    return DatasetIO(src_path, dest_path)
