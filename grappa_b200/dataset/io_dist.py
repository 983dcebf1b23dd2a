"""Chunk file names, dtypes and readers (reference: t10n/dataset/io_dist.py:10-283).

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
import os

import numpy as np

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


def get_dataset_io(path, n_part, dim):
    return ChunkIO(path, n_part, dim)
