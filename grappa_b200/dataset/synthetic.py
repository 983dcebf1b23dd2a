"""Seeded synthetic graphs of the benchmark shapes.

* RMAT edges with (a, b, c, d) probabilities: candidate edge e draws its quadrant
  bits from Philox(seed, e); candidates with an endpoint >= n and self-loops are
  dropped, each undirected edge is kept once (u < v), and the first
  ``n_edges`` distinct edges in generation order form the graph.  The same
  candidates come out of the CPU (grappa_b200._C) and GPU (grappa_b200._cuda)
  generators, so a graph is identical wherever it is built.
* node ids are then permuted by sorting a hash of (id, seed), spreading the RMAT
  hubs over the id space;
* features are i.i.d. N(0, 1) (Box-Muller over Philox);
* labels are the argmax of a fixed random 2-hop mean-aggregation teacher:
  y = argmax( A_mean relu(A_mean X W1) W2 - b ), A_mean the row-normalised
  adjacency with self-loops and b a per-class bias that centres the scores;
* splits come from a seeded permutation of the nodes (train / val / test
  fractions).

The reference reads real datasets (t10n/dataset/dgl_to_t10n.py); the benchmark
configurations of this project use these seeded graphs with the same shapes.
"""
import math
from dataclasses import dataclass

import numpy as np
import torch

from grappa_b200 import _native

RMAT_ABCD = (0.57, 0.19, 0.19, 0.05)


@dataclass
class SyntheticSpec:
    n_nodes: int
    n_edges: int              # undirected edges (the directed graph has twice as many)
    feat_dim: int
    n_classes: int
    train_frac: float
    val_frac: float
    seed: int = 0
    abcd: tuple = RMAT_ABCD
    teacher_hidden: int = 64
    name: str = "rmat"


# Benchmark graphs (seeded RMAT analogues of the reference's datasets, t10n/dataset/meta.py).
SPECS = {
    # CPU/gloo config: 16,384 nodes, 131,072 undirected edges, 64-dim, 8 classes, 60/20/20
    "rmat16k": SyntheticSpec(16384, 131072, 64, 8, 0.6, 0.2, seed=1, name="rmat16k"),
    # ogbn-products shape: 2,449,029 nodes, 61,859,140 undirected edges, 100-dim, 47 classes, 8/1.6/90.4
    "ogbpr": SyntheticSpec(2449029, 61859140, 100, 47, 0.08, 0.016, seed=2, name="ogbpr"),
    # reddit shape (dense degree): 232,965 nodes, 114.6M directed edges, 602-dim, 41 classes, 66/10/24
    "reddit": SyntheticSpec(232965, 57307946, 602, 41, 0.66, 0.10, seed=3, name="reddit"),
    # ogbn-papers100M shape: 111,059,956 nodes, 1.6B directed edges, 128-dim, 172 classes, 1.1% train
    "ogbpa": SyntheticSpec(111059956, 807842936, 128, 172, 0.011, 0.001, seed=4, name="ogbpa"),
    # reduced ogbn-products shape for per-kernel profiler captures: 1,000,000 nodes,
    # 25M undirected edges (50M directed), 100-dim, 47 classes; about 0.6 GB resident,
    # still larger than L2 so that DRAM counters keep their meaning
    "ogbpr_small": SyntheticSpec(1000000, 25000000, 100, 47, 0.08, 0.016, seed=6, name="ogbpr_small"),
    # small graphs for tests
    "tiny": SyntheticSpec(4096, 40000, 32, 8, 0.5, 0.2, seed=5, name="tiny"),
}


def _rmat_keys(spec, count, device):
    n = spec.n_nodes
    scale = max(1, math.ceil(math.log2(n)))
    a, b, c, _ = spec.abcd
    if device.type == "cuda":
        keys = torch.empty(count, dtype=torch.int64, device=device)
        _native.cuda().rmat_candidates(n, scale, a, b, c, spec.seed, 0, keys)
        return keys
    return torch.from_numpy(_native.host().graph.rmat_candidates(n, scale, a, b, c, spec.seed, 0, count))


def rmat_undirected(spec, device="cpu"):
    """First ``spec.n_edges`` distinct undirected edges (u < v) as an int64 key tensor u*n+v."""
    device = torch.device(device)
    m = spec.n_edges
    count = int(m * 1.5) + 1024
    while True:
        keys = _rmat_keys(spec, count, device)
        idx = torch.nonzero(keys >= 0).squeeze(1)
        k = keys[idx]
        del keys
        ks, order = torch.sort(k, stable=True)
        first = torch.ones_like(ks, dtype=torch.bool)
        first[1:] = ks[1:] != ks[:-1]
        uniq_keys = ks[first]
        uniq_idx = idx[order[first]]
        del ks, order, first, k, idx
        if uniq_keys.numel() >= m:
            sel = torch.argsort(uniq_idx)[:m]
            return uniq_keys[sel]
        count = int(count * 1.4)


def shuffle_keys(ids, seed, epoch):
    """Hash keys of int64 ids; sorting by them gives the same permutation on CPU and GPU."""
    if ids.is_cuda:
        keys = torch.empty_like(ids)
        _native.cuda().shuffle_keys(ids.contiguous(), int(seed), int(epoch), keys)
        return keys
    return torch.from_numpy(_native.host().graph.shuffle_keys(ids.contiguous().numpy(), int(seed), int(epoch)))


def node_permutation(n, seed, device):
    """perm[old_id] = new_id, from a sort of hashed ids (same on CPU and GPU)."""
    ids = torch.arange(n, dtype=torch.int64, device=device)
    order = torch.argsort(shuffle_keys(ids, seed ^ 0x5EED, 0), stable=True)
    perm = torch.empty_like(order)
    perm[order] = torch.arange(n, dtype=torch.int64, device=device)
    return perm


def normal(n, seed, device):
    if torch.device(device).type == "cuda":
        out = torch.empty(n, dtype=torch.float32, device=device)
        _native.cuda().normal_fill(out, int(seed))
        return out
    return torch.from_numpy(_native.host().normal(n, int(seed)))


def csc_from_edges(u, v, n):
    """CSC by destination (indptr int64, indices int32), sources ascending per row."""
    key, _ = torch.sort(v * n + u)
    src = (key % n).to(torch.int32)
    deg = torch.bincount(key // n, minlength=n)
    indptr = torch.zeros(n + 1, dtype=torch.int64, device=u.device)
    indptr[1:] = torch.cumsum(deg, 0)
    return indptr, src


def _mean_agg(indptr, indices, h, chunk=1 << 24):
    """out[v] = mean_{u in in(v)} h[u], edge-chunked (data generation only)."""
    n = indptr.numel() - 1
    out = torch.zeros((n, h.shape[1]), dtype=torch.float32, device=h.device)
    deg = (indptr[1:] - indptr[:-1]).to(torch.float32)
    e_total = int(indptr[-1])
    for e0 in range(0, e_total, chunk):
        e1 = min(e_total, e0 + chunk)
        pos = torch.arange(e0, e1, device=h.device)
        dst = torch.searchsorted(indptr, pos, right=True) - 1
        out.index_add_(0, dst, h[indices[e0:e1].long()])
    return out / deg.clamp(min=1).unsqueeze(1)


@dataclass
class SyntheticGraph:
    spec: SyntheticSpec
    u: torch.Tensor          # directed edges incl. both directions, no self-loops
    v: torch.Tensor
    feat: torch.Tensor       # float32 [n, d]
    label: torch.Tensor      # int64 [n]
    train_mask: torch.Tensor  # int8 [n]
    val_mask: torch.Tensor
    test_mask: torch.Tensor

    @property
    def n_nodes(self):
        return self.spec.n_nodes


def build(spec, device="cpu"):
    """Generate the graph, features, teacher labels and splits of ``spec``."""
    if isinstance(spec, str):
        spec = SPECS[spec]
    device = torch.device(device)
    n = spec.n_nodes
    keys = rmat_undirected(spec, device)
    perm = node_permutation(n, spec.seed, device)
    a = perm[keys // n]
    b = perm[keys % n]
    del keys
    u = torch.cat([a, b])
    v = torch.cat([b, a])
    del a, b
    feat = normal(n * spec.feat_dim, spec.seed ^ 0xFEA7, device).view(n, spec.feat_dim)
    # teacher labels on the graph with self-loops
    loops = torch.arange(n, dtype=torch.int64, device=device)
    indptr, indices = csc_from_edges(torch.cat([u, loops]), torch.cat([v, loops]), n)
    g = torch.Generator(device="cpu").manual_seed(spec.seed ^ 0x7EAC)
    w1 = (torch.randn(spec.feat_dim, spec.teacher_hidden, generator=g) / math.sqrt(spec.feat_dim)).to(device)
    w2 = (torch.randn(spec.teacher_hidden, spec.n_classes, generator=g) / math.sqrt(spec.teacher_hidden)).to(device)
    h1 = torch.relu(_mean_agg(indptr, indices, feat @ w1))
    logits = _mean_agg(indptr, indices, h1 @ w2)
    # the teacher's output bias centres every class score, so that no class dominates
    logits = (logits - logits.mean(0, keepdim=True)) / logits.std(0, keepdim=True).clamp(min=1e-6)
    label = torch.argmax(logits, dim=1)
    del h1, logits, indptr, indices
    # splits: nodes ordered by a seeded hash, cut at the fractions
    order = torch.argsort(shuffle_keys(torch.arange(n, dtype=torch.int64, device=device), spec.seed ^ 0x5B1, 0))
    n_tr = int(round(spec.train_frac * n))
    n_va = int(round(spec.val_frac * n))
    train = torch.zeros(n, dtype=torch.int8, device=device)
    val = torch.zeros(n, dtype=torch.int8, device=device)
    test = torch.zeros(n, dtype=torch.int8, device=device)
    train[order[:n_tr]] = 1
    val[order[n_tr:n_tr + n_va]] = 1
    test[order[n_tr + n_va:]] = 1
    return SyntheticGraph(spec, u, v, feat, label, train, val, test)


def to_t10n_layout(graph, out_dir):
    """Write ``graph`` in the reference's pre-partition layout: edge_index.bin.npy (u then v,
    with one self-loop per node), node_feat/label/*_mask .bin.npy and t10n.json
    (t10n/dataset/dgl_to_t10n.py:173-189)."""
    import json
    import os

    os.makedirs(out_dir, exist_ok=True)
    n = graph.n_nodes
    loops = torch.arange(n, dtype=torch.int64)
    u = torch.cat([graph.u.cpu(), loops])
    v = torch.cat([graph.v.cpu(), loops])
    np.save(os.path.join(out_dir, "edge_index.bin.npy"), torch.cat([u, v]).numpy())
    np.save(os.path.join(out_dir, "node_feat.bin.npy"), graph.feat.cpu().numpy().astype(np.float32))
    np.save(os.path.join(out_dir, "node_label.bin.npy"), graph.label.cpu().numpy().astype(np.float32))
    for name, m in (("train", graph.train_mask), ("val", graph.val_mask), ("test", graph.test_mask)):
        np.save(os.path.join(out_dir, f"{name}_mask.bin.npy"), m.cpu().numpy().astype(np.int8))
    cfg = {
        "num_nodes": n,
        "num_edges": int(u.numel()),
        "feat_dim": graph.spec.feat_dim,
        "num_labels": graph.spec.n_classes,
        "edge_file_bin": os.path.join(out_dir, "edge_index.bin.npy"),
        "node_feats_file_bin": os.path.join(out_dir, "node_feat.bin.npy"),
        "node_label_file": os.path.join(out_dir, "node_label.bin.npy"),
        "train_mask_file_bin": os.path.join(out_dir, "train_mask.bin.npy"),
        "val_mask_file_bin": os.path.join(out_dir, "val_mask.bin.npy"),
        "test_mask_file_bin": os.path.join(out_dir, "test_mask.bin.npy"),
        "num_train_nodes": int(graph.train_mask.sum()),
        "add_reverse_edge": True,
    }
    with open(os.path.join(out_dir, "t10n.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    return cfg


# ---------------------------------------------------------------------------------------
# Memory-lean build of one rank's partition (graphs of 10^8 nodes / 10^9 edges).
#
# ``build`` keeps fp32 features and both edge directions as int64 (about 170 GB for the
# ogbn-papers100M shape); this path never holds more than the CSC, the bf16 features and
# two [n, hidden] teacher buffers:
#   * the undirected RMAT edges are turned straight into a CSC by destination (with one
#     self-loop per node), sources ascending per row -- the same graph as ``build``;
#   * features are generated row-wise in bf16 from the same N(0,1) stream (element i of
#     the flattened [n, d] matrix is the same Philox draw as in ``build``);
#   * the 2-hop mean teacher runs in bf16 with the mean-aggregation kernel, using
#     A (A X W1) W2 = (A (A X W1)) W2 to keep the widest buffer at the hidden width;
#   * partitions are contiguous ranges of the (already hash-permuted) node ids, a
#     balanced random hash partition that needs no relabelling: rank r owns
#     [r n / W, (r + 1) n / W), and its in-edge CSR is a slice of the global CSC.
# ---------------------------------------------------------------------------------------
def lean_prefix(n, world):
    return [r * n // world for r in range(world + 1)]


def _csc_with_loops(spec, device):
    n = spec.n_nodes
    keys = rmat_undirected(spec, device)
    perm = node_permutation(n, spec.seed, device)
    m = keys.numel()
    # directed edges (src, dst) of both directions plus the loops, keyed dst * n + src
    dkey = torch.empty(2 * m + n, dtype=torch.int64, device=device)
    step = 1 << 27
    for s in range(0, m, step):
        k = keys[s:s + step]
        a = perm[k // n]
        b = perm[k % n]
        dkey[s:s + k.numel()] = b * n + a
        dkey[m + s:m + s + k.numel()] = a * n + b
        del k, a, b
    del keys, perm
    ids = torch.arange(n, dtype=torch.int64, device=device)
    dkey[2 * m:] = ids * (n + 1)
    del ids
    dkey, _ = torch.sort(dkey)
    indices = torch.empty(dkey.numel(), dtype=torch.int32, device=device)
    deg = torch.zeros(n, dtype=torch.int64, device=device)
    for s in range(0, dkey.numel(), step):
        k = dkey[s:s + step]
        indices[s:s + k.numel()] = (k % n).to(torch.int32)
        deg += torch.bincount(k // n, minlength=n)
        del k
    del dkey
    indptr = torch.zeros(n + 1, dtype=torch.int64, device=device)
    indptr[1:] = torch.cumsum(deg, 0)
    return indptr, indices


def normal_rows(n_rows, row0, d, ld, seed, device):
    """Rows [row0, row0 + n_rows) of the [*, d] N(0,1) matrix of ``normal(. * d, seed)`` as
    bf16 rows of width ld (columns past d are zero)."""
    device = torch.device(device)
    out = torch.zeros((n_rows, ld), dtype=torch.bfloat16, device=device)
    if n_rows == 0:
        return out
    if device.type == "cuda":
        _native.cuda().normal_rows(out, int(row0), int(d), int(seed))
        return out
    flat = torch.from_numpy(_native.host().normal((row0 + n_rows) * d, int(seed)))
    out[:, :d] = flat[row0 * d:].view(n_rows, d).to(torch.bfloat16)
    return out


def _mean_agg_bf16(indptr, indices, h, out, max_edges=1 << 30):
    """out[v] = mean_{u in in(v)} h[u] (bf16 rows, dst-chunked so that edge offsets fit in int32)."""
    n = indptr.numel() - 1
    dim = h.shape[1]
    if h.is_cuda:
        cu = _native.cuda()
        err = torch.zeros(1, dtype=torch.int32, device=h.device)
        ip = indptr.cpu()
        s = 0
        while s < n:
            e = int(torch.searchsorted(ip, ip[s] + max_edges, right=True)) - 1
            e = max(s + 1, min(n, e))
            e0, e1 = int(ip[s]), int(ip[e])
            local = (indptr[s:e + 1] - e0).to(torch.int32)
            cu.aggregate(local, indices[e0:e1], None, e - s, e - s, h, None, dim, 0, None, None, None, out[s:e], 0,
                         -1, 0.0, 0, err, None, 0, 0.0, None, 0)
            s = e
        torch.cuda.synchronize(h.device)
        if int(err.item()):
            raise RuntimeError(f"aggregation error word {int(err.item()):#x} in the teacher")
        return out
    res = _mean_agg(indptr, indices, h.float())
    out.copy_(res.to(out.dtype))
    return out


def _teacher_labels(spec, indptr, indices, feat, device, row_chunk=1 << 22):
    n, d = spec.n_nodes, spec.feat_dim
    g = torch.Generator(device="cpu").manual_seed(spec.seed ^ 0x7EAC)
    w1 = (torch.randn(d, spec.teacher_hidden, generator=g) / math.sqrt(d)).to(device)
    w2 = (torch.randn(spec.teacher_hidden, spec.n_classes, generator=g) / math.sqrt(spec.teacher_hidden)).to(device)
    hid = spec.teacher_hidden
    z = torch.zeros((n, hid), dtype=torch.bfloat16, device=device)
    for s in range(0, n, row_chunk):
        z[s:s + row_chunk] = (feat[s:s + row_chunk, :d].float() @ w1).to(torch.bfloat16)
    h1 = torch.zeros_like(z)
    _mean_agg_bf16(indptr, indices, z, h1)
    h1.relu_()
    _mean_agg_bf16(indptr, indices, h1, z)  # z <- A relu(A X W1)
    del h1
    s1 = torch.zeros(spec.n_classes, dtype=torch.float64, device=device)
    s2 = torch.zeros_like(s1)
    for s in range(0, n, row_chunk):
        lg = z[s:s + row_chunk].float() @ w2
        s1 += lg.sum(0, dtype=torch.float64)
        s2 += (lg.double() ** 2).sum(0)
    mean = s1 / n
    std = ((s2 - n * mean ** 2) / max(1, n - 1)).clamp(min=0).sqrt().clamp(min=1e-6)
    label = torch.empty(n, dtype=torch.int32, device=device)
    for s in range(0, n, row_chunk):
        lg = z[s:s + row_chunk].float() @ w2
        label[s:s + row_chunk] = torch.argmax((lg - mean.float()) / std.float(), dim=1).to(torch.int32)
    return label


def _split_masks(spec, lo, hi, device):
    n = spec.n_nodes
    order = torch.argsort(shuffle_keys(torch.arange(n, dtype=torch.int64, device=device), spec.seed ^ 0x5B1, 0))
    n_tr = int(round(spec.train_frac * n))
    n_va = int(round(spec.val_frac * n))
    split = torch.empty(n, dtype=torch.int8, device=device)  # 0 train, 1 val, 2 test
    split[order[:n_tr]] = 0
    split[order[n_tr:n_tr + n_va]] = 1
    split[order[n_tr + n_va:]] = 2
    del order
    own = split[lo:hi]
    return [(own == k).to(torch.int8) for k in range(3)]


def build_partition(spec, world, rank, device):
    """Rank ``rank``'s OwnPartition of ``spec``'s graph, built without the global fp32
    arrays of ``build`` (see the notes above).  Every rank builds the global CSC and the
    teacher on its own device and keeps its slice."""
    from grappa_b200.graph_store import OwnPartition
    from grappa_b200.models.flat import pad8

    if isinstance(spec, str):
        spec = SPECS[spec]
    device = torch.device(device)
    n, d = spec.n_nodes, spec.feat_dim
    prefix = lean_prefix(n, world)
    lo, hi = prefix[rank], prefix[rank + 1]
    indptr, indices = _csc_with_loops(spec, device)
    feat = normal_rows(n, 0, d, pad8(d), spec.seed ^ 0xFEA7, device)
    label = _teacher_labels(spec, indptr, indices, feat, device)
    gideg = (indptr[1:] - indptr[:-1] - 1)[lo:hi].clone()
    if world > 1:
        e0, e1 = int(indptr[lo]), int(indptr[hi])
        own_indptr = indptr[lo:hi + 1] - e0
        own_indices = indices[e0:e1].clone()
        del indptr, indices
        own_feat = feat[lo:hi].clone()
        del feat
        label = label[lo:hi].clone()
    else:
        own_indptr, own_indices, own_feat = indptr, indices, feat
    tr, va, te = _split_masks(spec, lo, hi, device)
    ext = own_indices[(own_indices < lo) | (own_indices >= hi)]
    ext_src = torch.unique(ext).to(torch.int32)
    del ext
    if device.type == "cuda":
        torch.cuda.empty_cache()
    return OwnPartition(rank, world, prefix, own_indptr, own_indices, own_feat, label, tr, va, te, gideg, ext_src,
                        feat_dim=d)


# graphs above this size are built per partition by ``build_partition``
LEAN_MIN_NODES = 20_000_000
