"""Raw graph -> the pre-partition layout read by the chunk builders
(reference: t10n/dataset/dgl_to_t10n.py:95-189, 295-418).

Layout of ``{dest}/{name}/``: ``edge_index.bin.npy`` (int64, all sources then all
destinations), ``node_feat.bin.npy`` (float32 [n, d]), ``node_label.bin.npy``
(float32), ``{train,val,test}_mask.bin.npy`` (int8) and ``t10n.json`` with the
reference's keys (node_label_file, edge_file_bin, node_feats_file_bin,
train/val/test_mask_file_bin, num_train_nodes, num_nodes, num_edges, feat_dim,
num_labels, add_reverse_edge).  As the reference's augmentation does, one
self-loop per node is added (t10n/dataset/dgl_to_t10n.py:95-99).

The reference loads its inputs through DGL/OGB dataset classes; this converter
reads the files those classes read, without DGL:
  * an OGB node-property directory (raw/edge.csv.gz, raw/node-feat.csv.gz,
    raw/node-label.csv.gz, split/<scheme>/{train,valid,test}.csv.gz), or its
    raw/data.npz + raw/node-label.npz form (ogbn-papers100M);
  * DGL's Reddit files (reddit_data.npz, reddit_graph.npz);
  * the IGB release's arrays (paper/node_feat.npy, paper/node_label_19.npy,
    paper__cites__paper/edge_index.npy), linked rather than copied;
  * a .npz archive with edge_index [2, m] (or src/dst), feat, label and
    train/val/test masks or index arrays.

The reference's function names are kept: ``load_as_dgl_g`` returns a ``GraphArrays``
(the slice of DGL's graph API the converter uses: ``edges()``, ``num_nodes()``,
``ndata``), ``augmentation_dgl_g`` replaces self-loops by one per node, and
``to_t10n_from_dgl_g`` / ``to_t10n_from_downloaded_ds`` write the layout.  A real DGL
graph is accepted wherever a GraphArrays is.  Cora and MAG240M ship in DGL's own
pickle/binary formats, which need DGL to read.

    python -m grappa_b200.dataset.dgl_to_t10n --src DIR_OR_NPZ --dest DIR --name NAME [--bidirected]
"""
import argparse
import json
import os

import numpy as np


def write_t10n(out_dir, src, dst, feat, label, train, val, test, add_self_loop=True, bidirected=False):
    """Write the layout; masks are 0/1 arrays of length n.  Returns the t10n.json dict."""
    os.makedirs(out_dir, exist_ok=True)
    n = int(feat.shape[0])
    src = np.asarray(src, dtype=np.int64)
    dst = np.asarray(dst, dtype=np.int64)
    if bidirected:
        src, dst = np.concatenate([src, dst]), np.concatenate([dst, src])
    if add_self_loop:
        keep = src != dst
        loops = np.arange(n, dtype=np.int64)
        src = np.concatenate([src[keep], loops])
        dst = np.concatenate([dst[keep], loops])
    files = {
        "edge_file_bin": "edge_index.bin.npy",
        "node_feats_file_bin": "node_feat.bin.npy",
        "node_label_file": "node_label.bin.npy",
        "train_mask_file_bin": "train_mask.bin.npy",
        "val_mask_file_bin": "val_mask.bin.npy",
        "test_mask_file_bin": "test_mask.bin.npy",
    }
    paths = {k: os.path.join(out_dir, v) for k, v in files.items()}
    np.save(paths["edge_file_bin"], np.concatenate([src, dst]))
    np.save(paths["node_feats_file_bin"], np.ascontiguousarray(feat, dtype=np.float32))
    lab = np.asarray(label, dtype=np.float32).reshape(-1)
    np.save(paths["node_label_file"], lab)
    for key, m in (("train_mask_file_bin", train), ("val_mask_file_bin", val), ("test_mask_file_bin", test)):
        np.save(paths[key], np.asarray(m, dtype=np.int8))
    valid = lab[np.isfinite(lab)]
    cfg = dict(paths)
    cfg.update({
        "num_train_nodes": int(np.asarray(train).sum()),
        "num_nodes": n,
        "num_edges": int(src.shape[0]),
        "feat_dim": int(feat.shape[1]),
        "num_labels": int(valid.max()) + 1 if valid.size else 0,
        "add_reverse_edge": bool(bidirected),
    })
    with open(os.path.join(out_dir, "t10n.json"), "w") as f:
        json.dump(cfg, f, indent=4)
    return cfg


def _mask(n, idx):
    m = np.zeros(n, dtype=np.int8)
    m[np.asarray(idx, dtype=np.int64).reshape(-1)] = 1
    return m


def load_ogb_raw(src_dir, split="sales_ranking"):
    """Arrays of an OGB node-property dataset directory (the files its loader reads)."""
    import pandas as pd

    raw = os.path.join(src_dir, "raw")
    edges = pd.read_csv(os.path.join(raw, "edge.csv.gz"), header=None).values.astype(np.int64)
    feat = pd.read_csv(os.path.join(raw, "node-feat.csv.gz"), header=None).values.astype(np.float32)
    label = pd.read_csv(os.path.join(raw, "node-label.csv.gz"), header=None).values.reshape(-1).astype(np.float32)
    split_dir = os.path.join(src_dir, "split")
    if not os.path.isdir(os.path.join(split_dir, split)):
        split = sorted(os.listdir(split_dir))[0]
    idx = {k: pd.read_csv(os.path.join(split_dir, split, f"{k}.csv.gz"), header=None).values.reshape(-1)
           for k in ("train", "valid", "test")}
    n = feat.shape[0]
    return edges[:, 0], edges[:, 1], feat, label, _mask(n, idx["train"]), _mask(n, idx["valid"]), _mask(n, idx["test"])


def load_npz(path):
    z = np.load(path)
    if "edge_index" in z:
        src, dst = z["edge_index"][0], z["edge_index"][1]
    else:
        src, dst = z["src"], z["dst"]
    feat, label = z["feat"], z["label"]
    n = feat.shape[0]

    def get(name):
        for k in (f"{name}_mask", name, f"{name}_idx"):
            if k in z:
                a = z[k]
                return a.astype(np.int8) if a.shape[0] == n and a.max() <= 1 else _mask(n, a)
        return np.zeros(n, dtype=np.int8)

    return src, dst, feat, label, get("train"), get("val"), get("test")


def convert(src, dest, name, bidirected=False):
    out = os.path.join(dest, name)
    arrays = load_npz(src) if src.endswith(".npz") else load_ogb_raw(src)
    return write_t10n(out, *arrays, add_self_loop=True, bidirected=bidirected)


class GraphArrays:
    """A graph as arrays with the part of DGL's graph API the converter reads."""

    def __init__(self, src, dst, num_nodes, ndata=None):
        self.src = np.asarray(src, dtype=np.int64)
        self.dst = np.asarray(dst, dtype=np.int64)
        self._n = int(num_nodes)
        self.ndata = dict(ndata or {})

    def edges(self):
        import torch

        return torch.from_numpy(self.src), torch.from_numpy(self.dst)

    def num_nodes(self):
        return self._n

    number_of_nodes = num_nodes

    def num_edges(self):
        return int(self.src.shape[0])


def _np(a):
    return a.numpy() if hasattr(a, "numpy") else np.asarray(a)


def _ogb_dir(root, meta):
    for d in (os.path.join(root, meta.origin_name.replace("-", "_")), os.path.join(root, meta.origin_name), root):
        if os.path.isdir(os.path.join(d, "raw")):
            return d
    raise FileNotFoundError(f"no OGB directory of {meta.origin_name} under {root}")


def _load_ogb_npz(d, split):
    """ogbn-papers100M's raw form: raw/data.npz (edge_index [2, m] or edge_idx [m, 2],
    node_feat, num_nodes_list), raw/node-label.npz, split/<scheme>/*.csv.gz."""
    import pandas as pd

    data = np.load(os.path.join(d, "raw", "data.npz"))
    if "edge_index" in data:
        e = data["edge_index"]
        src, dst = e[0], e[1]
    else:
        e = data["edge_idx"]
        src, dst = e[:, 0], e[:, 1]
    feat = data["node_feat"]
    n = int(data["num_nodes_list"][0]) if "num_nodes_list" in data else feat.shape[0]
    lab = np.load(os.path.join(d, "raw", "node-label.npz"))
    label = lab[lab.files[0]].astype(np.float32).reshape(-1)
    split_dir = os.path.join(d, "split")
    if not os.path.isdir(os.path.join(split_dir, split)):
        split = sorted(os.listdir(split_dir))[0]
    idx = {k: pd.read_csv(os.path.join(split_dir, split, f"{k}.csv.gz"), header=None).values.reshape(-1)
           for k in ("train", "valid", "test")}
    return src, dst, feat, label, _mask(n, idx["train"]), _mask(n, idx["valid"]), _mask(n, idx["test"])


def _load_reddit(root):
    """DGL's Reddit files: reddit_data.npz (feature, label, node_types 1/2/3 =
    train/val/test) and reddit_graph.npz (a scipy sparse adjacency)."""
    import scipy.sparse as sp

    d = os.path.join(root, "reddit") if os.path.isdir(os.path.join(root, "reddit")) else root
    data = np.load(os.path.join(d, "reddit_data.npz"))
    adj = sp.load_npz(os.path.join(d, "reddit_graph.npz")).tocoo()
    types = data["node_types"]
    return (adj.row, adj.col, data["feature"], data["label"].astype(np.float32), (types == 1).astype(np.int8),
            (types == 2).astype(np.int8), (types == 3).astype(np.int8))


def _igb_files(root, meta):
    base = os.path.join(root, meta.origin_path) if meta.origin_path else root
    if not os.path.isdir(os.path.join(base, "paper")):
        base = root
    return (os.path.join(base, "paper", "node_feat.npy"), os.path.join(base, "paper", "node_label_19.npy"),
            os.path.join(base, "paper__cites__paper", "edge_index.npy"))


def _open_array(path, dtype, shape=None):
    """np.load of an .npy file, or a raw memory map of ``dtype`` when the file has no
    .npy header."""
    with open(path, "rb") as f:
        magic = f.read(6)
    if magic == b"\x93NUMPY":
        return np.load(path, mmap_mode="r")
    return np.memmap(path, dtype=dtype, mode="r", shape=shape)


def _split_masks(n, train=0.6, val=0.2):
    """Index-range masks: the first 60 % train, the next 20 % validation, the rest test."""
    n_tr, n_va = int(n * train), int(n * val)
    masks = [np.zeros(n, dtype=np.int8) for _ in range(3)]
    masks[0][:n_tr] = 1
    masks[1][n_tr:n_tr + n_va] = 1
    masks[2][n_tr + n_va:] = 1
    return masks


def load_as_dgl_g(dest_path, dataset_name):
    """Load a downloaded dataset as a GraphArrays with ndata feat, label, train_mask,
    val_mask and test_mask (reference: t10n/dataset/dgl_to_t10n.py:19-92)."""
    from grappa_b200.dataset.meta import name_to_meta

    meta = name_to_meta(dataset_name)
    if dataset_name.startswith("ogb"):
        d = _ogb_dir(dest_path, meta)
        if os.path.exists(os.path.join(d, "raw", "data.npz")):
            arrays = _load_ogb_npz(d, "time")
        else:
            arrays = load_ogb_raw(d)
    elif dataset_name == "reddit":
        arrays = _load_reddit(dest_path)
    elif dataset_name == "igb260m":
        feat_f, label_f, edge_f = _igb_files(dest_path, meta)
        e = _open_array(edge_f, np.int64)
        label = np.asarray(_open_array(label_f, np.float32)).reshape(-1)
        n = label.shape[0]
        feat = _open_array(feat_f, np.float32, (n, meta.n_dim))
        arrays = (e[:, 0], e[:, 1], feat, label, *_split_masks(n))
    else:
        raise NotImplementedError(f"{dataset_name} ships in DGL's own format; load it with DGL and pass the graph "
                                  "to to_t10n_from_dgl_g, or save it as .npz for convert()")
    src, dst, feat, label, tr, va, te = arrays
    n = int(np.asarray(label).reshape(-1).shape[0])
    return GraphArrays(src, dst, n, {"feat": feat, "label": np.asarray(label, dtype=np.float32).reshape(-1),
                                     "train_mask": tr, "val_mask": va, "test_mask": te})


def augmentation_dgl_g(dgl_g):
    """The graph without its self-loops plus one self-loop per node (reference:
    t10n/dataset/dgl_to_t10n.py:95-98)."""
    if not isinstance(dgl_g, GraphArrays):
        import dgl  # a DGL graph: DGL's own operations

        return dgl.add_self_loop(dgl.remove_self_loop(dgl_g))
    keep = dgl_g.src != dgl_g.dst
    loops = np.arange(dgl_g.num_nodes(), dtype=np.int64)
    return GraphArrays(np.concatenate([dgl_g.src[keep], loops]), np.concatenate([dgl_g.dst[keep], loops]),
                       dgl_g.num_nodes(), dgl_g.ndata)


def get_num_labels(labels):
    """Distinct labels, NaN (unlabelled) excluded."""
    a = np.asarray(_np(labels), dtype=np.float64).reshape(-1)
    return int(np.unique(a[~np.isnan(a)]).shape[0])


def to_t10n_from_dgl_g(dest_path, dataset_name, dgl_g):
    """Write ``dgl_g`` (GraphArrays or a DGL graph with ndata feat/label/*_mask) as
    ``dest_path/dataset_name`` in the pre-partition layout, self-loops replaced by one
    per node (reference: t10n/dataset/dgl_to_t10n.py:107-189).  Returns the path of its
    t10n.json."""
    src, dst = dgl_g.edges()
    nd = dgl_g.ndata
    n = int(dgl_g.num_nodes())
    masks = [(_np(nd[k]) != 0).astype(np.int8) if k in nd else np.zeros(n, dtype=np.int8)
             for k in ("train_mask", "val_mask", "test_mask")]
    cfg = write_t10n(os.path.join(dest_path, dataset_name), _np(src), _np(dst), _np(nd["feat"]), _np(nd["label"]),
                     *masks, add_self_loop=True)
    cfg["num_labels"] = get_num_labels(nd["label"])
    path = os.path.join(dest_path, dataset_name, "t10n.json")
    with open(path, "w") as f:
        json.dump(cfg, f, indent=4)
    return path


def _igb_to_t10n(dest_path, src_path):
    """IGB260M: the release's arrays linked into the layout unchanged (row-pair edges
    without added self-loops, raw or .npy features and labels) plus index-range
    masks."""
    from grappa_b200.dataset.meta import name_to_meta

    meta = name_to_meta("igb260m")
    out = os.path.join(dest_path, meta.name)
    cfg_f = os.path.join(out, "t10n.json")
    if os.path.exists(cfg_f):
        return cfg_f
    os.makedirs(out, exist_ok=True)
    feat_f, label_f, edge_f = _igb_files(src_path, meta)
    e = _open_array(edge_f, np.int64)
    if e.ndim != 2 or e.shape[1] != 2:
        raise ValueError(f"{edge_f}: expected [m, 2] int64 edges, found {e.shape}")
    label = np.asarray(_open_array(label_f, np.float32)).reshape(-1)
    n = int(label.shape[0])
    feat = _open_array(feat_f, np.float32)
    dim = int(feat.shape[1]) if feat.ndim == 2 else int(feat.size // n)
    links = {"edge_file_bin": ("edge_index.bin.npy", edge_f),
             "node_feats_file_bin": ("node_feat.mmap.npy", feat_f),
             "node_label_file": ("node_label.mmap.npy", label_f)}
    cfg = {}
    for key, (name, target) in links.items():
        link = os.path.join(out, name)
        if not os.path.lexists(link):
            os.symlink(os.path.abspath(target), link)
        cfg[key] = link
    tr, va, te = _split_masks(n)
    for key, name, m in (("train_mask_file_bin", "train_mask.bin.npy", tr), ("val_mask_file_bin", "val_mask.bin.npy", va),
                         ("test_mask_file_bin", "test_mask.bin.npy", te)):
        np.save(os.path.join(out, name), m)
        cfg[key] = os.path.join(out, name)
    cfg.update({"num_train_nodes": int(tr.sum()), "num_nodes": n, "num_edges": int(e.shape[0]), "feat_dim": dim,
                "num_labels": get_num_labels(label), "add_reverse_edge": False})
    with open(cfg_f, "w") as f:
        json.dump(cfg, f, indent=4)
    return cfg_f


def _ogbpa_to_t10n(dest_path, src_path):
    from grappa_b200.dataset.meta import name_to_meta

    meta = name_to_meta("ogbpa")
    out = os.path.join(dest_path, meta.name)
    cfg_f = os.path.join(out, "t10n.json")
    if os.path.exists(cfg_f):
        return cfg_f
    src, dst, feat, label, tr, va, te = _load_ogb_npz(_ogb_dir(src_path, meta), "time")
    write_t10n(out, src, dst, feat, label, tr, va, te, add_self_loop=True)
    return cfg_f


def to_t10n_from_downloaded_ds(dest_path, dataset_name, src_path):
    """Convert a downloaded ogbn-papers100M (``ogbpa``) or IGB260M (``igb260m``) without
    going through a graph object (reference: t10n/dataset/dgl_to_t10n.py:193-418).
    Returns the path of the t10n.json."""
    if dataset_name == "ogbpa":
        return _ogbpa_to_t10n(dest_path, src_path)
    if dataset_name == "igb260m":
        return _igb_to_t10n(dest_path, src_path)
    raise ValueError(f"{dataset_name}: only ogbpa and igb260m convert from their downloaded files")


def main():
    ap = argparse.ArgumentParser(description="convert a raw graph to the t10n pre-partition layout")
    ap.add_argument("--src", required=True)
    ap.add_argument("--dest", required=True)
    ap.add_argument("--name", required=True)
    ap.add_argument("--bidirected", action="store_true", help="add the reverse of every edge")
    a = ap.parse_args()
    print(json.dumps(convert(a.src, a.dest, a.name, a.bidirected), indent=1))


if __name__ == "__main__":
    main()
