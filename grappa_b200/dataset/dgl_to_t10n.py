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
    raw/node-label.csv.gz, split/<scheme>/{train,valid,test}.csv.gz);
  * a .npz archive with edge_index [2, m] (or src/dst), feat, label and
    train/val/test masks or index arrays.

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
