"""Command line of the offline dataset pipeline: a graph in the pre-partition layout
(``t10n.json`` + ``*.bin.npy``) becomes the per-partition chunk directory
``{dest_path}/chunking_{graph}_{method}_{n_part:03}`` that the training entry points read.

Reference: experiments/grappa/dataset_to_t10n.py (conversion driver),
experiments/grappa/partition.sh.template (runs a ``build_chunks_dist.py`` that the
reference does not ship), t10n/dataset/chunk_seq.py:110-150 and
t10n/dataset/chunk_dist.py:278-318 (the two chunkers).

    # seeded synthetic graph of a benchmark shape, pre-partition layout
    python -m grappa_b200.dataset.partition generate --graph_name rmat16k --out DATA/t10n/rmat16k
    # chunks in one process (methods: hash, random, metis, lp)
    python -m grappa_b200.dataset.partition seq --src_path DATA/t10n/rmat16k --dest_path DATA \\
        --graph_name rmat16k --part_method metis --n_part 8
    # chunks with gloo ranks, each writing n_part / ranks partitions (hash partitioning)
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m grappa_b200.dataset.partition dist --src_path DATA/t10n/rmat16k --dest_path DATA \\
        --graph_name rmat16k --n_part 16
    # what a chunk directory holds: nodes, edges, bridges, training nodes per partition
    python -m grappa_b200.dataset.partition info --path DATA/chunking_rmat16k_metis_008
"""
import argparse
import glob
import json
import os
import re
import sys

import numpy as np


def generate(graph_name, out):
    """Write the seeded synthetic graph ``graph_name`` (a key of synthetic.SPECS) in the
    pre-partition layout under ``out``; returns its t10n.json dict."""
    from grappa_b200.dataset import synthetic

    if graph_name not in synthetic.SPECS:
        raise ValueError(f"unknown synthetic graph {graph_name}; one of {sorted(synthetic.SPECS)}")
    return synthetic.to_t10n_layout(synthetic.build(graph_name), out)


def chunk_info(path):
    """Per-partition counts of a chunk directory: nodes, intra edges (self-loops
    included), outgoing and incoming bridge edges, distinct remote sources of the incoming
    bridges (halo), training / validation / test nodes."""
    parts = sorted(int(m.group(1)) for f in glob.glob(os.path.join(path, "p*.oid.bin"))
                   if (m := re.search(r"p(\d+)\.oid\.bin$", f)))
    if not parts or parts != list(range(len(parts))):
        raise FileNotFoundError(f"{path} holds no complete chunk set (p0.oid.bin ... p(k-1).oid.bin)")
    k = len(parts)

    def n64(name):
        f = os.path.join(path, name)
        return os.path.getsize(f) // 8 if os.path.exists(f) else 0

    def n_set(name):
        f = os.path.join(path, name)
        return int(np.fromfile(f, dtype=np.int8).astype(np.int64).sum()) if os.path.exists(f) else 0

    def halo(i):
        # distinct nodes of other partitions with an edge into partition i: the rows a
        # working set holding partition i must fetch from elsewhere
        n = 0
        for j in range(k):
            f = os.path.join(path, f"b{j}_{i}.u.bin")
            if j != i and os.path.exists(f):
                n += int(np.unique(np.fromfile(f, dtype=np.int64)).shape[0])
        return n

    rows = []
    for i in range(k):
        out_b = sum(n64(f"b{i}_{j}.u.bin") for j in range(k) if j != i)
        in_b = sum(n64(f"b{j}_{i}.u.bin") for j in range(k) if j != i)
        rows.append({"part": i, "nodes": n64(f"p{i}.oid.bin"), "intra_edges": n64(f"p{i}.u.bin"),
                     "bridge_out": out_b, "bridge_in": in_b, "halo_in": halo(i), "train": n_set(f"p{i}.train.bin"),
                     "valid": n_set(f"p{i}.valid.bin"), "test": n_set(f"p{i}.test.bin")})
    total_intra = sum(r["intra_edges"] - r["nodes"] for r in rows)  # without the self-loops
    total_bridge = sum(r["bridge_out"] for r in rows)
    summary = {"n_part": k, "nodes": sum(r["nodes"] for r in rows),
               "edges": total_intra + total_bridge,
               "cut_fraction": total_bridge / max(1, total_intra + total_bridge),
               "node_imbalance": max(r["nodes"] for r in rows) * k / max(1, sum(r["nodes"] for r in rows)),
               "train_imbalance": max(r["train"] for r in rows) * k / max(1, sum(r["train"] for r in rows))}
    return summary, rows


def _table(summary, rows):
    cols = ["part", "nodes", "intra_edges", "bridge_out", "bridge_in", "halo_in", "train", "valid", "test"]
    out = ["| " + " | ".join(cols) + " |", "|" + "|".join(["---:"] * len(cols)) + "|"]
    out += ["| " + " | ".join(str(r[c]) for c in cols) + " |" for r in rows]
    out.append("")
    out.append(json.dumps(summary))
    return "\n".join(out)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("generate", help="seeded synthetic graph in the pre-partition layout")
    g.add_argument("--graph_name", required=True)
    g.add_argument("--out", required=True)
    for name, help_ in (("seq", "chunks in one process"), ("dist", "chunks with gloo ranks (n_part a multiple of them)")):
        p = sub.add_parser(name, help=help_)
        p.add_argument("--src_path", required=True, help="directory with t10n.json")
        p.add_argument("--dest_path", required=True)
        p.add_argument("--graph_name", required=True)
        p.add_argument("--seed", type=int, default=0)
        if name == "seq":
            p.add_argument("--part_method", default="hash", choices=["hash", "random", "metis", "lp"])
            p.add_argument("--n_part", type=int, required=True)
            p.add_argument("--verbose", action="store_true", help="per-phase seconds of the metis partitioner")
        else:
            p.add_argument("--part_method", default="hash", choices=["hash", "random"])
            p.add_argument("--n_part", type=int, default=None, help="a multiple of the ranks (default: the ranks)")
            p.add_argument("--pg_timeout", type=int, default=600, help="seconds")
    i = sub.add_parser("info", help="per-partition counts of a chunk directory")
    i.add_argument("--path", required=True)
    i.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)

    if a.cmd == "generate":
        cfg = generate(a.graph_name, a.out)
        print(json.dumps({k: cfg[k] for k in ("num_nodes", "num_edges", "feat_dim", "num_labels",
                                              "num_train_nodes")}))
        return 0
    if a.cmd == "seq":
        from grappa_b200.dataset.chunk_seq import build_chunks_seq

        if a.verbose:
            os.environ["GRAPPA_MLPART_VERBOSE"] = "1"  # read by the partitioner at each call

        out, _ = build_chunks_seq(a.dest_path, a.graph_name, a.src_path, a.part_method, a.n_part, a.seed)
        print(_table(*chunk_info(out)))
        return 0
    if a.cmd == "dist":
        import datetime

        import torch.distributed as dist

        from grappa_b200.dataset.chunk_dist import build_chunks_dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=a.pg_timeout))
        try:
            out = build_chunks_dist(dist.get_world_size(), dist.get_rank(), a.dest_path, a.graph_name, a.src_path,
                                    a.part_method, a.n_part, a.seed)
            if dist.get_rank() == 0:
                print(_table(*chunk_info(out)))
        finally:
            dist.destroy_process_group()
        return 0
    summary, rows = chunk_info(a.path)
    print(json.dumps({"summary": summary, "parts": rows}) if a.json else _table(summary, rows))
    return 0


if __name__ == "__main__":
    sys.exit(main())
