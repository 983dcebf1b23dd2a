"""Timings of the host (CPU) engine's paths on fixed inputs:

* ``xborder``  ``XBorder.group_by_partition`` with its [P, n] mask on the input of the
  reference's own timing script (test/test_xborder.py:8-55: 16 partitions of 1M ids,
  1M ids drawn over partitions 1-15 and 9M over partition 0), median of 10;
* ``csc``      ``HostGraph`` (in-edge CSC, deduplicated, sorted) of a seeded synthetic
  graph, median of 3;
* ``sample``   ``sample_batch`` of 1024 seeds with fan-out [15, 10, 5] on that graph,
  mean of 20;
* ``metis``    the multilevel partitioner (the chunkers' ``metis`` method) into
  ``--parts`` parts, one run, with its edge cut.

    python -m grappa_b200.utils.bench_host [--graph ogbpr] [--parts 8] [--only xborder,csc]

Prints one JSON object per measurement.  Threads: OMP_NUM_THREADS (default: all CPUs).
"""
import argparse
import json
import os
import time

import numpy as np
import torch

from grappa_b200 import host


def bench_xborder(reps=10):
    from grappa_b200.xborder import xb_group_by_partition

    n_part, npp = 16, 1000000
    prefix = [npp * i for i in range(n_part + 1)]
    g = torch.Generator().manual_seed(0)
    ids = torch.cat([torch.randint(npp, 16 * npp, (npp,), generator=g), torch.randint(0, npp, (9 * npp,), generator=g)])
    xb = host().xborder.XBorder(0, n_part, prefix)
    for _ in range(3):
        xb_group_by_partition(xb, ids, n_part)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        xb_group_by_partition(xb, ids, n_part)
        ts.append(time.perf_counter() - t0)
    return {"bench": "xborder.group_by_partition", "ids": int(ids.numel()), "parts": n_part,
            "median_s": float(np.median(ts)), "min_s": float(min(ts))}


def _graph(name):
    from grappa_b200.dataset import synthetic

    spec = synthetic.SPECS[name]
    keys = synthetic.rmat_undirected(spec, "cpu")
    n = spec.n_nodes
    perm = synthetic.node_permutation(n, spec.seed, "cpu")
    a, b = perm[keys // n], perm[keys % n]
    del keys
    tr = np.zeros(n, dtype=np.int8)
    tr[np.random.default_rng(spec.seed).permutation(n)[: int(spec.train_frac * n)]] = 1
    return n, torch.cat([a, b]).numpy(), torch.cat([b, a]).numpy(), tr


def bench_csc(n, u, v, reps=3):
    G = host().graph
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        g = G.HostGraph(u, v, n)
        ts.append(time.perf_counter() - t0)
        m = g.n_edges
        del g
    return {"bench": "HostGraph", "nodes": n, "directed_edges": int(len(u)), "csc_edges": int(m),
            "median_s": float(np.median(ts))}


def bench_sample(n, u, v, reps=20):
    G = host().graph
    g = G.HostGraph(u, v, n)
    seeds = np.arange(0, n, max(1, n // 1024), dtype=np.int64)[:1024]
    G.sample_batch(g, [15, 10, 5], seeds, None, 0, 0, 0, False)
    t0 = time.perf_counter()
    for s in range(reps):
        G.sample_batch(g, [15, 10, 5], seeds, None, 0, 0, s, False)
    return {"bench": "sample_batch", "seeds": int(len(seeds)), "fanout": [15, 10, 5],
            "mean_ms": (time.perf_counter() - t0) / reps * 1e3}


def bench_metis(n, u, v, tr, parts):
    c = host().c_seq
    t0 = time.perf_counter()
    p = c.multilevel_partition(n, u, v, parts, tr, 0, 0.03)
    t = time.perf_counter() - t0
    cut = int(c.edge_cut(n, u, v, p)) if hasattr(c, "edge_cut") else None
    sizes = np.bincount(p, minlength=parts)
    return {"bench": "multilevel_partition", "nodes": n, "directed_edges": int(len(u)), "parts": parts,
            "seconds": t, "edge_cut": cut, "undirected_edges": int(len(u) // 2),
            "node_imbalance": float(sizes.max() * parts / n)}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--graph", default="ogbpr", help="synthetic graph for csc / sample / metis")
    ap.add_argument("--parts", type=int, default=8)
    ap.add_argument("--only", default="xborder,csc,sample,metis")
    a = ap.parse_args(argv)
    only = set(a.only.split(","))
    threads = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    out = []
    if "xborder" in only:
        out.append(bench_xborder())
    if only & {"csc", "sample", "metis"}:
        n, u, v, tr = _graph(a.graph)
        if "csc" in only:
            out.append(bench_csc(n, u, v))
        if "sample" in only:
            out.append(bench_sample(n, u, v))
        if "metis" in only:
            out.append(bench_metis(n, u, v, tr, a.parts))
    for r in out:
        r.update(threads=threads, graph=a.graph if r["bench"] != "xborder.group_by_partition" else "reference input")
        print(json.dumps(r), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
