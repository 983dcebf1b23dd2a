"""Host memory and host<->GPU copy bandwidth per NUMA node (reference: test/numa_bench.c,
which measures OpenMP write/read bandwidth of a 256 MB buffer on node 0 and node 1).

* host matrix: write and read GB/s of a buffer placed on each memory node, streamed by
  threads pinned to each CPU node (libnuma-free: first touch under a preferred-node
  policy, see grappa_b200/csrc/host/numa.cc);
* with CUDA: pinned host buffers placed on each memory node, copied to and from each GPU
  with ``cudaMemcpyAsync`` (``Tensor.copy_`` with non_blocking) timed by CUDA events, best
  of ``--reps``; the GPU's own NUMA node is printed beside it.  These are the copies of the
  end-to-end step (pinned seed tables and batch inputs in, losses out).

    python -m grappa_b200.utils.numa_bench [--mbytes 256] [--threads 0] [--reps 3] [--json]
"""
import argparse
import json
import sys

import numpy as np
import torch

from grappa_b200 import host
from grappa_b200.device_allocator import T10nDeviceAllocator


def host_matrix(mbytes=256, threads=0, reps=3):
    """[{cpu_node, mem_node, mem_node_seen, write_gbs, read_gbs}] over all node pairs."""
    numa = host().numa
    nodes = numa.nodes()
    rows = []
    for c in nodes:
        if not numa.node_cpus(c):
            continue  # a memory-only node, or CPUs outside this process's cpuset
        for m in nodes:
            rows.append(numa.bandwidth(c, m, mbytes, threads, reps))
    return rows


def pinned_on(node, nbytes):
    """A pinned host buffer whose pages come from NUMA node ``node`` (first touch by the
    pinning call under a preferred-node policy), and the node the kernel reports."""
    numa = host().numa
    with numa.MemPolicy(node):
        buf = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
        buf.fill_(1)
    return buf, numa.node_of(buf.numpy())


def copy_bandwidth(device, buf, reps=3):
    """Best-of-reps H2D and D2H GB/s between a pinned host buffer and ``device``."""
    dev = torch.empty(buf.numel(), dtype=torch.uint8, device=device)
    s = torch.cuda.Stream(device=device)
    best = {"h2d": float("inf"), "d2h": float("inf")}
    with torch.cuda.device(device), torch.cuda.stream(s):
        for name, dst, src in (("h2d", dev, buf), ("d2h", buf, dev)):
            for i in range(reps + 1):  # the first pass warms the path up
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize(device)
                a.record(s)
                dst.copy_(src, non_blocking=True)
                b.record(s)
                b.synchronize()
                if i:
                    best[name] = min(best[name], a.elapsed_time(b) / 1e3)
    n = buf.numel()
    return {"h2d_gbs": n / best["h2d"] / 1e9, "d2h_gbs": n / best["d2h"] / 1e9}


def gpu_matrix(mbytes=256, reps=3):
    """[{gpu, gpu_numa_node, mem_node, mem_node_seen, h2d_gbs, d2h_gbs}] for every GPU and
    memory node; empty without CUDA."""
    if not torch.cuda.is_available():
        return []
    ta = T10nDeviceAllocator(torch.cuda.device_count())
    rows = []
    for m in host().numa.nodes():
        buf, seen = pinned_on(m, mbytes << 20)
        for g in range(torch.cuda.device_count()):
            r = copy_bandwidth(torch.device("cuda", g), buf, reps)
            rows.append({"gpu": g, "gpu_numa_node": ta.get_numa_affinity(g), "mem_node": m, "mem_node_seen": seen,
                         **r})
        del buf
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--mbytes", type=int, default=256)
    ap.add_argument("--threads", type=int, default=0, help="threads per CPU node (0: all its CPUs)")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--no_gpu", action="store_true")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    hrows = host_matrix(a.mbytes, a.threads, a.reps)
    grows = [] if a.no_gpu else gpu_matrix(a.mbytes, a.reps)
    if a.json:
        print(json.dumps({"host": hrows, "gpu": grows}))
        return 0
    print(f"NUMA nodes: {host().numa.nodes()}")
    print("| CPU node | memory node | placed on | write GB/s | read GB/s |")
    print("|---:|---:|---:|---:|---:|")
    for r in hrows:
        print(f"| {r['cpu_node']} | {r['mem_node']} | {r['mem_node_seen']} | {r['write_gbs']:.1f} | "
              f"{r['read_gbs']:.1f} |")
    if grows:
        print()
        print("| GPU | GPU's node | pinned memory node | placed on | H2D GB/s | D2H GB/s |")
        print("|---:|---:|---:|---:|---:|---:|")
        for r in grows:
            print(f"| {r['gpu']} | {r['gpu_numa_node']} | {r['mem_node']} | {r['mem_node_seen']} | "
                  f"{r['h2d_gbs']:.1f} | {r['d2h_gbs']:.1f} |")
    return 0


if __name__ == "__main__":
    sys.exit(main())
