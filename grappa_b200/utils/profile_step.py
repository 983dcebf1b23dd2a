"""Profiling entry point: one mini-batch training step of a model inside an NVTX
range named ``prof_step`` (after one eager warm-up step).

Kernel captures stay small.  On the full-size graph only the one-pass launch list
is collected:

    ncu --metrics gpu__time_duration.sum --clock-control none --nvtx \
        --nvtx-include "prof_step/" --csv --log-file launches.csv \
        python -m grappa_b200.utils.profile_step --workload sage

and a full section set is taken for ONE kernel, a few launches, on the reduced
graph ``ogbpr_small`` (1M nodes, 50M directed edges, about 0.6 GB resident):

    ncu --set full --clock-control none --nvtx --nvtx-include "prof_step/" \
        -k regex:aggregate_kernel -c 1 -o prof_aggregate \
        python -m grappa_b200.utils.profile_step --workload sage --config ogbpr_small

With ``--phases N`` the CUDA-event device time of each step phase (sample,
forward, backward, update) averaged over N eager steps is printed; with
``--graphs N`` the device time of N replays of each captured graph: sampling
alone, the step without and with the next step's sampling on its side stream (the
overlap that the training loop uses); with ``--kernel-times N`` the CUDA-event time of
every kernel binding call, averaged over N eager steps; with ``--trace N`` each
kernel's device time inside N replays of the step graph (CUPTI activity records,
for the ranking only: a profiled number is not a benchmark value).  Workloads: 3-layer models on the
ogbn-products-shaped synthetic graph (``--config`` picks another spec), 1024 seeds
per batch, one GPU.
"""
import argparse
import json

import torch

from grappa_b200.dataset import synthetic as S
from grappa_b200.graph_store import partition_from_global
from grappa_b200.models import get_model
from grappa_b200.trainer import MiniBatchTrainer

WORKLOADS = {"sage": ("sage", 256, [15, 10, 5]), "gcn": ("gcn", 256, [15, 10, 5]), "gin": ("gin", 256, [15, 10, 5]),
             "gat": ("gat", 64, [10, 10, 10]), "pinsage": ("pinsage", 256, [5, 5, 5])}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="sage", choices=sorted(WORKLOADS))
    ap.add_argument("--config", default="ogbpr")
    ap.add_argument("--batch", type=int, default=1024)
    ap.add_argument("--phases", type=int, default=0, help="time the phases of this many eager steps")
    ap.add_argument("--graphs", type=int, default=0, help="time this many replays of each step graph")
    ap.add_argument("--kernel-times", type=int, default=0,
                    help="CUDA-event time of every kernel binding call over this many eager steps")
    ap.add_argument("--trace", type=int, default=0,
                    help="per-kernel device time inside this many replays of the step graph (CUPTI activity "
                         "records through torch.profiler; warm caches, kernels as they overlap in the step)")
    a = ap.parse_args()
    name, hidden, fanouts = WORKLOADS[a.workload]
    dev = torch.device("cuda", 0)
    spec = S.SPECS[a.config]
    if spec.n_nodes >= S.LEAN_MIN_NODES:
        own = S.build_partition(spec, 1, 0, dev)  # graphs of 100M+ nodes: built without the global copy
    else:
        g = S.build(spec, dev)
        own = partition_from_global(g, 1, 0, dev, part_seed=spec.seed)
        del g
    torch.cuda.empty_cache()
    torch.manual_seed(0)
    model = get_model(name, spec.feat_dim, spec.n_classes, num_hidden=hidden, num_layers=3, dropout=0.5, n_heads=4)
    tr = MiniBatchTrainer(model, own, fanouts, a.batch, comm=None, seed=3, use_cuda_graph=False)
    eng = tr.engine
    seeds, counts = tr.epoch_seeds(0, on_host=False)
    eng.set_epoch(0)
    eng.step(seeds[0], counts[0])
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("prof_step")
    eng.step(seeds[1], counts[1])
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    eng.check_errors()
    out = {"workload": a.workload, "launches_per_step": eng.launches_per_step, "block_counts": eng.sm.cnt.tolist()}
    if a.phases:
        out["phase_ms"] = eng.time_phases(seeds, counts, a.phases)
    if a.kernel_times:
        out["kernel_us"] = kernel_times(eng, seeds, counts, a.kernel_times)
    tr.close()
    if a.graphs:
        out["graph_ms"] = time_graphs(model, own, fanouts, a.batch, a.graphs)
    if a.trace:
        out["trace"] = trace_graph(model, own, fanouts, a.batch, a.trace)
    print(json.dumps(out))


def kernel_times(eng, seeds, counts, n):
    """Mean device time (us per step) of each kernel binding call of an eager step, keyed
    by its order in the step ("12:gat_bwd"), from CUDA events on the stream that issued
    it.  Calls on the side streams overlap others, so the times do not add up to the
    step; the ranking shows where a step's device time goes."""
    eng.cu.timer = []
    per = {}
    for s in range(n):
        eng.cu.timer.clear()
        eng.step(seeds[(s + 2) % seeds.shape[0]], counts[(s + 2) % counts.shape[0]])
        torch.cuda.synchronize()
        for i, (name, e0, e1) in enumerate(eng.cu.timer):
            key = f"{i:02d}:{name}"
            per[key] = per.get(key, 0.0) + e0.elapsed_time(e1) * 1000.0 / n
    eng.cu.timer = None
    return {k: round(v, 1) for k, v in sorted(per.items(), key=lambda kv: -kv[1])}


def trace_graph(model, own, fanouts, batch, n):
    """Replays of the step graph with the next step's sampling beside it (the training
    loop's unit) under torch.profiler: every kernel's mean device time per replay, the
    busy span of each replay and the sum of kernel times."""
    from torch.profiler import ProfilerActivity, profile

    tr = MiniBatchTrainer(model, own, fanouts, batch, comm=None, seed=3, use_cuda_graph=True)
    tr.warmup()
    eng = tr.engine
    seeds, counts = tr.epoch_seeds(0, on_host=False)
    eng.set_epoch(0)
    eng._load_into(0, seeds[0], counts[0])
    eng._load_into(1, seeds[1], counts[1])
    g = eng._graph_for(("step", 0, True))
    for _ in range(5):
        g.replay()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(n):
            g.replay()
        torch.cuda.synchronize()
    eng.check_errors()
    tr.close()
    per, spans = {}, []
    evs = [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    for e in evs:
        name = e.name[:80]
        t = per.setdefault(name, [0.0, 0])
        t[0] += e.time_range.end - e.time_range.start
        t[1] += 1
    total = sum(v[0] for v in per.values()) / n
    if evs:
        t0 = min(e.time_range.start for e in evs)
        t1 = max(e.time_range.end for e in evs)
        spans = (t1 - t0) / n
    rows = sorted(((v[0] / n, v[1] / n, k) for k, v in per.items()), reverse=True)
    return {"replays": n, "span_us_per_replay": round(spans, 1) if spans else None,
            "kernel_us_sum_per_replay": round(total, 1),
            "kernels": [{"name": k, "us_per_replay": round(v, 2), "launches_per_replay": round(c, 2)}
                        for v, c, k in rows]}


def time_graphs(model, own, fanouts, batch, n):
    tr = MiniBatchTrainer(model, own, fanouts, batch, comm=None, seed=3, use_cuda_graph=True)
    tr.warmup()
    eng = tr.engine
    seeds, counts = tr.epoch_seeds(0, on_host=False)
    eng.set_epoch(0)
    eng._load_into(0, seeds[0], counts[0])
    eng._load_into(1, seeds[1], counts[1])
    res = {}
    for name, key in (("sample", ("sample", 0)), ("step_compute_only", ("step", 0, False)),
                      ("step_with_next_sampling", ("step", 0, True))):
        g = eng._graph_for(key)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(n):
            g.replay()
        a1.record()
        torch.cuda.synchronize()
        res[name] = a0.elapsed_time(a1) / n
    eng.check_errors()
    tr.close()
    return res


if __name__ == "__main__":
    main()
