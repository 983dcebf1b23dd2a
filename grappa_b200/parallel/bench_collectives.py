"""Collective microbenchmarks at 2/4/8 GPUs, each against the NCCL path it replaces.

(a) coverage-corrected gradient all-reduce fused with Adam, fp32 and bf16 gradient
    buffers from 1 KB to 1 GB, per-rank coverage weights uniform in [0.5, 1]:
      one_shot  one kernel: publish a scaled copy, read all W copies, Adam on everything
      shard     one kernel: reduce-scatter from the peers' gradient buffers, Adam on the
                owned shard, all-gather of the updated fp32 master weights
      nccl      scale by c_r / W, NCCL all_reduce (then a cast of bf16 gradients), then
                the same Adam kernel
    Every variant is captured ``iters`` times into one CUDA graph, so the device time
    per call excludes the host's launch cost (the training step replays graphs too).
(b) repartition all-to-all of 128-dim bf16 feature rows plus int64 CSR chunks with
    uniformly random destination partitions, 1M-100M edges per GPU:
      pull     one kernel pulling every peer's segment over NVLink (a2a_pull)
      nccl     all_to_all_single of the same bytes

Times are CUDA-event device times, after warm-up, the max over ranks.  The NVLink
roofline of (a) is the bytes that must cross NVLink per GPU and direction at the
measured 770 GB/s peer bandwidth (nominal 900 GB/s): 2 (W-1)/W * S for an all-reduce
of S gradient bytes (``roofline_ar_ms``); the shard kernel moves (W-1)/W of the
gradient plus (W-1)/W of the fp32 parameters, which is the same for fp32 gradients
and 1.5x it for bf16 gradients (``roofline_shard_ms``).  The HBM side, at the measured
copy bandwidth, is the Adam pass over 1/W of the elements plus the shard kernel's
local traffic; the reported roofline is the slower of the two.

    python -m torch.distributed.run --nproc-per-node W --master-addr 127.0.0.1 \\
        -m grappa_b200.parallel.bench_collectives [--part a|b|ab] [--max-bytes N]
Prints one JSON line per measurement (rank 0).
"""
import argparse
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0  # measured peer copy bandwidth per direction per GPU (nominal 900)
HBM_GBS = 6536.4  # measured HBM copy bandwidth of this GPU type


def _max_over_ranks(x, dev):
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _time(fn, iters, warmup, dev):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize(dev)
    return _max_over_ranks(a.elapsed_time(b) / iters, dev)


def _time_graph(fn, iters, dev):
    """Device time per call of ``fn`` captured ``iters`` times into one CUDA graph (two
    warm-up calls first, one warm-up replay), max over ranks."""
    fn()
    fn()
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for _ in range(iters):
                fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    g.replay()
    torch.cuda.synchronize(dev)
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize(dev)
    t = _max_over_ranks(a.elapsed_time(b) / iters, dev)
    del g
    return t


def bench_allreduce(comm, dev, sizes, iters_for, dtypes=("float32", "bfloat16")):
    from grappa_b200 import _native
    from grappa_b200.parallel.allreduce import ONE_SHOT, SHARD, FusedAllReduceAdam
    from grappa_b200.sampler_gpu import new_counters

    cu = _native.cuda()
    W, r = comm.world, comm.rank
    out = []
    for dname in dtypes:
        dtype = getattr(torch, dname)
        esz = 4 if dtype == torch.float32 else 2
        for nbytes in sizes:
            n = max(8, nbytes // esz // 8 * 8)
            iters = iters_for(n * esz)
            g = torch.Generator(device="cpu").manual_seed(1000 + r)
            c = 0.5 + 0.5 * torch.rand(1, generator=g).item()
            cov = torch.tensor([c * 4.0, 4.0], device=dev)
            m, v = torch.zeros(n, device=dev), torch.zeros(n, device=dev)
            wbf = torch.zeros(n, dtype=torch.bfloat16, device=dev)
            err = torch.zeros(1, dtype=torch.int32, device=dev)
            counters = new_counters(0, dev)
            row = {"bench": "allreduce_adam", "world": W, "grad_dtype": dname, "bytes": n * esz}
            variants = [("one_shot", ONE_SHOT), ("shard", SHARD)]
            if n * esz > (256 << 20) and W > 2:
                variants = [("shard", SHARD)]  # one-shot reads W-1 full copies: far off at this size
            for name, mode in variants:
                ar = FusedAllReduceAdam(comm, n, grad_dtype=dtype, modes=[mode])
                ar.grad.normal_()
                ar.bind(counters, m, v, wbf, 1e-3, err=err, cov=cov)

                def run_fused():
                    ar.launch(0)
                    cu.step_end(counters)

                row[name + "_ms"] = _time_graph(run_fused, iters, dev)
                torch.cuda.synchronize(dev)
                assert int(err.item()) == 0, f"fused all-reduce reported error word {int(err.item())}"
                row[name + "_grid"] = ar.grids[0]
                ar.close()
            grad = torch.randn(n, device=dev).to(dtype)
            g32 = torch.zeros(n, device=dev)
            param = torch.zeros(n, device=dev)
            scale = torch.tensor([c / W], device=dev).to(dtype)

            def run_nccl():
                grad.mul_(scale)
                dist.all_reduce(grad)
                if dtype == torch.float32:
                    cu.adam(param, m, v, grad, wbf, 1e-3, 0.9, 0.999, 1e-8, 0.0, counters, 1.0, None, True)
                else:
                    g32.copy_(grad)
                    cu.adam(param, m, v, g32, wbf, 1e-3, 0.9, 0.999, 1e-8, 0.0, counters, 1.0, None, True)
                cu.step_end(counters)

            row["nccl_ms"] = _time_graph(run_nccl, iters, dev)
            S = n * esz
            link_ar = 2.0 * (W - 1) / W * S / (LINK_GBS * 1e9) * 1e3
            link_shard = (W - 1) / W * (S + 4 * n) / (LINK_GBS * 1e9) * 1e3
            # shard kernel's local HBM bytes per element: gradient served to the owners and
            # cleared (2 esz), Adam on 1/W (26 B), all-gather writes of fp32 + bf16 (6 (W-1)/W)
            # and the owned shard served to the peers (4 (W-1)/W)
            hbm_ms = (2 * esz + 26.0 / W + 10.0 * (W - 1) / W) * n / (HBM_GBS * 1e9) * 1e3
            row["roofline_ar_ms"] = link_ar
            row["roofline_shard_ms"] = link_shard
            row["roofline_hbm_ms"] = hbm_ms
            roof = max(link_shard, hbm_ms)
            row["roofline_ms"] = roof
            best = min(v_ for k_, v_ in row.items() if k_ in ("one_shot_ms", "shard_ms"))
            row["fused_best_ms"] = best
            row["fused_frac_of_roofline"] = roof / best if best > 0 else None
            row["fused_frac_of_ar_link_roofline"] = max(link_ar, hbm_ms) / best if best > 0 else None
            row["nccl_frac_of_ar_link_roofline"] = max(link_ar, hbm_ms) / row["nccl_ms"] if row["nccl_ms"] > 0 else None
            row["fused_busbw_gbs"] = 2.0 * (W - 1) / W * S / (best * 1e-3) / 1e9
            out.append(row)
            if r == 0:
                print(json.dumps(row), flush=True)
            del grad, param, m, v, wbf, g32
            torch.cuda.empty_cache()
    return out


def _split_sizes(total_rows, W, seed, row_bytes, edge_bytes_per_row):
    """Bytes sent to every destination when each row (with its edges) picks a uniform
    random destination partition; multiples of 16 bytes."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    dest = torch.randint(0, W, (total_rows,), generator=g)
    rows = torch.bincount(dest, minlength=W)
    return [int((int(c) * (row_bytes + edge_bytes_per_row) + 15) // 16 * 16) for c in rows]


def bench_alltoall(comm, dev, edge_counts, iters):
    from grappa_b200 import _native
    from grappa_b200.parallel.comm import PeerBuffer

    cu = _native.cuda()
    W, r = comm.world, comm.rank
    out = []
    avg_deg = 16
    row_bytes = 128 * 2 + 8           # bf16 feature row + int64 row pointer
    edge_bytes = avg_deg * 8          # int64 CSR indices of the row
    for E in edge_counts:
        rows = E // avg_deg
        send_sizes = _split_sizes(rows, W, 77 + r, row_bytes, edge_bytes)
        table = comm.all_gather_object(send_sizes)          # table[p][q]: bytes p sends to q
        send_total = sum(send_sizes)
        recv_sizes = [table[p][r] for p in range(W)]
        recv_total = sum(recv_sizes)
        sbuf = PeerBuffer(comm, send_total + 256)
        send = sbuf.tensor(torch.uint8, [send_total])
        send.copy_(torch.randint(0, 255, (send_total,), dtype=torch.uint8, device=dev))
        recv = torch.empty(recv_total + 16, dtype=torch.uint8, device=dev)
        flags = PeerBuffer(comm, 256)
        epoch = torch.zeros(1, dtype=torch.int64, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        src_off = [sum(table[p][:r]) for p in range(W)]
        dst_off = [sum(recv_sizes[:p]) for p in range(W)]
        fl = [flags.ptrs[p] for p in range(W)]
        torch.cuda.synchronize(dev)
        comm.barrier()

        def run_pull():
            cu.peer_barrier(r, W, flags.local, fl, epoch, int(10e9), err)
            cu.a2a_pull(list(sbuf.ptrs), src_off, recv_sizes, dst_off, recv.data_ptr(), (r + 1) % W)
            cu.peer_barrier(r, W, flags.local, fl, epoch, int(10e9), err)

        row = {"bench": "repartition_alltoall", "world": W, "edges_per_gpu": E, "bytes_sent_per_gpu": send_total}
        row["pull_ms"] = _time(run_pull, iters, 2, dev)
        assert int(err.item()) == 0, "peer barrier timed out"
        nin = torch.empty(recv_total, dtype=torch.uint8, device=dev)

        def run_nccl():
            dist.all_to_all_single(nin, send, output_split_sizes=recv_sizes, input_split_sizes=send_sizes)

        row["nccl_ms"] = _time(run_nccl, iters, 2, dev)
        same = torch.equal(nin, recv[:recv_total])
        row["pull_matches_nccl"] = bool(_max_over_ranks(0.0 if same else 1.0, dev) == 0.0)
        remote = send_total - send_sizes[r]
        cross = _max_over_ranks(float(max(remote, recv_total - recv_sizes[r])), dev)
        row["roofline_ms"] = cross / (LINK_GBS * 1e9) * 1e3
        row["pull_frac_of_roofline"] = row["roofline_ms"] / row["pull_ms"]
        row["nccl_frac_of_roofline"] = row["roofline_ms"] / row["nccl_ms"]
        out.append(row)
        sbuf.close()
        flags.close()
        del send, recv, nin
        torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--part", default="ab")
    ap.add_argument("--max-bytes", type=int, default=1 << 30)
    ap.add_argument("--max-edges", type=int, default=100_000_000)
    ap.add_argument("--dtypes", default="float32,bfloat16", help="gradient dtypes of part (a)")
    args = ap.parse_args()
    from grappa_b200.parallel.comm import Comm, init_distributed

    rank, world = init_distributed("nccl")
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = Comm()
    rows = []
    if "a" in args.part:
        sizes = [1 << k for k in range(10, 31, 2) if (1 << k) <= args.max_bytes]
        bench_allreduce(comm, dev, sizes, lambda b: 200 if b <= (1 << 20) else (50 if b <= (1 << 24) else 10),
                        dtypes=args.dtypes.split(","))
    if "b" in args.part:
        edges = [e for e in (1_000_000, 10_000_000, 100_000_000) if e <= args.max_edges]
        rows += bench_alltoall(comm, dev, edges, 10)
    if rank == 0:
        for r in rows:
            print(json.dumps(r), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
