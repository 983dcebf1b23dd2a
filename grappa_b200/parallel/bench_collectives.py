"""Collective microbenchmarks at 2/4/8 GPUs, each against the NCCL path it replaces.

(a) coverage-corrected gradient all-reduce fused with Adam, fp32 gradient buffers
    from 1 KB to 1 GB, per-rank coverage weights uniform in [0.5, 1]:
      fused    one kernel over NVLink peer memory (one-shot / two-shot by size)
      nccl     scale by c_r / W, NCCL all_reduce, then the same Adam kernel
(b) repartition all-to-all of 128-dim bf16 feature rows plus int64 CSR chunks with
    uniformly random destination partitions, 1M-100M edges per GPU:
      pull     one kernel pulling every peer's segment over NVLink (a2a_pull)
      nccl     all_to_all_single of the same bytes

Times are CUDA-event device times of the collective alone, after warm-up, the max
over ranks.  The roofline time is the slower of the bytes that must cross NVLink
per GPU and direction at the measured 770 GB/s peer bandwidth (2 (W-1)/W * S for
an all-reduce of S bytes, the remote part of the sent bytes for the all-to-all)
and, for the all-reduce fused with Adam, the local HBM bytes of the update at the
measured 6.56 TB/s.

    python -m torch.distributed.run --nproc-per-node W --master-addr 127.0.0.1 \\
        -m grappa_b200.parallel.bench_collectives [--part a|b|ab] [--max-bytes N]
Prints one JSON line per measurement (rank 0).
"""
import argparse
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0  # measured peer copy bandwidth per direction per GPU
HBM_GBS = 6555.8  # measured HBM copy bandwidth of this GPU type


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


def bench_allreduce(comm, dev, sizes, iters_for):
    from grappa_b200 import _native
    from grappa_b200.engine import FusedAllReduceAdam
    from grappa_b200.sampler_gpu import new_counters

    cu = _native.cuda()
    W, r = comm.world, comm.rank
    out = []
    for nbytes in sizes:
        n = max(4, nbytes // 4)
        iters = iters_for(nbytes)
        g = torch.Generator(device="cpu").manual_seed(1000 + r)
        c = 0.5 + 0.5 * torch.rand(1, generator=g).item()
        cov = torch.tensor([c * 4.0, 4.0], device=dev)
        grad = torch.randn(n, device=dev)
        param = torch.zeros(n, device=dev)
        m, v = torch.zeros_like(param), torch.zeros_like(param)
        wbf = torch.zeros(n, dtype=torch.bfloat16, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        counters = new_counters(0, dev)
        row = {"bench": "allreduce_adam", "world": W, "bytes": n * 4}
        variants = [("fused", None)]
        if W > 2:
            variants = [("fused_one_shot", False), ("fused_two_shot", True)]
        for name, two in variants:
            ar = FusedAllReduceAdam(comm, n, two_shot=two)

            def run_fused():
                ar.step(grad, cov, counters, param, m, v, wbf, 1e-3, 0.9, 0.999, 1e-8, err, cu=cu)
                cu.step_end(counters)

            row[name + "_ms"] = _time(run_fused, iters, 3, dev)
            torch.cuda.synchronize(dev)
            assert int(err.item()) == 0, f"fused all-reduce reported error word {int(err.item())}"
            ar.close()
        scale = torch.tensor([c / W], device=dev)

        def run_nccl():
            grad.mul_(scale)
            dist.all_reduce(grad)
            cu.adam(param, m, v, grad, wbf, 1e-3, 0.9, 0.999, 1e-8, 0.0, counters, 1.0, None, True)
            cu.step_end(counters)

        row["nccl_ms"] = _time(run_nccl, iters, 3, dev)
        link_ms = 2.0 * (W - 1) / W * n * 4 / (LINK_GBS * 1e9) * 1e3
        # local HBM bytes per element: publish (grad read + clear, send write) 12, the
        # peers' reads of this rank's copy 4 (W-1), Adam (param, m, v read and write,
        # bf16 copy) 26, the reduced value 4
        hbm_ms = (42.0 + 4.0 * (W - 1)) * n / (HBM_GBS * 1e9) * 1e3
        roof_ms = max(link_ms, hbm_ms)
        row["roofline_link_ms"] = link_ms
        row["roofline_hbm_ms"] = hbm_ms
        row["roofline_ms"] = roof_ms
        best = min(v for k, v in row.items() if k.startswith("fused") and k.endswith("_ms"))
        row["fused_best_ms"] = best
        row["fused_frac_of_roofline"] = roof_ms / best if best > 0 else None
        row["nccl_frac_of_roofline"] = roof_ms / row["nccl_ms"] if row["nccl_ms"] > 0 else None
        row["fused_busbw_gbs"] = 2.0 * (W - 1) / W * n * 4 / (best * 1e-3) / 1e9
        out.append(row)
        del grad, param, m, v, wbf
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
        rows += bench_allreduce(comm, dev, sizes, lambda b: 50 if b <= (1 << 24) else 10)
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
