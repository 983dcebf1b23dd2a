"""Kernel microbenchmarks on one GPU: the tcgen05 GEMM against torch.matmul (cuBLAS)
on the training shapes, the aggregation kernel against the HBM roofline, and the
fused all-reduce + Adam kernel on one rank (its local HBM side).  CUDA-event device
times after warm-up, inputs sized as in a training step of the ogbn-products-shaped
workload (``--scale`` multiplies the row counts).

    python -m grappa_b200.utils.bench_kernels [--scale 1] [--part gemm,aggregate,ar]
Prints one JSON line per measurement.
"""
import argparse
import json
import math

import torch

from grappa_b200 import _native

# measured on this GPU type: STREAM-style copy, cuBLAS bf16 GEMM as a burst and
# sustained for seconds under the power cap (the figure for kernels inside a long step)
HBM_GBS = 6536.4
BF16_TFLOPS = 1615.2
BF16_TFLOPS_SUSTAINED = 1375.2


def _time(fn, iters=50, warmup=5):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def gemm_case(M, K, N, bn=None, p=0.0):
    from grappa_b200.engine import gemm_bn

    cu = _native.cuda()
    dev = torch.device("cuda", 0)
    A = torch.randn(M, K, device=dev).to(torch.bfloat16)
    B = (torch.randn(N, K, device=dev) / math.sqrt(K)).to(torch.bfloat16)
    bias = torch.zeros(N, device=dev)
    C = torch.zeros(M, N, device=dev, dtype=torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    counters = torch.zeros(6, dtype=torch.int64, device=dev)
    bn = bn or gemm_bn(M, N)

    def ours():
        cu.gemm(A, False, B, False, M, None, N, K, None, 1, C, 0, bias, 1, p, counters if p > 0 else None, 0, None,
                0, None, None, None, None, None, None, err, bn)

    def torch_ref():
        torch.relu(torch.addmm(bias.to(torch.bfloat16), A, B.t()))

    t_ours, t_ref = _time(ours), _time(torch_ref)
    flops = 2.0 * M * N * K
    bytes_ = 2.0 * (M * K + N * K + M * N)
    assert int(err.item()) == 0
    return {"bench": "gemm", "M": M, "K": K, "N": N, "bn": bn, "dropout": p, "ours_ms": t_ours, "torch_ms": t_ref,
            "ours_tflops": flops / t_ours / 1e9, "ours_frac_of_hbm": bytes_ / (t_ours * 1e-3) / 1e9 / HBM_GBS,
            "ours_frac_of_bf16_peak": flops / (t_ours * 1e-3) / 1e12 / BF16_TFLOPS}


def dw_case(live, cap, M, N):
    """Split-K weight gradient gW[M, N] += dY^T X over the live rows of capacity-sized
    operands (dY [cap, M], X [cap, N], both MN-major), as in the training step."""
    from grappa_b200.engine import split_k

    cu = _native.cuda()
    dev = torch.device("cuda", 0)
    dY = torch.zeros(cap, M, device=dev, dtype=torch.bfloat16)
    X = torch.zeros(cap, N, device=dev, dtype=torch.bfloat16)
    dY[:live] = torch.randn(live, M, device=dev).to(torch.bfloat16)
    X[:live] = torch.randn(live, N, device=dev).to(torch.bfloat16)
    gW = torch.zeros(M, N, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    kdev = torch.tensor([live], dtype=torch.int32, device=dev)
    n_tiles = math.ceil(M / 128) * math.ceil(N / 256)
    splits = split_k(cap, n_tiles)

    def ours():
        cu.gemm(dY, True, X, True, M, None, N, cap, kdev, splits, gW, 2, None, 0, 0.0, None, 0, None, 0, None, None,
                None, None, None, None, err, 256)

    def torch_ref():
        gW.add_(dY[:live].t() @ X[:live])

    t_ours, t_ref = _time(ours), _time(torch_ref)
    assert int(err.item()) == 0
    return {"bench": "gemm_dw_split_k", "live_rows": live, "cap_rows": cap, "M": M, "N": N, "splits_host": splits,
            "ours_ms": t_ours, "torch_ms": t_ref}


def aggregate_case(n_dst, n_src, deg, dim):
    cu = _native.cuda()
    dev = torch.device("cuda", 0)
    indptr = torch.arange(0, (n_dst + 1) * deg, deg, dtype=torch.int32, device=dev)
    indices = torch.randint(0, n_src, (n_dst * deg,), dtype=torch.int32, device=dev)
    src = torch.randn(n_src, dim, device=dev).to(torch.bfloat16)
    out = torch.zeros(n_dst, 2 * dim, device=dev, dtype=torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    def run():
        cu.aggregate(indptr, indices, None, n_dst, n_dst, src, None, dim, 0, None, None, None, out, dim, 0, 0.0, 0, err)

    t = _time(run)
    bytes_ = 2.0 * (n_dst * deg * dim + n_dst * dim + n_dst * 2 * dim) + 4.0 * n_dst * deg
    return {"bench": "aggregate_mean", "n_dst": n_dst, "n_src": n_src, "deg": deg, "dim": dim, "ms": t,
            "frac_of_hbm": bytes_ / (t * 1e-3) / 1e9 / HBM_GBS}


def ar_case(nbytes, mode, dtype=torch.float32):
    """The fused all-reduce + Adam kernel on one rank (W = 1): the local HBM traffic of
    a bucket (gradient read and clear, Adam on fp32 master weights, moments and the bf16
    copy), without peers.  ``mode`` 0 = one-shot, 1 = shard."""
    from grappa_b200.parallel.allreduce import FusedAllReduceAdam
    from grappa_b200.parallel.comm import Comm
    from grappa_b200.sampler_gpu import new_counters

    dev = torch.device("cuda", 0)
    esz = 4 if dtype == torch.float32 else 2
    n = max(8, nbytes // esz // 8 * 8)
    ar = FusedAllReduceAdam(Comm(), n, grad_dtype=dtype, modes=[mode])
    m, v = torch.zeros(n, device=dev), torch.zeros(n, device=dev)
    wbf = torch.zeros(n, dtype=torch.bfloat16, device=dev)
    counters = new_counters(0, dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ar.bind(counters, m, v, wbf, 1e-3, err=err)
    cu = _native.cuda()

    def run():
        ar.launch(0)
        cu.step_end(counters)

    t = _time(run, iters=20, warmup=3)
    assert int(err.item()) == 0
    # gradient read + clear, param/m/v read + write, bf16 write (+ the slot copy of one-shot)
    bytes_ = n * (2 * esz + 24 + 2 + (8 if mode == 0 else 0))
    ar.close()
    return {"bench": "allreduce_adam_1rank", "mode": mode, "grad_dtype": str(dtype).split(".")[-1], "bytes": n * esz,
            "ms": t, "frac_of_hbm": bytes_ / (t * 1e-3) / 1e9 / HBM_GBS}


def _time_graph(fn, reps=20, iters=20):
    """Device time of one fn() from a CUDA graph holding reps calls (launch overhead
    excluded, as inside the training step graph)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / (iters * reps)


def head_case(n_dst=1021, n_src=3250, deg=5, ip=256, C=47):
    """GraphSAGE output layer of a 1024-seed step: the fused head kernel against the
    aggregation + cross-entropy GEMM + dX GEMM it replaces (both inside CUDA graphs)."""
    from grappa_b200.engine import bn_for

    cu = _native.cuda()
    dev = torch.device("cuda", 0)
    cap = 1024
    op = (C + 7) // 8 * 8
    indptr = torch.arange(0, (n_dst + 1) * deg, deg, dtype=torch.int32, device=dev)
    indices = torch.randint(0, n_src, (n_dst * deg,), dtype=torch.int32, device=dev)
    h = torch.randn(n_src, ip, device=dev).to(torch.bfloat16)
    w = torch.zeros(op, 2 * ip, device=dev, dtype=torch.bfloat16)
    w[:C] = (torch.randn(C, 2 * ip, device=dev) / math.sqrt(2 * ip)).to(torch.bfloat16)
    bias = torch.zeros(op, device=dev)
    labels = torch.randint(0, C, (cap,), dtype=torch.int32, device=dev)
    x = torch.zeros(cap, 2 * ip, device=dev, dtype=torch.bfloat16)
    dl = torch.zeros(cap, op, device=dev, dtype=torch.bfloat16)
    dx = torch.zeros(cap, 2 * ip, device=dev, dtype=torch.bfloat16)
    loss, correct = torch.zeros(1, device=dev), torch.zeros(1, dtype=torch.int32, device=dev)
    db = torch.zeros(op, device=dev)
    nd = torch.tensor([n_dst], dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    dummy = torch.zeros((1, 1), device=dev)

    def fused():
        cu.sage_head(indptr, indices, nd, cap, h, ip, w, bias, C, labels, x, dl, dx, loss, correct, db)

    def unfused():
        cu.aggregate(indptr, indices, nd, 0, cap, h, None, ip, 0, None, None, None, x, ip, 0, 0.0, 0, err)
        cu.gemm(x, False, w, False, cap, nd, op, 2 * ip, None, 1, dummy, 3, bias, 0, 0.0, None, 0, labels, C, dl, loss,
                correct, None, nd, db, err, bn_for(op))
        cu.gemm(dl, False, w, True, cap, nd, 2 * ip, op, None, 1, dx, 0, None, 0, 0.0, None, 0, None, 0, None, None,
                None, None, None, None, err, 256)

    t_f, t_u = _time_graph(fused), _time_graph(unfused)
    assert int(err.item()) == 0
    return {"bench": "sage_head", "n_dst": n_dst, "ip": ip, "classes": C, "fused_us": t_f * 1e3,
            "aggregate_ce_gemm_dx_gemm_us": t_u * 1e3}


def repart_case(n_part=600_000, deg=50, n_global=2_449_029, halo=400_000, dim=104):
    """The repartition kernels on local memory (the peer pointers replaced by this GPU's
    own buffers, so the numbers are HBM-side; over NVLink the same kernels read the
    neighbour's memory): CSR merge of two partitions of n_part nodes and deg in-edges each
    through the global-id map, halo compaction over n_global marks, a pull of `halo`
    feature rows by global id and the bulk copy of a partition's rows.  CUDA-event
    device times; achieved bytes against the measured HBM copy bandwidth."""
    cu = _native.cuda()
    dev = torch.device("cuda", 0)
    i32, i64 = dict(dtype=torch.int32, device=dev), dict(dtype=torch.int64, device=dev)
    E = n_part * deg
    ip = torch.arange(0, (n_part + 1) * deg, deg, **i64)
    ia = torch.randint(0, n_global, (E,), **i32)
    ib = torch.randint(0, n_global, (E,), **i32)
    mp = torch.randint(0, 2 * n_part + halo, (n_global,), **i32)
    mp[: 2 * n_part] = torch.arange(2 * n_part, **i32)  # own and neighbour ranges (translated arithmetically)
    out_ip = torch.zeros(2 * n_part + 1, **i64)
    out_ix = torch.zeros(2 * E, **i32)
    err = torch.zeros(1, **i32)

    def merge():
        cu.csr_merge(ip.data_ptr(), ia.data_ptr(), n_part, ip.data_ptr(), ib.data_ptr(), n_part, mp, out_ip, out_ix,
                     err, g0_a=0, g0_b=n_part)

    t_merge = _time(merge, iters=20)
    merge_bytes = 2 * E * 4 * 2 + 2 * E * 4 + 2 * (n_part + 1) * 8 * 2  # indices r/w, map gathers, indptr
    mark = torch.zeros(n_global, dtype=torch.uint8, device=dev)
    ids = torch.randint(0, n_global, (halo * 2,), **i32)
    out_ids = torch.zeros(n_global, **i64)
    n_out = torch.zeros(1, **i32)
    scr = torch.zeros(cu.mark_compact_scratch_words(n_global), **i64)

    def marks():
        cu.mark_ids(ids.data_ptr(), None, ids.numel(), mark)
        cu.mark_compact(mark, out_ids, mp, 0, n_out, scr, err)

    t_marks = _time(marks, iters=20)
    marks_bytes = ids.numel() * (4 + 32) + n_global + int(n_out.item()) * 12
    table = torch.randn(n_global, dim, device=dev).to(torch.bfloat16)
    gids = torch.randint(0, n_global, (halo,), **i64)
    prefix = torch.tensor([0, n_global], **i64)
    out = torch.zeros(halo, dim, device=dev, dtype=torch.bfloat16)

    def pull():
        cu.pull_rows([table.data_ptr()], dim, 2, dim * 2, gids, None, halo, prefix, out.data_ptr(), dim, 0, halo, err)

    t_pull = _time(pull, iters=20)
    pull_bytes = halo * (dim * 2 * 2 + 8)
    rows = table[:n_part]
    dst = torch.empty_like(rows)

    def copy():
        cu.peer_copy(dst.data_ptr(), rows.data_ptr(), rows.numel() * 2)

    t_copy = _time(copy, iters=20)
    copy_bytes = rows.numel() * 2 * 2
    assert int(err.item()) == 0
    res = []
    for name, t, b in (("csr_merge", t_merge, merge_bytes), ("mark_ids+mark_compact", t_marks, marks_bytes),
                       ("pull_rows", t_pull, pull_bytes), ("bulk_copy", t_copy, copy_bytes)):
        res.append({"bench": "repartition_kernel", "kernel": name, "ms": t, "bytes": int(b),
                    "frac_of_hbm": b / (t * 1e-3) / 1e9 / HBM_GBS})
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--scale", type=float, default=1.0)
    ap.add_argument("--part", default="gemm,aggregate", help="comma list of gemm, aggregate, head, repart, ar")
    ap.add_argument("--ar-bytes", type=int, default=256 << 20)
    a = ap.parse_args()
    s = a.scale
    parts = a.part.split(",")
    rows = []
    if "gemm" in parts:
        rows += [gemm_case(int(20853 * s), 208, 256), gemm_case(int(20853 * s), 208, 256, p=0.5),
                 gemm_case(int(3250 * s), 512, 256), gemm_case(int(139058 * s), 104, 256),
                 gemm_case(65536, 256, 256), gemm_case(131072, 1024, 1024)]
        rows += [dw_case(int(20853 * s), int(180224 * s), 256, 208), dw_case(int(3250 * s), int(16384 * s), 256, 512),
                 dw_case(int(1021 * s), int(1024 * s), 48, 512)]
    if "aggregate" in parts:
        rows += [aggregate_case(int(20853 * s), int(133975 * s), 14, 104),
                 aggregate_case(int(3250 * s), int(20853 * s), 8, 256)]
    if "head" in parts:
        rows += [head_case()]
    if "repart" in parts:
        rows += repart_case()
    if "ar" in parts:
        rows += [ar_case(a.ar_bytes, 1), ar_case(a.ar_bytes, 0), ar_case(a.ar_bytes, 1, torch.bfloat16)]
    for r in rows:
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
