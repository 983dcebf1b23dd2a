"""Kernel microbenchmarks on one GPU: the tcgen05 GEMM against torch.matmul (cuBLAS)
on the training shapes, and the aggregation / sampling kernels against the HBM
roofline.  CUDA-event device times after warm-up, inputs sized as in a training
step of the ogbn-products-shaped workload (``--scale`` multiplies the row counts).

    python -m grappa_b200.utils.bench_kernels [--scale 1]
Prints one JSON line per measurement.
"""
import argparse
import json
import math

import torch

from grappa_b200 import _native

HBM_GBS = 6555.8
BF16_TFLOPS = 1655.8


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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--scale", type=float, default=1.0)
    a = ap.parse_args()
    s = a.scale
    rows = [gemm_case(int(20853 * s), 208, 256), gemm_case(int(20853 * s), 208, 256, p=0.5),
            gemm_case(int(3250 * s), 512, 256), gemm_case(int(139058 * s), 104, 256),
            gemm_case(65536, 256, 256), gemm_case(131072, 1024, 1024)]
    rows += [dw_case(int(20853 * s), int(180224 * s), 256, 208), dw_case(int(3250 * s), int(16384 * s), 256, 512),
             dw_case(int(1021 * s), int(1024 * s), 48, 512)]
    rows += [aggregate_case(int(20853 * s), int(133975 * s), 14, 104), aggregate_case(int(3250 * s), int(20853 * s), 8, 256)]
    for r in rows:
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
