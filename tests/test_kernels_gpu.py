"""GPU numerics tests of the sm_100a kernels: each one is compared with a plain
PyTorch fp32 reference of the same op (or, for sampling, with the exact-replay
CPU oracle of the host engine)."""
import math

import numpy as np
import pytest
import torch

from grappa_b200 import _native
from grappa_b200.block import Block
from grappa_b200.ops import ref
from grappa_b200.sampler_gpu import GpuNeighborSampler, new_counters

pytestmark = pytest.mark.gpu

DEV = "cuda"


def cu():
    return _native.cuda()


def host_graph(n=2000, m=30000, seed=0):
    rng = np.random.default_rng(seed)
    u = rng.integers(0, n, m)
    v = rng.integers(0, n, m)
    v[: m // 5] = rng.integers(0, 8, m // 5)  # hubs
    u2 = np.concatenate([u, v, np.arange(n)])
    v2 = np.concatenate([v, u, np.arange(n)])
    g = _native.host().graph.HostGraph(u2, v2, n)
    ip = torch.from_numpy(g.indptr()).to(DEV)
    ix = torch.from_numpy(g.indices()).to(torch.int32).to(DEV)
    return g, ip, ix, n


def err_tensor():
    return torch.zeros(1, dtype=torch.int32, device=DEV)


# ----------------------------------------------------------------------------- sampling
def _compare_blocks(gpu_blocks, ref_blocks):
    for h, rb in enumerate(ref_blocks):
        b = gpu_blocks[len(gpu_blocks) - 1 - h]
        assert b.n_dst == rb["n_dst"] and b.n_src == rb["n_src"], (h, b, rb["n_dst"], rb["n_src"])
        np.testing.assert_array_equal(b.indptr.cpu().numpy(), rb["indptr"])
        np.testing.assert_array_equal(b.indices.cpu().numpy(), rb["indices"])
        np.testing.assert_array_equal(b.srcdata["_ID"].cpu().numpy(), rb["src_nid"])
        np.testing.assert_array_equal(b.src_sampled.cpu().numpy(), rb["src_sampled"])


def test_sampler_matches_cpu_oracle_exactly():
    g, ip, ix, n = host_graph()
    fan = [15, 10, 5]
    seeds = np.arange(0, 1536, 6, dtype=np.int64)
    sm = GpuNeighborSampler(fan, 256, n, DEV)
    counters = new_counters(11, DEV)
    gideg_all = torch.full((n,), 30, dtype=torch.int64, device=DEV)
    for step in range(3):  # three calls: exercises the tagged map across generations
        counters[1], counters[2] = 2, step
        cov = torch.zeros(2, device=DEV)
        sm.load_seeds(torch.from_numpy(seeds))
        sm.sample(ip, ix, counters, gideg=gideg_all, cov=cov)
        cu().step_end(counters)  # advances the generation of the compaction tags
        torch.cuda.synchronize()
        assert sm.err.item() == 0
        rb, cs, cn = _native.host().graph.sample_batch(g, fan, seeds, np.full(len(seeds), 30), 11, 2, step, False)
        _compare_blocks(sm.blocks(), rb)
        assert abs(cov[0].item() - cs) < 1e-2 and cov[1].item() == cn


def test_sampler_partial_batch_and_frontier():
    g, ip, ix, n = host_graph(seed=1)
    fan = [3, 4]
    seeds = np.array([5, 17, 100, 3, 1999, 0, 7], dtype=np.int64)
    sm = GpuNeighborSampler(fan, 64, n, DEV)
    counters = new_counters(3, DEV)
    sm.load_seeds(torch.from_numpy(seeds))
    sm.sample(ip, ix, counters)
    torch.cuda.synchronize()
    rb, _, _ = _native.host().graph.sample_batch(g, fan, seeds, None, 3, 0, 0, False)
    _compare_blocks(sm.blocks(), rb)


# ----------------------------------------------------------------------------- GEMM
def bf(x):
    return x.to(torch.bfloat16)


def run_gemm(A, a_mn, B, b_mn, M_cap, M_dev, N, K_cap, K_dev, splits, C, mode, bias=None, act=0, p=0.0,
             counters=None, salt=0, labels=None, n_classes=0, dl=None, loss=None, correct=None, n_rows=None,
             dbias=None, bn=256):
    err = err_tensor()
    cu().gemm(A, a_mn, B, b_mn, M_cap, M_dev, N, K_cap, K_dev, splits, C, mode, bias, act, p, counters, salt,
              labels, n_classes, dl, loss, correct, None, n_rows, dbias, err, bn)
    torch.cuda.synchronize()
    assert err.item() == 0
    return C


@pytest.mark.parametrize("M,K,N,bn", [(300, 208, 256, 256), (1000, 512, 48, 48), (129, 64, 64, 64),
                                      (257, 200, 128, 128), (5000, 512, 256, 256),
                                      # many tiles per persistent CTA, both TMEM buffers in turn
                                      (40001, 256, 256, 64), (70000, 128, 512, 256), (9000, 64, 48, 48)])
def test_gemm_kmajor_bias_relu(M, K, N, bn):
    torch.manual_seed(0)
    cap = (M + 127) // 128 * 128 + 128
    A = bf(torch.randn(cap, K, device=DEV))
    B = bf(torch.randn(N, K, device=DEV) / math.sqrt(K))
    bias = torch.randn(N, device=DEV)
    C = torch.full((cap, N), 7.0, device=DEV, dtype=torch.bfloat16)
    Mdev = torch.tensor([M], dtype=torch.int32, device=DEV)
    run_gemm(A, False, B, False, cap, Mdev, N, K, None, 1, C, 0, bias=bias, act=1, bn=bn)
    want = torch.relu(A[:M].float() @ B.float().t() + bias)
    torch.testing.assert_close(C[:M].float(), want, rtol=2e-2, atol=2e-2)
    assert bool((C[M:] == 7).all())


def test_gemm_dropout_matches_host_mask():
    torch.manual_seed(1)
    M, K, N, p = 256, 128, 256, 0.5
    A = bf(torch.randn(M, K, device=DEV))
    B = bf(torch.randn(N, K, device=DEV) / math.sqrt(K))
    bias = torch.zeros(N, device=DEV)
    C = torch.zeros((M, N), device=DEV, dtype=torch.bfloat16)
    counters = new_counters(21, DEV)
    counters[1], counters[2] = 4, 9
    run_gemm(A, False, B, False, M, None, N, K, None, 1, C, 0, bias=bias, act=1, p=p, counters=counters, salt=2)
    mask = torch.from_numpy(_native.host().dropout_mask(21, 4, 9, 2, M, N, N, p)).view(M, N).to(DEV).float()
    want = torch.relu(A.float() @ B.float().t()) * mask / (1 - p)
    torch.testing.assert_close(C.float(), want, rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("cap,live,N,K,bn", [(1024, 700, 256, 256, 256), (512, 130, 64, 512, 64),
                                             (2048, 2000, 128, 96, 128)])
def test_gemm_activation_backward_epilogue(cap, live, N, K, bn):
    """bf16 store with the ReLU/dropout backward fused: out = (H != 0) * (A B^T) * scale on
    the live rows, zeros on the tail rows up to the next multiple of 64."""
    torch.manual_seed(4)
    A = bf(torch.randn(cap, K, device=DEV))
    B = bf(torch.randn(N, K, device=DEV) / math.sqrt(K))
    H = bf(torch.relu(torch.randn(cap, N, device=DEV)))  # about half exact zeros
    C = torch.full((cap, N), 7.0, dtype=torch.bfloat16, device=DEV)
    m_dev = torch.tensor([live], dtype=torch.int32, device=DEV)
    err = err_tensor()
    cu().gemm(A, False, B, False, cap, m_dev, N, K, None, 1, C, 0, None, 0, 0.0, None, 0, None, 0, None, None, None,
              None, None, None, err, bn, H, 2.0, 64)
    torch.cuda.synchronize()
    assert err.item() == 0
    want = torch.where(H[:live] != 0, (A[:live].float() @ B.float().t()) * 2.0, torch.zeros((), device=DEV))
    torch.testing.assert_close(C[:live].float(), want, rtol=2e-2, atol=3e-2)
    tail = min(cap, (live + 63) // 64 * 64)
    assert bool((C[live:tail] == 0).all())
    assert bool((C[tail:] == 7.0).all())


@pytest.mark.parametrize("M,live,n_dst,H,F_,K,bn", [(4096, 3000, 700, 4, 64, 128, 256), (1024, 1000, 1000, 4, 172, 256, 256),
                                                   (700, 650, 90, 3, 24, 104, 64)])
def test_gemm_attention_logit_epilogue(M, live, n_dst, H, F_, K, bn):
    """z = x W^T stored bf16 with the GAT logits in the epilogue: el[m, h] = z[m, h] . a_l[h]
    for live rows, er the same with a_r for the first n_dst rows, from the stored values
    (heads of 172 columns straddle the 32-column chunks and the 256-column tiles)."""
    torch.manual_seed(6)
    N = H * F_
    A = bf(torch.randn(M, K, device=DEV))
    B = bf(torch.randn(N, K, device=DEV) / math.sqrt(K))
    al, ar = torch.randn(N, device=DEV), torch.randn(N, device=DEV)
    C = torch.zeros((M, N), dtype=torch.bfloat16, device=DEV)
    el, er = torch.zeros(M * H, device=DEV), torch.zeros(M * H, device=DEV)
    m_dev = torch.tensor([live], dtype=torch.int32, device=DEV)
    nd = torch.tensor([n_dst], dtype=torch.int32, device=DEV)
    err = err_tensor()
    cu().gemm(A, False, B, False, M, m_dev, N, K, None, 1, C, 0, None, 0, 0.0, None, 0, None, 0, None, None, None,
              None, None, None, err, bn, att_l=al, att_r=ar, att_el=el, att_er=er, att_heads=H, att_feat=F_,
              att_n_dst=nd)
    torch.cuda.synchronize()
    assert err.item() == 0
    z = C[:live].float().view(live, H, F_)
    torch.testing.assert_close(C[:live].float(), A[:live].float() @ B.float().t(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(el.view(M, H)[:live], (z * al.view(H, F_)).sum(-1), rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(er.view(M, H)[:n_dst], (z[:n_dst] * ar.view(H, F_)).sum(-1), rtol=1e-3, atol=1e-3)
    assert bool((el.view(M, H)[live:] == 0).all()) and bool((er.view(M, H)[n_dst:] == 0).all())


@pytest.mark.parametrize("Mo,Kx,R,live,splits", [(48, 208, 700, 650, 3), (256, 512, 4096, 4000, 8),
                                                 (256, 208, 130, 100, 1), (1024, 1024, 8192, 8000, 4)])
def test_gemm_dw_mn_major_split_k(Mo, Kx, R, live, splits):
    torch.manual_seed(2)
    dY = bf(torch.randn(R, Mo, device=DEV))
    dY[live:] = 0
    X = bf(torch.randn(R, Kx, device=DEV))
    C = torch.zeros((Mo, Kx), device=DEV, dtype=torch.float32)
    Kdev = torch.tensor([live], dtype=torch.int32, device=DEV)
    run_gemm(dY, True, X, True, Mo, None, Kx, R, Kdev, splits, C, 2, bn=256)
    want = dY[:live].float().t() @ X[:live].float()
    torch.testing.assert_close(C, want, rtol=1e-2, atol=5e-2)


@pytest.mark.parametrize("R,live,No,Kx", [(700, 650, 48, 512), (300, 300, 256, 512), (128, 77, 256, 208)])
def test_gemm_dx_mn_major_b(R, live, No, Kx):
    torch.manual_seed(3)
    dY = bf(torch.randn(R, No, device=DEV))
    W = bf(torch.randn(No, Kx, device=DEV) / math.sqrt(No))
    C = torch.full((R, Kx), 3.0, device=DEV, dtype=torch.bfloat16)
    Mdev = torch.tensor([live], dtype=torch.int32, device=DEV)
    run_gemm(dY, False, W, True, R, Mdev, Kx, No, None, 1, C, 0, bn=256)
    want = dY[:live].float() @ W.float()
    torch.testing.assert_close(C[:live].float(), want, rtol=2e-2, atol=2e-2)


def test_gemm_cross_entropy_epilogue():
    torch.manual_seed(4)
    M, cap, K, N, n_cls = 1000, 1152, 512, 48, 47
    X = bf(torch.randn(cap, K, device=DEV))
    W = bf(torch.randn(N, K, device=DEV) / math.sqrt(K))
    W[n_cls:] = 0
    bias = torch.randn(N, device=DEV) * 0.1
    labels = torch.randint(0, n_cls, (cap,), dtype=torch.int32, device=DEV)
    dl = torch.full((cap, N), 5.0, device=DEV, dtype=torch.bfloat16)
    loss = torch.zeros(1, device=DEV)
    correct = torch.zeros(1, dtype=torch.int32, device=DEV)
    dbias = torch.zeros(N, device=DEV)
    n_rows = torch.tensor([M], dtype=torch.int32, device=DEV)
    dummy = torch.zeros((1, 1), device=DEV)
    run_gemm(X, False, W, False, cap, n_rows, N, K, None, 1, dummy, 3, bias=bias, labels=labels, n_classes=n_cls,
             dl=dl, loss=loss, correct=correct, n_rows=n_rows, dbias=dbias, bn=48)
    logits = (X[:M].float() @ W.float().t() + bias)[:, :n_cls].requires_grad_(True)
    ce = torch.nn.functional.cross_entropy(logits, labels[:M].long())
    ce.backward()
    assert abs(loss.item() - ce.item()) < 2e-2 * max(1.0, ce.item())
    torch.testing.assert_close(dl[:M, :n_cls].float(), logits.grad, rtol=3e-2, atol=2e-5)
    assert bool((dl[:M, n_cls:] == 0).all())
    assert bool((dl[M:(M + 63) // 64 * 64] == 0).all())
    assert abs(correct.item() - int((logits.argmax(1) == labels[:M].long()).sum())) <= 3
    torch.testing.assert_close(dbias[:n_cls], logits.grad.sum(0), rtol=5e-2, atol=5e-4)


# ----------------------------------------------------------------------------- aggregation
def random_block(n_dst, n_src, max_deg, seed):
    g = torch.Generator().manual_seed(seed)
    deg = torch.randint(0, max_deg + 1, (n_dst,), generator=g)
    indptr = torch.zeros(n_dst + 1, dtype=torch.int32)
    indptr[1:] = torch.cumsum(deg, 0)
    indices = torch.randint(0, n_src, (int(indptr[-1]),), generator=g, dtype=torch.int32)
    src = torch.arange(n_src, dtype=torch.int32)
    return Block(indptr, indices, src, n_dst, n_src)


@pytest.mark.parametrize("mode,dim", [("mean", 104), ("mean", 256), ("sum", 64), ("gcn", 256), ("weighted", 600)])
def test_aggregate_forward(mode, dim):
    b = random_block(300, 1000, 20, 5)
    torch.manual_seed(5)
    h = bf(torch.randn(1000, dim))
    modes = {"mean": 0, "sum": 1, "gcn": 2, "weighted": 3}
    ew = torch.rand(b.num_edges()) if mode == "weighted" else None
    snorm = ref.gcn_src_norm(b) if mode == "gcn" else None
    out = torch.zeros((300, 2 * dim), dtype=torch.bfloat16, device=DEV)
    err = err_tensor()
    n_dev = torch.tensor([300], dtype=torch.int32, device=DEV)
    cu().aggregate(b.indptr.to(DEV), b.indices.to(DEV), n_dev, 0, 300, h.to(DEV), None, dim, modes[mode],
                   None if ew is None else ew.to(DEV), None if snorm is None else snorm.to(DEV), None, out, dim, 0,
                   0.0, 0, err)
    torch.cuda.synchronize()
    want = ref.aggregate(b, h.float(), mode, edge_weight=ew, src_norm=snorm)
    torch.testing.assert_close(out[:, dim:].float().cpu(), want, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(out[:, :dim].float().cpu(), h[:300].float())


def test_aggregate_through_src_map():
    b = random_block(200, 500, 12, 6)
    table = bf(torch.randn(5000, 104))
    src_map = torch.randperm(5000)[:500].to(torch.int32)
    out = torch.zeros((256, 208), dtype=torch.bfloat16, device=DEV)
    err = err_tensor()
    n_dev = torch.tensor([200], dtype=torch.int32, device=DEV)
    cu().aggregate(b.indptr.to(DEV), b.indices.to(DEV), n_dev, 0, 256, table.to(DEV), src_map.to(DEV), 104, 0,
                   None, None, None, out, 104, 0, 0.0, 0, err)
    torch.cuda.synchronize()
    h = table[src_map.long()].float()
    torch.testing.assert_close(out[:200, 104:].float().cpu(), ref.aggregate(b, h, "mean"), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(out[:200, :104].float().cpu(), h[:200])


@pytest.mark.parametrize("mode,dim", [("mean", 256), ("sum", 64), ("gcn", 128), ("weighted", 104)])
def test_aggregate_backward(mode, dim):
    b = random_block(300, 900, 16, 7)
    torch.manual_seed(7)
    h = torch.randn(900, dim, requires_grad=True)
    modes = {"mean": 0, "sum": 1, "gcn": 2, "weighted": 3}
    ew = torch.rand(b.num_edges()) if mode == "weighted" else None
    snorm = ref.gcn_src_norm(b) if mode == "gcn" else None
    out = torch.cat([h[:300], ref.aggregate(b, h, mode, edge_weight=ew, src_norm=snorm)], 1)
    dout = bf(torch.randn(300, 2 * dim))
    out.backward(dout.float())
    dsrc = torch.zeros((900, dim), device=DEV)
    err = err_tensor()
    n_dev = torch.tensor([300], dtype=torch.int32, device=DEV)
    cu().aggregate_bwd(b.indptr.to(DEV), b.indices.to(DEV), n_dev, 0, 300, dout.to(DEV), dim, 0, 0.0, dim,
                       modes[mode], None if ew is None else ew.to(DEV), None if snorm is None else snorm.to(DEV), None,
                       dsrc, err)
    torch.cuda.synchronize()
    torch.testing.assert_close(dsrc.cpu(), h.grad, rtol=1e-3, atol=1e-3)


def test_block_transpose_and_gathered_mean_backward():
    """The block transpose (CSR by source) and the gathered mean backward with the fused
    activation backward against a scatter reference in fp32."""
    torch.manual_seed(8)
    n_dst, n_src, cap, dim = 300, 1000, 1088, 64
    deg = torch.randint(0, 12, (n_dst,))
    indptr = torch.zeros(n_dst + 1, dtype=torch.int32)
    indptr[1:] = torch.cumsum(deg, 0)
    E = int(indptr[-1])
    indices = torch.randint(0, n_src, (E,), dtype=torch.int32)
    # edge ranks among each source's edges (what compaction K3 records with atomics)
    t_cnt = torch.zeros(cap, dtype=torch.int32)
    t_rank = torch.zeros(E, dtype=torch.int32)
    for e in torch.randperm(E).tolist():
        u = int(indices[e])
        t_rank[e] = t_cnt[u]
        t_cnt[u] += 1
    d = dict(device=DEV)
    tptr = torch.zeros(cap + 1, dtype=torch.int32, **d)
    tdst = torch.full((E,), -1, dtype=torch.int32, **d)
    nd, ns = torch.tensor([n_dst], dtype=torch.int32, **d), torch.tensor([n_src], dtype=torch.int32, **d)
    err = err_tensor()
    t_cnt_d = t_cnt.to(DEV)
    cu().block_transpose(indptr.to(DEV), indices.to(DEV), nd, ns, t_cnt_d, t_rank.to(DEV), tptr, tdst, err)
    torch.cuda.synchronize()
    assert err.item() == 0 and bool((t_cnt_d == 0).all())
    # every (src, dst) edge appears once in the transposed lists
    v_of_e = torch.repeat_interleave(torch.arange(n_dst), deg)
    tp, td = tptr.cpu(), tdst.cpu()
    got = sorted((u, int(td[k])) for u in range(n_src) for k in range(int(tp[u]), int(tp[u + 1])))
    assert got == sorted(zip(indices.tolist(), v_of_e.tolist()))
    dX = bf(torch.randn(n_dst, 2 * dim, device=DEV))
    H = bf(torch.relu(torch.randn(cap, dim, device=DEV)))
    dy = torch.full((cap, dim), 5.0, dtype=torch.bfloat16, **d)
    db = torch.zeros(dim, **d)
    cu().aggregate_bwd_gather(indptr.to(DEV), tptr, tdst, nd, ns, dX, 0, dim, dim, H, 2.0, dy, db, err)
    torch.cuda.synchronize()
    assert err.item() == 0
    g = torch.zeros(n_src, dim, **d)
    g[:n_dst] += dX[:, :dim].float()
    w = (1.0 / deg.clamp(min=1).float())[v_of_e].to(DEV)
    g.index_add_(0, indices.long().to(DEV), dX[v_of_e.to(DEV), dim:].float() * w[:, None])
    want = torch.where(H[:n_src] != 0, g * 2.0, torch.zeros((), **d))
    torch.testing.assert_close(dy[:n_src].float(), want, rtol=2e-2, atol=2e-2)
    tail = (n_src + 63) // 64 * 64
    assert bool((dy[n_src:tail] == 0).all()) and bool((dy[tail:] == 5.0).all())
    # dbias sums the fp32 values before their bf16 rounding
    torch.testing.assert_close(db, want.sum(0), rtol=1e-3, atol=1e-2)


def test_act_bwd_mask_bias_and_clear():
    torch.manual_seed(8)
    R, n, dim = 700, 613, 256
    dh = torch.randn(R, dim, device=DEV)
    dh_copy = dh.clone()
    h = bf(torch.relu(torch.randn(R, dim, device=DEV)))
    dy = torch.full((R, dim), 9.0, device=DEV, dtype=torch.bfloat16)
    dbias = torch.zeros(dim, device=DEV)
    n_dev = torch.tensor([n], dtype=torch.int32, device=DEV)
    cu().act_bwd(dh, h, dy, n_dev, 0, dim, 2.0, dbias, R)
    torch.cuda.synchronize()
    want = torch.where(h[:n] != 0, dh_copy[:n] * 2.0, torch.zeros_like(dh_copy[:n]))
    torch.testing.assert_close(dy[:n].float(), want, rtol=1e-2, atol=1e-2)
    assert bool((dy[n:(n + 63) // 64 * 64] == 0).all())
    assert bool((dh[:n] == 0).all())
    torch.testing.assert_close(dbias, bf(want).float().sum(0), rtol=1e-4, atol=1e-3)


def test_gather_rows():
    table = torch.randn(3000, 104, device=DEV)
    ids = torch.randint(0, 3000, (500,), dtype=torch.int32, device=DEV)
    out = torch.zeros((512, 104), dtype=torch.bfloat16, device=DEV)
    cu().gather_rows(table, ids, None, 500, 512, 104, out)
    torch.testing.assert_close(out[:500].float(), bf(table[ids.long()]).float())


def test_pull_rows_checks_ids_and_capacity():
    """pull_rows over two local "rank" tables: rows are fetched by global id; an id outside
    the global range is skipped with kErrBadIndex, a count above the capacity is clamped
    with kErrCapacity (no write past the output)."""
    t0 = torch.randn(100, 16, device=DEV).to(torch.bfloat16)
    t1 = torch.randn(50, 16, device=DEV).to(torch.bfloat16)
    prefix = torch.tensor([0, 100, 150], dtype=torch.int64, device=DEV)
    gids = torch.tensor([3, 120, 99, 100, 149, 0], dtype=torch.int64, device=DEV)
    full = torch.cat([t0, t1])
    out = torch.zeros((8, 16), dtype=torch.bfloat16, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    tables = [t0.data_ptr(), t1.data_ptr()]
    n = torch.tensor([6], dtype=torch.int32, device=DEV)
    cu().pull_rows(tables, 16, 2, 32, gids, n, 0, prefix, out.data_ptr(), 16, 1, 7, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    torch.testing.assert_close(out[1:7], full[gids.long()])
    assert bool((out[0] == 0).all()) and bool((out[7] == 0).all())
    # a bad id (-1 and 150) is skipped and flagged; the other rows still arrive
    out.zero_()
    bad = torch.tensor([5, -1, 150, 140], dtype=torch.int64, device=DEV)
    cu().pull_rows(tables, 16, 2, 32, bad, torch.tensor([4], dtype=torch.int32, device=DEV), 0, prefix,
                   out.data_ptr(), 16, 0, 8, err)
    torch.cuda.synchronize()
    assert int(err.item()) & (1 << 2)
    torch.testing.assert_close(out[0], full[5])
    torch.testing.assert_close(out[3], full[140])
    assert bool((out[1:3] == 0).all())
    # a device count above the capacity is clamped: rows past cap stay untouched
    err.zero_()
    out.zero_()
    sentinel = torch.full((4, 16), 7.0, dtype=torch.bfloat16, device=DEV)
    out2 = torch.cat([torch.zeros((2, 16), dtype=torch.bfloat16, device=DEV), sentinel])
    cu().pull_rows(tables, 16, 2, 32, gids, torch.tensor([6], dtype=torch.int32, device=DEV), 0, prefix,
                   out2.data_ptr(), 16, 0, 2, err)
    torch.cuda.synchronize()
    assert int(err.item()) & (1 << 1)
    torch.testing.assert_close(out2[:2], full[gids[:2].long()])
    assert bool((out2[2:] == 7.0).all())


# ----------------------------------------------------------------------------- optimizer
def test_adam_matches_torch():
    torch.manual_seed(9)
    n = 10000
    p0 = torch.randn(n)
    p_ref = torch.nn.Parameter(p0.clone())
    opt = torch.optim.Adam([p_ref], lr=3e-3)
    param, m, v = p0.clone().to(DEV), torch.zeros(n, device=DEV), torch.zeros(n, device=DEV)
    wbf = torch.zeros(n, dtype=torch.bfloat16, device=DEV)
    counters = new_counters(0, DEV)
    for _ in range(3):
        g = torch.randn(n)
        p_ref.grad = g.clone()
        opt.step()
        grad = g.to(DEV)
        cu().adam(param, m, v, grad, wbf, 3e-3, 0.9, 0.999, 1e-8, 0.0, counters, 1.0, None, True)
        cu().step_end(counters)
        torch.cuda.synchronize()
        assert bool((grad == 0).all())
    torch.testing.assert_close(param.cpu(), p_ref.detach(), rtol=1e-5, atol=1e-6)
    # the bf16 working copy is the rounding of the kernel's own fp32 master weights
    assert torch.equal(wbf, bf(param))


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fused_allreduce_adam_single_rank(mode, dtype):
    """One rank, two buckets (launched last first), a ragged end: the fused kernel's Adam
    on the coverage-scaled gradient against torch's Adam; the gradient is cleared and
    the bf16 copy is the rounding of the fp32 master."""
    from grappa_b200.parallel.allreduce import FusedAllReduceAdam
    from grappa_b200.parallel.comm import Comm

    torch.manual_seed(10)
    n = 50003
    p0 = torch.randn(n)
    p_ref = torch.nn.Parameter(p0.clone())
    opt = torch.optim.Adam([p_ref], lr=1e-2)
    ar = FusedAllReduceAdam(Comm(), n, buckets=[(0, 20000), (20000, n)], grad_dtype=dtype, modes=[mode, mode])
    ar.param.copy_(p0)
    m, v = torch.zeros(n, device=DEV), torch.zeros(n, device=DEV)
    wbf = torch.zeros(n, dtype=torch.bfloat16, device=DEV)
    counters = new_counters(0, DEV)
    err = err_tensor()
    cov = torch.tensor([16.0, 20.0], device=DEV)  # c_r = 0.8
    ar.bind(counters, m, v, wbf, 1e-2, err=err, cov=cov)
    for _ in range(4):
        g = torch.randn(n).to(dtype)
        p_ref.grad = g.float() * 0.8
        opt.step()
        ar.grad.copy_(g.to(DEV))
        ar.launch(1)
        ar.launch(0)
        cu().step_end(counters)
        torch.cuda.synchronize()
        assert err.item() == 0
        assert bool((ar.grad == 0).all())
    torch.testing.assert_close(ar.param.cpu(), p_ref.detach(), rtol=1e-5, atol=1e-6)
    assert torch.equal(wbf, ar.param.to(torch.bfloat16))
    ar.close()



@pytest.mark.parametrize("a0,b0", [(0, 0), (3, 5), (1, 2)])
def test_csr_merge_and_copy(a0, b0):
    """csr_merge (two CSRs concatenated, sources translated through the map; 16-byte
    source words after a scalar head, so edge offsets that are not multiples of four
    are covered) and the unrolled copy against torch, on local memory."""
    torch.manual_seed(5)
    n_glob = 5000
    da, db = torch.randint(0, 40, (300,)), torch.randint(0, 40, (211,))
    ipa = torch.cat([torch.zeros(1, dtype=torch.int64), torch.cumsum(da, 0)]) + a0
    ipb = torch.cat([torch.zeros(1, dtype=torch.int64), torch.cumsum(db, 0)]) + b0
    ia = torch.randint(0, n_glob, (int(ipa[-1]) + 7,), dtype=torch.int32)
    ib = torch.randint(0, n_glob, (int(ipb[-1]) + 7,), dtype=torch.int32)
    mp = torch.randperm(n_glob).to(torch.int32)
    ipa_d, ipb_d, ia_d, ib_d, mp_d = (t.to(DEV) for t in (ipa, ipb, ia, ib, mp))
    ea, eb = int(ipa[-1] - a0), int(ipb[-1] - b0)
    out_ip = torch.full((300 + 211 + 4,), -1, dtype=torch.int64, device=DEV)
    out_ix = torch.full((ea + eb + 9,), -1, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    cu().csr_merge(ipa_d.data_ptr(), ia_d.data_ptr(), 300, ipb_d.data_ptr(), ib_d.data_ptr(), 211, mp_d, out_ip,
                   out_ix, err)
    torch.cuda.synchronize()
    want_ip = torch.cat([ipa - a0, (ipb[1:] - b0) + ea, torch.full((3,), ea + eb, dtype=torch.int64)])
    assert torch.equal(out_ip.cpu(), want_ip)
    want_ix = mp[torch.cat([ia[a0:a0 + ea], ib[b0:b0 + eb]]).long()]
    assert torch.equal(out_ix[:ea + eb].cpu(), want_ix)
    assert torch.all(out_ix[ea + eb:] == -1) and int(err) == 0
    # partition ranges translated arithmetically: the same result as a map holding
    # iotas there
    g0a, g0b = 1000, 3000
    mp2 = mp.clone()
    mp2[g0a:g0a + 300] = torch.arange(300, dtype=torch.int32)
    mp2[g0b:g0b + 211] = 300 + torch.arange(211, dtype=torch.int32)
    want2 = mp2[torch.cat([ia[a0:a0 + ea], ib[b0:b0 + eb]]).long()]
    mp2_d = mp2.to(DEV)
    mp2_d[g0a:g0a + 300] = -5  # not read for sources in the ranges
    mp2_d[g0b:g0b + 211] = -5
    out_ix.fill_(-1)
    cu().csr_merge(ipa_d.data_ptr(), ia_d.data_ptr(), 300, ipb_d.data_ptr(), ib_d.data_ptr(), 211, mp2_d, out_ip,
                   out_ix, err, g0_a=g0a, g0_b=g0b)
    torch.cuda.synchronize()
    assert torch.equal(out_ix[:ea + eb].cpu(), want2)
    # copy: 16-byte words, a count that is not a multiple of the unroll
    src = torch.randint(0, 1 << 30, (4 * 100003,), dtype=torch.int32, device=DEV)
    dst = torch.zeros_like(src)
    cu().peer_copy(dst.data_ptr(), src.data_ptr(), src.numel() * 4)
    torch.cuda.synchronize()
    assert torch.equal(dst, src)


@pytest.mark.parametrize("n_global", [100003, 4096 * 3, 17])
def test_mark_compact_halo_ids(n_global):
    """Halo discovery of the repartition: marked ids (minus the iota-mapped own and
    neighbour ranges) are compacted in id order into out_ids, the map gets base + rank,
    the count goes to n_out and the marks are cleared; run twice on the same buffers
    (16-byte mark words, a ragged tail, the tagged look-back scan)."""
    torch.manual_seed(8)
    mark = torch.zeros(n_global, dtype=torch.uint8, device=DEV)
    mp = torch.full((n_global,), -1, dtype=torch.int32, device=DEV)
    scratch = torch.zeros(cu().mark_compact_scratch_words(n_global), dtype=torch.int64, device=DEV)
    out = torch.full((n_global,), -1, dtype=torch.int64, device=DEV)
    n_out = torch.zeros(1, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    for it in range(2):
        ids = torch.randint(0, n_global, (max(1, n_global // 7),), dtype=torch.int32, device=DEV)
        cu().mark_ids(ids.data_ptr(), None, ids.numel(), mark)
        lo, cnt = n_global // 3, n_global // 5
        cu().iota_map(mp, lo, cnt, 0, mark)
        base = cnt
        cu().mark_compact(mark, out, mp, base, n_out, scratch, err)
        torch.cuda.synchronize()
        want = torch.unique(ids.long())
        want = want[(want < lo) | (want >= lo + cnt)]
        k = int(n_out)
        assert k == want.numel() and int(err) == 0
        assert torch.equal(out[:k].cpu(), want.cpu())
        assert torch.equal(mp[want].cpu(), torch.arange(base, base + k, dtype=torch.int32))
        assert int(mark.sum()) == 0


@pytest.mark.parametrize("dim,n_ids", [(32, 1000), (104, 5001), (128, 777), (608, 3001), (1104, 400)])
def test_pull_rows_widths(dim, n_ids):
    """pull_rows at every row width class (8, 16 or 32 lanes per row with several rows
    per warp in flight, and one warp per row above 2 KB) from three local "rank" tables,
    into rows at an offset of a wider output."""
    torch.manual_seed(10)
    sizes = [300, 1, 500]
    tabs = [torch.randn(s, dim, device=DEV).to(torch.bfloat16) for s in sizes]
    full = torch.cat(tabs)
    prefix = torch.tensor([0, 300, 301, 801], dtype=torch.int64, device=DEV)
    gids = torch.randint(0, 801, (n_ids,), dtype=torch.int64, device=DEV)
    ld = dim + 8
    out = torch.zeros((n_ids + 10, ld), dtype=torch.bfloat16, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    cu().pull_rows([t.data_ptr() for t in tabs], dim, 2, dim * 2, gids, None, n_ids, prefix, out.data_ptr(), ld, 5,
                   n_ids, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(out[5:5 + n_ids, :dim], full[gids.long()])
    assert bool((out[:5] == 0).all()) and bool((out[5 + n_ids:] == 0).all()) and bool((out[:, dim:] == 0).all())
