"""Numerics of the row-wise network kernels (nn.cu, gat.cu) against plain PyTorch
fp32 references of the same ops, on bf16-exact inputs."""
import math
import pytest
import torch
import torch.nn.functional as F

from grappa_b200 import _native

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def cu():
    return _native.cuda()


def bf(x):
    return x.to(torch.bfloat16)


def test_cross_entropy_kernel():
    torch.manual_seed(0)
    n, cap, C, ld = 300, 320, 47, 48
    logits = bf(torch.randn(cap, ld, device=DEV) * 3)
    labels = torch.randint(0, C, (cap,), dtype=torch.int32, device=DEV)
    mask = (torch.rand(cap, device=DEV) > 0.3).to(torch.uint8)
    n_rows = torch.tensor([n], dtype=torch.int32, device=DEV)
    n_sel = torch.tensor([int(mask[:n].sum())], dtype=torch.int32, device=DEV)
    dl = torch.full((cap, ld), 7.0, dtype=torch.bfloat16, device=DEV)
    dbias = torch.zeros(ld, device=DEV)
    loss = torch.zeros(1, device=DEV)
    correct = torch.zeros(1, dtype=torch.int32, device=DEV)
    cu().cross_entropy(logits, C, labels, n_rows, cap, mask, n_sel, dl, dbias, loss, correct)
    torch.cuda.synchronize()
    sel = mask[:n].bool()
    x = logits[:n, :C].float().requires_grad_(True)
    ref = F.cross_entropy(x[sel], labels[:n][sel].long(), reduction="sum") / float(n_sel)
    ref.backward()
    assert abs(float(loss) - float(ref)) < 1e-3 * max(1.0, float(ref))
    torch.testing.assert_close(dl[:n, :C].float(), x.grad, atol=2e-3, rtol=1e-2)
    assert torch.all(dl[n:320] == 0) and torch.all(dl[:n, C:] == 0)
    torch.testing.assert_close(dbias[:C], x.grad.sum(0), atol=2e-3, rtol=2e-2)
    pred = logits[:n, :C].float().argmax(1)
    assert int(correct) == int(((pred == labels[:n].long()) & sel).sum())


@pytest.mark.parametrize("act", [0, 1])
def test_batchnorm_kernels(act):
    torch.manual_seed(1)
    n, cap, dim, C = 500, 576, 64, 60  # C < dim: padded columns
    x = bf(torch.randn(cap, dim, device=DEV) * 2 + 0.5)
    gamma = torch.randn(dim, device=DEV)
    beta = torch.randn(dim, device=DEV)
    gamma[C:] = 0
    beta[C:] = 0
    rm = torch.zeros(C, device=DEV)
    rv = torch.ones(C, device=DEV)
    nb = torch.zeros((), dtype=torch.int64, device=DEV)
    sums = torch.zeros(2 * dim, device=DEV)
    y = torch.zeros(cap, dim, dtype=torch.bfloat16, device=DEV)
    nd = torch.tensor([n], dtype=torch.int32, device=DEV)
    cu().batchnorm_fwd(x, dim, nd, cap, sums, gamma, beta, rm, rv, nb, 0.1, 1e-5, True, act, y)
    xr = x[:n, :C].float().requires_grad_(True)
    bn = torch.nn.BatchNorm1d(C).to(DEV)
    with torch.no_grad():
        bn.weight.copy_(gamma[:C])
        bn.bias.copy_(beta[:C])
    yr = bn(xr)
    if act:
        yr = F.relu(yr)
    torch.testing.assert_close(y[:n, :C].float(), yr, atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(rm, bn.running_mean, atol=1e-4, rtol=1e-3)
    torch.testing.assert_close(rv, bn.running_var, atol=1e-4, rtol=1e-3)
    assert int(nb) == 1
    # backward
    gy = torch.randn(n, C, device=DEV)
    dy = torch.zeros(cap, dim, device=DEV)
    dy[:n, :C] = gy
    bsums = torch.zeros(2 * dim, device=DEV)
    dgamma = torch.zeros(dim, device=DEV)
    dbeta = torch.zeros(dim, device=DEV)
    dx = torch.zeros(cap, dim, dtype=torch.bfloat16, device=DEV)
    cu().batchnorm_bwd(x, y if act else None, dy, True, dim, nd, cap, sums, bsums, gamma, dgamma, dbeta, 1e-5, dx)
    torch.cuda.synchronize()
    # the ReLU mask of the kernel is its own bf16 output; use the same mask in the reference
    yr.backward(gy * (y[:n, :C].float() != 0) if act else gy)
    torch.testing.assert_close(dx[:n, :C].float(), xr.grad, atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(dgamma[:C], bn.weight.grad, atol=5e-2, rtol=2e-2)
    torch.testing.assert_close(dbeta[:C], bn.bias.grad, atol=5e-2, rtol=2e-2)
    assert torch.all(dy == 0)
    assert torch.all(dx[n:576] == 0)


def test_l2norm_kernels():
    torch.manual_seed(2)
    n, cap, dim = 200, 256, 48
    z = bf(torch.relu(torch.randn(cap, dim, device=DEV)))
    z[5] = 0  # zero row: norm 1
    y = torch.zeros(cap, dim, dtype=torch.bfloat16, device=DEV)
    norms = torch.zeros(cap, device=DEV)
    nd = torch.tensor([n], dtype=torch.int32, device=DEV)
    cu().l2norm_fwd(z, dim, nd, cap, y, norms)
    zr = z[:n].float().requires_grad_(True)
    nr = zr.norm(2, 1, keepdim=True)
    nr = torch.where(nr == 0, torch.ones_like(nr), nr)
    yr = zr / nr
    torch.testing.assert_close(y[:n].float(), yr, atol=1e-2, rtol=1e-2)
    g = torch.randn(n, dim, device=DEV)
    dy = torch.zeros(cap, dim, device=DEV)
    dy[:n] = g
    dz = torch.zeros(cap, dim, device=DEV)
    cu().l2norm_bwd(y, dy, norms, dim, nd, cap, dz)
    torch.cuda.synchronize()
    yr.backward(g)
    torch.testing.assert_close(dz[:n], zr.grad, atol=2e-2, rtol=2e-2)
    assert torch.all(dy == 0)


def test_dropout_rows_matches_mask():
    n, cap, dim, ld = 100, 128, 64, 80
    x = bf(torch.randn(cap, ld, device=DEV))
    out = torch.zeros(cap, ld, dtype=torch.bfloat16, device=DEV)
    counters = torch.tensor([3, 1, 4, 0, 0, 0], dtype=torch.int64, device=DEV)
    nd = torch.tensor([n], dtype=torch.int32, device=DEV)
    cu().dropout_rows(x[:, :dim], out[:, :dim], dim, ld, nd, cap, 0.5, counters, 9)
    torch.cuda.synchronize()
    mask = torch.from_numpy(_native.host().dropout_mask(3, 1, 4, 9, n, dim, ld, 0.5)).view(n, dim).to(DEV)
    ref = x[:n, :dim].float() * mask.float() * 2.0
    torch.testing.assert_close(out[:n, :dim].float(), ref, atol=1e-2, rtol=1e-2)
    assert torch.all(out[n:, :dim] == 0)
    g = torch.randn(cap, dim, device=DEV)
    g0 = g.clone()
    cu().dropout_grad(g, dim, ld, nd, cap, 0.5, counters, 9)
    torch.testing.assert_close(g[:n], g0[:n] * mask.float() * 2.0)


def _gat_ref(indptr, indices, n_dst, z, al, ar, bias, H, F_, slope, mean_heads):
    """fp32 oracle with an explicit loop over the destinations: for each v, the scores
    of its in-edges, their softmax per head and the weighted sum of the source rows."""
    zz = z.view(z.shape[0], H, F_)
    a_l, a_r = al.view(H, F_), ar.view(H, F_)
    ip = indptr.tolist()
    rows = []
    for v in range(n_dst):
        u = indices[ip[v]:ip[v + 1]].long()
        if u.numel() == 0:
            rows.append(bias.view(H, F_).clone())
            continue
        el = (zz[u] * a_l).sum(-1)                  # [deg, H]
        er = (zz[v] * a_r).sum(-1)                  # [H]
        att = torch.softmax(F.leaky_relu(el + er, slope), dim=0)
        rows.append((att.unsqueeze(-1) * zz[u]).sum(0) + bias.view(H, F_))
    out = torch.stack(rows)
    return out.mean(1) if mean_heads else out.flatten(1)


@pytest.mark.parametrize("H,F_,mean_heads,max_deg", [(4, 16, False, 8), (4, 12, True, 8), (2, 20, True, 8),
                                                       (4, 64, False, 80), (4, 24, True, 70)])
def test_gat_kernels(H, F_, mean_heads, max_deg):
    """GAT scores, the one-pass forward (online softmax over batches of 32 in-edges: the
    max_deg=80 cases cross batches) and the backward against the loop oracle."""
    torch.manual_seed(3)
    n_dst, n_src = 70, 300
    deg = torch.randint(0, max_deg + 1, (n_dst,))
    indptr = torch.zeros(n_dst + 1, dtype=torch.int32)
    indptr[1:] = torch.cumsum(deg, 0)
    E = int(indptr[-1])
    indices = torch.randint(0, n_src, (E,), dtype=torch.int32)
    indptr, indices = indptr.to(DEV), indices.to(DEV)
    HF = H * F_
    hfp = (HF + 7) // 8 * 8
    z = torch.zeros(n_src, hfp, dtype=torch.bfloat16, device=DEV)
    z[:, :HF] = bf(torch.randn(n_src, HF, device=DEV))
    al = torch.randn(HF, device=DEV) * 0.3
    ar = torch.randn(HF, device=DEV) * 0.3
    bias = torch.randn(HF, device=DEV) * 0.1
    f32 = dict(dtype=torch.float32, device=DEV)
    el, er = torch.zeros(n_src * H, **f32), torch.zeros(n_dst * H, **f32)
    smax, ssum = torch.zeros(n_dst * H, **f32), torch.zeros(n_dst * H, **f32)
    fo = (F_ + 7) // 8 * 8 if mean_heads else hfp
    out = torch.zeros(n_dst, fo, dtype=torch.bfloat16, device=DEV)
    nd = torch.tensor([n_dst], dtype=torch.int32, device=DEV)
    ns = torch.tensor([n_src], dtype=torch.int32, device=DEV)
    args = (indptr, indices, nd, n_dst, ns, n_src, H, F_, z, al, ar, el, er, smax, ssum, 0.2)
    cu().gat_scores(*args)
    cu().gat_fwd(*args, bias, mean_heads, 0, 0.0, None, 0, out)
    zf = z[:, :HF].float().requires_grad_(True)
    alr, arr, br = al.clone().requires_grad_(True), ar.clone().requires_grad_(True), bias.clone().requires_grad_(True)
    ref = _gat_ref(indptr, indices, n_dst, zf, alr, arr, br, H, F_, 0.2, mean_heads)
    w = F_ if mean_heads else HF
    torch.testing.assert_close(out[:, :w].float(), ref, atol=2e-2, rtol=2e-2)
    # backward
    g = bf(torch.randn(n_dst, fo, device=DEV))
    if mean_heads:
        g[:, F_:] = 0
    escr = torch.zeros(max(E, 1) * H, **f32)
    dl_, dr_ = torch.zeros(n_src * H, **f32), torch.zeros(n_dst * H, **f32)
    dz = torch.zeros(n_src, hfp, **f32)
    dzb = torch.zeros(n_src + 64, hfp, dtype=torch.bfloat16, device=DEV)
    db, dal, dar = torch.zeros(HF, **f32), torch.zeros(HF, **f32), torch.zeros(HF, **f32)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    cu().gat_bwd(*args, mean_heads, g, escr, dl_, dr_, dz, db, dal, dar, dzb, err)
    torch.cuda.synchronize()
    ref.backward(g[:, :w].float())
    torch.testing.assert_close(dzb[:n_src, :HF].float(), zf.grad, atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(db, br.grad, atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(dal, alr.grad, atol=5e-2, rtol=3e-2)
    torch.testing.assert_close(dar, arr.grad, atol=5e-2, rtol=3e-2)
    assert torch.all(dz == 0) and torch.all(dl_ == 0)
    assert int(err) == 0


@pytest.mark.parametrize("H,F_,ip,max_deg", [(4, 64, 104, 40), (2, 24, 40, 8), (3, 16, 16, 70)])
def test_gat_input_layer_projection_after_aggregation(H, F_, ip, max_deg):
    """Input layer with the attention on x and the projection after the aggregation
    (gat_in_prep, gat_in_scores, gat_in_fwd, then y Wbd^T) against the loop oracle on
    z = x W^T; its backward (gat_in_bwd on dL/dy = dout Wbd, gat_in_dw on dout^T y,
    col_sum_bf16) against autograd through the oracle.  torch stands in for the GEMMs."""
    torch.manual_seed(4)
    n_dst, n_src = 70, 300
    deg = torch.randint(0, max_deg + 1, (n_dst,))
    indptr = torch.zeros(n_dst + 1, dtype=torch.int32)
    indptr[1:] = torch.cumsum(deg, 0)
    E = int(indptr[-1])
    indices = torch.randint(0, n_src, (E,), dtype=torch.int32)
    indptr, indices = indptr.to(DEV), indices.to(DEV)
    HF, hin = H * F_, H * ip
    f32 = dict(dtype=torch.float32, device=DEV)
    x = bf(torch.randn(n_src, ip, device=DEV))
    W = bf(torch.randn(HF, ip, device=DEV) * 0.1)
    al = torch.randn(HF, device=DEV) * 0.3
    ar = torch.randn(HF, device=DEV) * 0.3
    wl, wr = torch.zeros(hin, **f32), torch.zeros(hin, **f32)
    Wbd = torch.full((HF, hin), 7.0, dtype=torch.bfloat16, device=DEV)
    cu().gat_in_prep(W, al, ar, H, F_, ip, wl, wr, Wbd)
    Wh = W.float().view(H, F_, ip)
    torch.testing.assert_close(wl, (al.view(H, F_, 1) * Wh).sum(1).flatten(), atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(wr, (ar.view(H, F_, 1) * Wh).sum(1).flatten(), atol=1e-4, rtol=1e-4)
    assert torch.equal(Wbd.float(), torch.block_diag(*Wh))
    el, er = torch.zeros(n_src * H, **f32), torch.zeros(n_dst * H, **f32)
    smax, ssum = torch.zeros(n_dst * H, **f32), torch.zeros(n_dst * H, **f32)
    nd = torch.tensor([n_dst], dtype=torch.int32, device=DEV)
    ns = torch.tensor([n_src], dtype=torch.int32, device=DEV)
    args = (indptr, indices, nd, n_dst, ns, n_src, H, ip, x, wl, wr, el, er, smax, ssum, 0.2)
    cu().gat_in_scores(*args)
    Y = torch.zeros(n_dst, hin, dtype=torch.bfloat16, device=DEV)
    cu().gat_in_fwd(*args, Y)
    xf = x.float()
    Wr = W.float().clone().requires_grad_(True)
    alr, arr = al.clone().requires_grad_(True), ar.clone().requires_grad_(True)
    ref = _gat_ref(indptr, indices, n_dst, xf @ Wr.t(), alr, arr, torch.zeros(HF, **f32), H, F_, 0.2, False)
    torch.testing.assert_close(Y.float() @ Wbd.float().t(), ref, atol=3e-2, rtol=3e-2)
    # backward
    g = bf(torch.randn(n_dst, HF, device=DEV))
    G = (g.float() @ Wbd.float()).bfloat16()
    escr = torch.zeros(max(E, 1) * H, **f32)
    dl_, dr_ = torch.zeros(n_src * H, **f32), torch.zeros(n_dst * H, **f32)
    xl, xr = torch.zeros(hin, **f32), torch.zeros(hin, **f32)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    cu().gat_in_bwd(*args, G, escr, dl_, dr_, xl, xr, err)
    T = g.float().t() @ Y.float()
    dW = torch.zeros(HF, ip, **f32)
    dal, dar = torch.zeros(HF, **f32), torch.zeros(HF, **f32)
    cu().gat_in_dw(T, xl, xr, al, ar, W.float(), H, F_, ip, dW, dal, dar)
    db = torch.zeros(HF, **f32)
    cu().col_sum_bf16(g, nd, HF, db)
    torch.cuda.synchronize()
    ref.backward(g.float())

    def rel(a, b):
        return float((a - b).norm() / b.norm().clamp(min=1e-12))

    assert rel(dW, Wr.grad) < 2e-2, rel(dW, Wr.grad)
    assert rel(dal, alr.grad) < 3e-2, rel(dal, alr.grad)
    assert rel(dar, arr.grad) < 3e-2, rel(dar, arr.grad)
    torch.testing.assert_close(db, g.float().sum(0), atol=1e-2, rtol=1e-3)
    assert torch.all(dl_ == 0)
    assert int(err) == 0


@pytest.mark.parametrize("ip,C,n_dst,max_deg", [(256, 47, 1021, 5), (104, 20, 300, 9), (64, 64, 130, 0)])
def test_sage_head_matches_torch(ip, C, n_dst, max_deg):
    """Fused GraphSAGE output layer: [h_v | mean h_u], logits, mean cross-entropy, the
    bf16 dlogits (tail rows to the next multiple of 64 zeroed), the bias gradient, the
    correct count and dX = dlogits W, against fp32 torch on the same bf16 operands."""
    torch.manual_seed(7)
    n_src = n_dst + 500
    cap = (n_dst + 63) // 64 * 64 + 64
    deg = torch.randint(0, max_deg + 1, (n_dst,))
    indptr = torch.zeros(n_dst + 1, dtype=torch.int32)
    indptr[1:] = torch.cumsum(deg, 0)
    indices = torch.randint(0, n_src, (int(indptr[-1]) + 1,), dtype=torch.int32)
    h = bf(torch.randn(n_src, ip, device=DEV))
    cp = (C + 7) // 8 * 8
    w = torch.zeros(cp, 2 * ip, dtype=torch.bfloat16, device=DEV)
    w[:C] = bf(torch.randn(C, 2 * ip, device=DEV) / math.sqrt(2 * ip))
    bias = torch.randn(cp, device=DEV) * 0.1
    labels = torch.randint(0, C, (cap,), dtype=torch.int32, device=DEV)
    x = torch.zeros(cap, 2 * ip, dtype=torch.bfloat16, device=DEV)
    dl = torch.full((cap, cp), 5.0, dtype=torch.bfloat16, device=DEV)
    dx = torch.zeros(cap, 2 * ip, dtype=torch.bfloat16, device=DEV)
    loss, correct = torch.zeros(1, device=DEV), torch.zeros(1, dtype=torch.int32, device=DEV)
    db = torch.zeros(cp, device=DEV)
    nd = torch.tensor([n_dst], dtype=torch.int32, device=DEV)
    cu().sage_head(indptr.to(DEV), indices.to(DEV), nd, cap, h, ip, w, bias, C, labels, x, dl, dx, loss, correct, db)
    torch.cuda.synchronize()
    # oracle
    hf = h.float().cpu()
    rows = []
    for v in range(n_dst):
        u = indices[indptr[v]:indptr[v + 1]].long()
        agg = hf[u].mean(0) if u.numel() else torch.zeros(ip)
        rows.append(torch.cat([hf[v], agg]))
    xr = bf(torch.stack(rows)).float()
    torch.testing.assert_close(x[:n_dst].float().cpu(), xr, atol=1e-2, rtol=1e-2)
    z = xr @ w[:C].float().cpu().t() + bias[:C].cpu()
    y = labels[:n_dst].long().cpu()
    want_loss = F.cross_entropy(z, y)
    assert abs(float(loss) - float(want_loss)) < 2e-3 * max(1.0, float(want_loss))
    assert int(correct) == int((z.argmax(1) == y).sum())
    g = (torch.softmax(z, 1) - F.one_hot(y, C).float()) / n_dst
    torch.testing.assert_close(dl[:n_dst, :C].float().cpu(), g, atol=2e-4, rtol=2e-2)
    assert bool((dl[:n_dst, C:] == 0).all())
    tail = min(cap, (n_dst + 63) // 64 * 64)
    assert bool((dl[n_dst:tail] == 0).all()) and bool((dl[tail:] == 5.0).all())
    torch.testing.assert_close(db[:C].cpu(), bf(g).float().sum(0), atol=1e-4, rtol=1e-3)
    want_dx = bf(g).float() @ w[:C].float().cpu()
    torch.testing.assert_close(dx[:n_dst].float().cpu(), want_dx, atol=1e-4, rtol=2e-2)
    if not cu().sage_head_fused_bwd():
        return
    # the aggregation's backward fused into the tile kernel (dx not written)
    dsrc = torch.zeros(n_src, ip, device=DEV)
    cu().sage_head(indptr.to(DEV), indices.to(DEV), nd, cap, h, ip, w, bias, C, labels, x, dl, None, loss, correct, db,
                   dsrc=dsrc)
    torch.cuda.synchronize()
    gx = dx[:n_dst].float().cpu()
    want = torch.zeros(n_src, ip)
    want[:n_dst] += gx[:, :ip]
    for v in range(n_dst):
        u = indices[indptr[v]:indptr[v + 1]].long()
        if u.numel():
            want.index_add_(0, u, (gx[v, ip:] / u.numel()).expand(u.numel(), ip))
    torch.testing.assert_close(dsrc.cpu(), want, atol=1e-5, rtol=1e-3)


@pytest.mark.parametrize("ip,op,n_dst,max_deg,p", [(256, 256, 3250, 9, 0.0), (256, 256, 700, 12, 0.5),
                                                   (128, 128, 100, 0, 0.0)])
def test_sage_layer_tiles_match_torch(ip, op, n_dst, max_deg, p):
    """Hidden GraphSAGE layer as MMA tiles: forward H = dropout(relu([h_v | mean h_u] W^T + b))
    (and the aggregated rows X), backward dsrc += the aggregation's transpose of dY W,
    against fp32 torch on the same bf16 operands (dropout mask from the host mirror)."""
    from grappa_b200.sampler_gpu import new_counters

    torch.manual_seed(9)
    n_src = n_dst + 900
    cap = (n_dst + 15) // 16 * 16 + 16
    deg = torch.randint(0, max_deg + 1, (n_dst,))
    indptr = torch.zeros(n_dst + 1, dtype=torch.int32)
    indptr[1:] = torch.cumsum(deg, 0)
    indices = torch.randint(0, n_src, (int(indptr[-1]) + 1,), dtype=torch.int32)
    h = bf(torch.randn(n_src, ip, device=DEV))
    w = bf(torch.randn(op, 2 * ip, device=DEV) / math.sqrt(2 * ip))
    bias = torch.randn(op, device=DEV) * 0.1
    x = torch.zeros(cap, 2 * ip, dtype=torch.bfloat16, device=DEV)
    out = torch.full((cap, op), 3.0, dtype=torch.bfloat16, device=DEV)
    nd = torch.tensor([n_dst], dtype=torch.int32, device=DEV)
    counters = new_counters(13, DEV)
    counters[1], counters[2] = 2, 7
    cu().sage_layer_fwd(indptr.to(DEV), indices.to(DEV), nd, cap, h, ip, w, op, bias, 1, p,
                        counters if p > 0 else None, 1, x, out)
    torch.cuda.synchronize()
    hf = h.float().cpu()
    rows = []
    for v in range(n_dst):
        u = indices[indptr[v]:indptr[v + 1]].long()
        rows.append(torch.cat([hf[v], hf[u].mean(0) if u.numel() else torch.zeros(ip)]))
    xr = bf(torch.stack(rows)).float()
    torch.testing.assert_close(x[:n_dst].float().cpu(), xr, atol=1e-2, rtol=1e-2)
    want = torch.relu(xr @ w.float().cpu().t() + bias.cpu())
    if p > 0:
        mask = torch.from_numpy(_native.host().dropout_mask(13, 2, 7, 1, n_dst, op, op, p)).view(n_dst, op).float()
        want = want * mask / (1 - p)
    torch.testing.assert_close(out[:n_dst].float().cpu(), want, atol=3e-2, rtol=2e-2)
    # backward
    dy = bf(torch.randn(cap, op, device=DEV) * 0.1)
    dsrc = torch.zeros(n_src, ip, device=DEV)
    cu().sage_layer_bwd(indptr.to(DEV), indices.to(DEV), nd, cap, dy, ip, w, op, dsrc)
    torch.cuda.synchronize()
    dx = bf(dy[:n_dst].float() @ w.float()).float().cpu()
    wantd = torch.zeros(n_src, ip)
    wantd[:n_dst] += dx[:, :ip]
    for v in range(n_dst):
        u = indices[indptr[v]:indptr[v + 1]].long()
        if u.numel():
            wantd.index_add_(0, u, (dx[v, ip:] / u.numel()).expand(u.numel(), ip))
    torch.testing.assert_close(dsrc.cpu(), wantd, atol=2e-3, rtol=2e-2)
