"""One GNN layer over a full-neighbour block on the sm_100a kernels (eval mode).

Layer-wise inference (grappa_b200.infer.run_infer_xborder_by_layer; reference
t10n/infer.py:96-190) applies layer l to every node of the working graph before
layer l+1, one block of destination nodes at a time.  ``infer_layer`` is that step
for CUDA tensors: the same kernel sequence as the training engines' forward pass
(grappa_b200.engine, ``_forward`` of each engine) with dropout off and BatchNorm on
its running statistics, on buffers sized for the block.

    out = infer_layer(model, l, block, h)      # h: [n_src, in] on cuda, out: [n_dst, out] fp32
"""
import torch

from grappa_b200 import _native
from grappa_b200.engine import AGG_GCN, AGG_MEAN, AGG_SUM, AGG_WEIGHTED, GEMM_STORE_BF16, gemm_bn
from grappa_b200.models.flat import pad8


def _rows(n):
    return max(128, (int(n) + 127) // 128 * 128)


class _Ctx:
    """Per-call device state: bf16 weights, fp32 parameters, counts and the error word."""

    def __init__(self, model, device):
        self.cu = _native.cuda()
        self.dev = device
        self.model = model
        flat = model.flat.detach()
        self.f32 = flat.to(device) if flat.device != device else flat
        self.wbf = self.f32.to(torch.bfloat16)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)

    def seg(self, name, bf16=True):
        return self.model.segment(name).view(self.wbf if bf16 else self.f32)

    def count(self, n):
        return torch.tensor([int(n)], dtype=torch.int32, device=self.dev)

    def zeros(self, rows, cols, dtype=torch.bfloat16):
        return torch.zeros((rows, cols), dtype=dtype, device=self.dev)

    def gemm(self, A, B, b_mn, M_cap, M_dev, N, K, C, bias=None, act=0):
        self.cu.gemm(A, False, B, b_mn, M_cap, M_dev, N, K, None, 1, C, GEMM_STORE_BF16, bias, act, 0.0, None, 0,
                     None, 0, None, None, None, None, None, None, self.err, gemm_bn(M_cap, N, b_mn))

    def check(self):
        e = int(self.err.item())
        if e:
            raise RuntimeError(f"device error word {e:#x} in layer inference")


def _input_rows(ctx, h, n_src, ip):
    """h as bf16 rows of width ip (zero pad columns), rows rounded up to the GEMM tile."""
    x = ctx.zeros(_rows(n_src), ip)
    x[:n_src, :h.shape[1]] = h[:n_src].to(torch.bfloat16)
    return x


def _sage(ctx, layer, last, ip_, ix, n_dst, n_src, x):
    cu = ctx.cu
    ip, op = pad8(layer.in_feats), pad8(layer.out_feats)
    R = _rows(n_dst)
    X = ctx.zeros(R, 2 * ip)
    cu.aggregate(ip_, ix, None, n_dst, R, x, None, ip, AGG_MEAN, None, None, None, X, ip, 0, 0.0, 0, ctx.err)
    H = ctx.zeros(R, op)
    ctx.gemm(X, ctx.seg(layer.seg_w), False, R, ctx.count(n_dst), op, 2 * ip, H, ctx.seg(layer.seg_b, False)[0],
             0 if last else 1)
    return H[:n_dst, :layer.out_feats]


def _gcn(ctx, layer, last, ip_, ix, n_dst, n_src, x):
    cu = ctx.cu
    ip, op = pad8(layer.in_feats), pad8(layer.out_feats)
    R, S = _rows(n_dst), _rows(n_src)
    act = 0 if last else 1
    n_e = ctx.count(ix.numel())
    degs = torch.zeros(S, dtype=torch.float32, device=ctx.dev)
    snorm = torch.zeros(S, dtype=torch.float32, device=ctx.dev)
    cu.src_norm(ix, n_e, max(1, ix.numel()), ctx.count(n_src), S, degs, snorm)
    W, b = ctx.seg(layer.seg_w), ctx.seg(layer.seg_b, False)[0]
    H = ctx.zeros(R, op)
    if layer.in_feats > layer.out_feats:
        Z = ctx.zeros(S, op)
        ctx.gemm(x, W, True, S, ctx.count(n_src), op, ip, Z)
        cu.aggregate(ip_, ix, None, n_dst, R, Z, None, op, AGG_GCN, None, snorm, None, H, 0, -1, 0.0, 64, ctx.err,
                     bias=b, act=act)
    else:
        X = ctx.zeros(R, ip)
        cu.aggregate(ip_, ix, None, n_dst, R, x, None, ip, AGG_GCN, None, snorm, None, X, 0, -1, 0.0, 64, ctx.err)
        ctx.gemm(X, W, True, R, ctx.count(n_dst), op, ip, H, b, act)
    return H[:n_dst, :layer.out_feats]


def _gin(ctx, model, l, ip_, ix, n_dst, n_src, x):
    cu = ctx.cu
    conv = model.layers[l]
    mlp = conv.apply_func
    lin0, lin1 = mlp.linears
    ip, hp, op = pad8(lin0.in_features), pad8(lin0.out_features), pad8(lin1.out_features)
    R = _rows(n_dst)
    n = ctx.count(n_dst)
    X = ctx.zeros(R, ip)
    cu.aggregate(ip_, ix, None, n_dst, R, x, None, ip, AGG_SUM, None, None, None, X, 0, -1,
                 1.0 + float(conv.eps.item()), 64, ctx.err)

    def bn(t, dim, seg, mod, y):
        gb = ctx.seg(seg, False)
        rm, rv = mod.running_mean.to(ctx.dev), mod.running_var.to(ctx.dev)
        sums = torch.zeros(2 * dim, dtype=torch.float32, device=ctx.dev)
        cu.batchnorm_fwd(t, dim, n, R, sums, gb[0], gb[1], rm, rv, None, mod.momentum, mod.eps, False, 1, y)

    T0, U = ctx.zeros(R, hp), ctx.zeros(R, hp)
    ctx.gemm(X, ctx.seg(mlp.seg_w0), False, R, n, hp, ip, T0)
    bn(T0, hp, mlp.seg_bn, mlp.batch_norm, U)
    T1, H = ctx.zeros(R, op), ctx.zeros(R, op)
    ctx.gemm(U, ctx.seg(mlp.seg_w1), False, R, n, op, hp, T1)
    bn(T1, op, f"batch_norms.{l}", model.batch_norms[l], H)
    return H[:n_dst, :lin1.out_features]


def _gat(ctx, layer, last, ip_, ix, n_dst, n_src, x):
    cu = ctx.cu
    Hh, F = layer.num_heads, layer.out_feats
    HF = Hh * F
    ip, hfp = pad8(layer.in_feats), pad8(HF)
    R, S = _rows(n_dst), _rows(n_src)
    f32 = dict(dtype=torch.float32, device=ctx.dev)
    Z = ctx.zeros(S, hfp)
    ctx.gemm(x, ctx.seg(layer.seg_w), False, S, ctx.count(n_src), HF, ip, Z)
    A = ctx.seg(layer.seg_a, False)
    el, er = torch.zeros(S * Hh, **f32), torch.zeros(R * Hh, **f32)
    smax, ssum = torch.zeros(R * Hh, **f32), torch.zeros(R * Hh, **f32)
    out = ctx.zeros(R, pad8(F) if last else hfp)
    args = (ip_, ix, ctx.count(n_dst), R, ctx.count(n_src), S, Hh, F, Z, A[0], A[1], el, er, smax, ssum, 0.2)
    cu.gat_scores(*args)
    cu.gat_fwd(*args, ctx.seg(layer.seg_b, False)[0], last, 0 if last else 1, 0.0, None, 0, out)
    return out[:n_dst, :F] if last else out[:n_dst, :HF]


def _pinsage(ctx, layer, last, ip_, ix, n_dst, n_src, x, w):
    cu = ctx.cu
    ip, hid, op = pad8(layer.input_dims), layer.hidden_dims, pad8(layer.output_dims)
    kw = pad8(hid + layer.input_dims)
    R, S = _rows(n_dst), _rows(n_src)
    N = ctx.zeros(S, hid)
    ctx.gemm(x, ctx.seg(layer.seg_q), False, S, ctx.count(n_src), hid, ip, N, ctx.seg(layer.seg_qb, False)[0], 1)
    X = ctx.zeros(R, kw)
    cu.aggregate(ip_, ix, None, n_dst, R, N, None, hid, AGG_WEIGHTED, w, None, None, X, 0, -1, 0.0, 64, ctx.err)
    X[:n_dst, hid:hid + layer.input_dims] = x[:n_dst, :layer.input_dims]
    Z, H = ctx.zeros(R, op), ctx.zeros(R, op)
    ctx.gemm(X, ctx.seg(layer.seg_w), False, R, ctx.count(n_dst), op, kw, Z, ctx.seg(layer.seg_wb, False)[0], 1)
    norms = torch.zeros(R, dtype=torch.float32, device=ctx.dev)
    cu.l2norm_fwd(Z, op, ctx.count(n_dst), R, H, norms)
    return H[:n_dst, :layer.output_dims]


def infer_layer(model, layer_i, block, h):
    """Layer ``layer_i`` of ``model`` (and its inter-layer activation) on ``block`` for the
    source rows ``h`` (a CUDA tensor); returns the fp32 destination rows."""
    dev = h.device
    if dev.type != "cuda":
        raise ValueError("infer_layer runs on CUDA tensors")
    ctx = _Ctx(model, dev)
    n_dst, n_src = block.num_dst_nodes(), block.num_src_nodes()
    ip_ = block.indptr.to(dev, torch.int32).contiguous()
    ix = block.indices.to(dev, torch.int32).contiguous()
    last = layer_i == len(model.layers) - 1
    layer = model.layers[layer_i]
    name = model.name
    if name == "sage":
        out = _sage(ctx, layer, last, ip_, ix, n_dst, n_src, _input_rows(ctx, h, n_src, pad8(layer.in_feats)))
    elif name == "gcn":
        out = _gcn(ctx, layer, last, ip_, ix, n_dst, n_src, _input_rows(ctx, h, n_src, pad8(layer.in_feats)))
    elif name == "gin":
        ip = pad8(layer.apply_func.linears[0].in_features)
        out = _gin(ctx, model, layer_i, ip_, ix, n_dst, n_src, _input_rows(ctx, h, n_src, ip))
    elif name == "gat":
        out = _gat(ctx, layer, last, ip_, ix, n_dst, n_src, _input_rows(ctx, h, n_src, pad8(layer.in_feats)))
    elif name == "pinsage":
        w = block.edata.get("weights")
        w = (torch.ones(block.num_edges(), dtype=torch.float32, device=dev) if w is None
             else w.to(dev, torch.float32).contiguous())
        out = _pinsage(ctx, layer, last, ip_, ix, n_dst, n_src,
                       _input_rows(ctx, h, n_src, pad8(layer.input_dims)), w)
    else:
        raise ValueError(f"{name} is not supported")
    ctx.check()
    return out.float()


def _layer_in_width(model, layer_i):
    layer = model.layers[layer_i]
    if model.name == "gin":
        return pad8(layer.apply_func.linears[0].in_features)
    if model.name == "pinsage":
        return pad8(layer.input_dims)
    return pad8(layer.in_feats)


class ExactInference:
    """Exact full-neighbour layer-wise inference of every own node on the GPU, across
    partitions (reference: run_infer_xborder_by_layer, t10n/infer.py:89-198).

    Each rank holds the complete in-edge CSR of its own nodes, so the block of a layer
    is local: destinations = own nodes, sources = own nodes plus ``own.ext_src`` (the
    sorted external in-neighbours).  Per layer every rank (1) writes its own nodes'
    layer input into a peer-mapped table, (2) after a barrier pulls the rows of its
    external sources straight from their owners' tables over NVLink (pull_rows, one
    kernel: the global id says which rank and row to read, so no id exchange is
    needed), (3) runs the layer on the sm_100a kernels (``infer_layer``).  The last
    layer's logits give the accuracy on the own nodes of each mask, summed over ranks.
    Collective: every rank calls ``accuracy`` with the same masks."""

    def __init__(self, model, own, comm=None):
        from grappa_b200.block import Block
        from grappa_b200.parallel.comm import Comm, PeerBuffer

        self.model, self.own = model, own
        self.comm = comm if comm is not None else Comm()
        dev = own.indices.device
        self.device = dev
        r = own.rank
        lo, hi = own.prefix[r], own.prefix[r + 1]
        n_own = hi - lo
        ext = own.ext_src.to(dev, torch.int64)
        self.n_own, self.n_ext = n_own, int(ext.numel())
        g = own.indices.to(torch.int64)
        inside = (g >= lo) & (g < hi)
        loc = torch.where(inside, g - lo, n_own + torch.searchsorted(ext, g))
        src_ids = torch.cat([torch.arange(lo, hi, device=dev, dtype=torch.int64), ext])
        self.block = Block(own.indptr, loc.to(torch.int32), src_ids, n_own, n_own + self.n_ext)
        self.ext_ids = ext
        self.n_ext_dev = torch.tensor([self.n_ext], dtype=torch.int32, device=dev)
        self.width = max(_layer_in_width(model, i) for i in range(len(model.layers)))
        self.prefix_dev = torch.tensor(own.prefix, dtype=torch.int64, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        # this rank's layer-input rows, readable by every rank
        self.table = PeerBuffer(self.comm, max(256, n_own * self.width * 2))
        self.T = self.table.tensor(torch.bfloat16, [max(1, n_own), self.width])

    def _sync(self):
        torch.cuda.synchronize(self.device)
        self.comm.barrier()

    def logits(self):
        """fp32 [n_own, n_classes] logits of the own nodes with full neighbourhoods."""
        model, own = self.model, self.own
        d0 = own.feat.shape[1]
        self.T.zero_()
        self.T[:, :d0].copy_(own.feat)
        h = None
        with torch.no_grad():
            for l in range(len(model.layers)):
                w = _layer_in_width(model, l)
                X = torch.zeros((self.n_own + self.n_ext, w), dtype=torch.bfloat16, device=self.device)
                X[: self.n_own].copy_(self.T[:, :w])
                self._sync()  # every rank's table holds layer l's input
                if self.n_ext:
                    tables = [self.table.ptrs[p] for p in range(own.world)]
                    _native.cuda().pull_rows(tables, self.width, 2, w * 2, self.ext_ids, self.n_ext_dev, 0,
                                             self.prefix_dev, X.data_ptr(), w, self.n_own, self.n_ext, self.err)
                self._sync()  # every rank has read the tables: they may be overwritten
                h = infer_layer(model, l, self.block, X)
                if l + 1 < len(model.layers):
                    self.T.zero_()
                    self.T[:, :h.shape[1]].copy_(h.to(torch.bfloat16))
        if int(self.err.item()):
            raise RuntimeError(f"device error word {int(self.err.item()):#x} in exact inference")
        return h

    def accuracy(self, masks):
        """Accuracy on the own nodes selected by each mask, over all ranks."""
        logits = self.logits()
        pred = torch.argmax(logits, dim=1)
        ok = pred == self.own.label.to(pred.device).long()
        vals = []
        for m in masks:
            m = m.to(pred.device).bool()
            vals += [float(ok[m].sum()), float(m.sum())]
        if self.comm.world > 1:
            vals = self.comm.all_reduce_sum(vals)
        return [vals[2 * i] / max(vals[2 * i + 1], 1.0) for i in range(len(masks))]

    def close(self):
        self.table.close()
