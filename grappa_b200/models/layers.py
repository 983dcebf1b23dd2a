"""Graph convolution layers with DGL 1.x parameter names and math.

Each layer declares its parameters as segments of its model's flat buffer
(``grappa_b200.models.flat``).  ``forward`` is the PyTorch path (CPU execution and
the fp32 oracle); on CUDA the same parameters are driven by the sm_100a engine
(``grappa_b200.engine``), and calling the torch path on CUDA tensors raises
instead of silently running library kernels.

Reference layers (mpi-dsg/grappa uses DGL's modules):
  SAGEConv 'mean'    experiments/grappa/train/graphsage.py:11-42
  GraphConv 'both'   experiments/grappa/train/gcn.py:15-64
  GATConv            experiments/grappa/train/gat.py:12-60
  GINConv 'sum'      experiments/grappa/train/gin.py:20-124
  WeightedSAGEConv   experiments/grappa/train/pinsage.py:11-52
"""
import math

import torch
import torch.nn.functional as F
from torch import nn

from grappa_b200.models.flat import pad8, xavier_normal_, xavier_uniform_
from grappa_b200.ops import ref

RELU_GAIN = math.sqrt(2.0)


def _cpu_only(x):
    if isinstance(x, tuple):
        x = x[0]
    if x.is_cuda:
        raise RuntimeError(
            "the torch layer path runs on CPU tensors; CUDA training and inference go through "
            "grappa_b200.engine (sm_100a kernels)"
        )


class SAGEConv(nn.Module):
    """out = fc_self(h_dst) + fc_neigh(mean_{u in N(v)} h_u) + bias.

    Flat layout: segment W = [pad8(out), 2*pad8(in)] holding [fc_self | fc_neigh]
    (the concatenated operand of one GEMM), segment b = [1, pad8(out)]."""

    def __init__(self, owner, name, in_feats, out_feats):
        super().__init__()
        self.in_feats, self.out_feats = in_feats, out_feats
        self.fc_self = nn.Linear(in_feats, out_feats, bias=False)
        self.fc_neigh = nn.Linear(in_feats, out_feats, bias=False)
        self.bias = nn.Parameter(torch.zeros(out_feats))
        ip = pad8(in_feats)
        self.seg_w = f"{name}.W"
        self.seg_b = f"{name}.b"
        owner.add_segment(self.seg_w, pad8(out_feats), 2 * ip)
        owner.add_segment(self.seg_b, 1, out_feats)
        owner.bind(self.fc_self, "weight", self.seg_w, slice(0, out_feats), slice(0, in_feats))
        owner.bind(self.fc_neigh, "weight", self.seg_w, slice(0, out_feats), slice(ip, ip + in_feats))
        owner.bind(self, "bias", self.seg_b, 0, slice(0, out_feats))

    def reset_parameters(self):
        xavier_uniform_(self.fc_self.weight, RELU_GAIN)
        xavier_uniform_(self.fc_neigh.weight, RELU_GAIN)
        self.bias.zero_()

    def forward(self, block, h):
        _cpu_only(h)
        if isinstance(h, tuple):
            h = h[0]
        h_dst = h[: block.n_dst]
        agg = ref.aggregate(block, h, "mean")
        return h_dst @ self.fc_self.weight.t() + agg @ self.fc_neigh.weight.t() + self.bias


class GraphConv(nn.Module):
    """DGL GraphConv(norm='both'): D_dst^-1/2 A D_src^-1/2 h W + b, optional activation.

    Flat layout: segment W = [pad8(in), pad8(out)] (weight is [in, out] as in DGL)."""

    def __init__(self, owner, name, in_feats, out_feats, activation=None):
        super().__init__()
        self.in_feats, self.out_feats = in_feats, out_feats
        self.weight = nn.Parameter(torch.zeros(in_feats, out_feats))
        self.bias = nn.Parameter(torch.zeros(out_feats))
        self.activation = activation
        self.seg_w = f"{name}.W"
        self.seg_b = f"{name}.b"
        owner.add_segment(self.seg_w, pad8(in_feats), out_feats)
        owner.add_segment(self.seg_b, 1, out_feats)
        owner.bind(self, "weight", self.seg_w, slice(0, in_feats), slice(0, out_feats))
        owner.bind(self, "bias", self.seg_b, 0, slice(0, out_feats))

    def reset_parameters(self):
        xavier_uniform_(self.weight.t(), 1.0)
        self.bias.zero_()

    def forward(self, block, h):
        _cpu_only(h)
        snorm = ref.gcn_src_norm(block, h.dtype)
        if self.in_feats > self.out_feats:
            rst = ref.aggregate(block, h @ self.weight, "gcn", src_norm=snorm)
        else:
            rst = ref.aggregate(block, h, "gcn", src_norm=snorm) @ self.weight
        rst = rst + self.bias
        if self.activation is not None:
            rst = self.activation(rst)
        return rst


class GATConv(nn.Module):
    """DGL GATConv: z = fc(h); e_uv = LeakyReLU(a_l.z_u + a_r.z_v, 0.2);
    alpha = softmax over in-edges; out_v = sum alpha_uv z_u + bias  ->  [n_dst, H, F].

    Flat layout: fc W = [pad8(H*F), pad8(in)], attention A = [2, H*F] (rows attn_l,
    attn_r), bias b = [1, H*F]."""

    def __init__(self, owner, name, in_feats, out_feats, num_heads, negative_slope=0.2):
        super().__init__()
        self.in_feats, self.out_feats, self.num_heads = in_feats, out_feats, num_heads
        self.negative_slope = negative_slope
        hf = out_feats * num_heads
        self.fc = nn.Linear(in_feats, hf, bias=False)
        self.attn_l = nn.Parameter(torch.zeros(1, num_heads, out_feats))
        self.attn_r = nn.Parameter(torch.zeros(1, num_heads, out_feats))
        self.bias = nn.Parameter(torch.zeros(hf))
        self.register_buffer("res_fc", None)
        self.seg_w, self.seg_a, self.seg_b = f"{name}.W", f"{name}.A", f"{name}.b"
        owner.add_segment(self.seg_w, pad8(hf), in_feats)
        owner.add_segment(self.seg_a, 2, hf)
        owner.add_segment(self.seg_b, 1, hf)
        owner.bind(self.fc, "weight", self.seg_w, slice(0, hf), slice(0, in_feats))
        owner.bind(self, "attn_l", self.seg_a, slice(0, 1), slice(0, hf), shape=(1, num_heads, out_feats))
        owner.bind(self, "attn_r", self.seg_a, slice(1, 2), slice(0, hf), shape=(1, num_heads, out_feats))
        owner.bind(self, "bias", self.seg_b, 0, slice(0, hf))

    def reset_parameters(self):
        xavier_normal_(self.fc.weight, RELU_GAIN)
        H, Fo = self.num_heads, self.out_feats
        # torch's fan computation for a [1, H, F] tensor: fan_in = H*F, fan_out = F
        std = RELU_GAIN * math.sqrt(2.0 / (H * Fo + Fo))
        for a in (self.attn_l, self.attn_r):
            a.normal_(0.0, std)
        self.bias.zero_()

    def forward(self, block, h):
        _cpu_only(h)
        if isinstance(h, tuple):
            h = h[0]
        H, Fo = self.num_heads, self.out_feats
        z = (h @ self.fc.weight.t()).view(-1, H, Fo)
        el = (z * self.attn_l).sum(-1)
        er = (z[: block.n_dst] * self.attn_r).sum(-1)
        u, v = block.edges()
        e = F.leaky_relu(el[u] + er[v], self.negative_slope)
        a = ref.edge_softmax(block, e)
        out = torch.zeros((block.n_dst, H, Fo), dtype=z.dtype).index_add_(0, v, z[u] * a.unsqueeze(-1))
        return out + self.bias.view(1, H, Fo)


class GINMLP(nn.Module):
    """Linear(no bias) -> BatchNorm1d -> ReLU -> Linear(no bias) (reference gin.py:22-37)."""

    def __init__(self, owner, name, input_dim, hidden_dim, output_dim):
        super().__init__()
        self.linears = nn.ModuleList([nn.Linear(input_dim, hidden_dim, bias=False),
                                      nn.Linear(hidden_dim, output_dim, bias=False)])
        self.batch_norm = nn.BatchNorm1d(hidden_dim)
        self.seg_w0, self.seg_w1 = f"{name}.W0", f"{name}.W1"
        owner.add_segment(self.seg_w0, pad8(hidden_dim), input_dim)
        owner.add_segment(self.seg_w1, pad8(output_dim), hidden_dim)
        owner.bind(self.linears[0], "weight", self.seg_w0, slice(0, hidden_dim), slice(0, input_dim))
        owner.bind(self.linears[1], "weight", self.seg_w1, slice(0, output_dim), slice(0, hidden_dim))
        self.seg_bn = f"{name}.bn"
        owner.add_segment(self.seg_bn, 2, hidden_dim)
        owner.bind(self.batch_norm, "weight", self.seg_bn, 0, slice(0, hidden_dim))
        owner.bind(self.batch_norm, "bias", self.seg_bn, 1, slice(0, hidden_dim))

    def reset_parameters(self):
        for lin in self.linears:
            bound = 1.0 / math.sqrt(lin.weight.shape[1])
            lin.weight.uniform_(-bound, bound)
        self.batch_norm.weight.fill_(1.0)
        self.batch_norm.bias.zero_()
        self.batch_norm.reset_running_stats()

    def forward(self, x):
        return self.linears[1](F.relu(self.batch_norm(self.linears[0](x))))


class GINConv(nn.Module):
    """DGL GINConv(apply_func, 'sum', learn_eps=False): apply_func((1+eps) h_v + sum h_u)."""

    def __init__(self, apply_func, init_eps=0.0):
        super().__init__()
        self.apply_func = apply_func
        self.register_buffer("eps", torch.tensor([float(init_eps)]))

    def forward(self, block, h):
        _cpu_only(h)
        if isinstance(h, tuple):
            h = h[0]
        rst = (1.0 + self.eps) * h[: block.n_dst] + ref.aggregate(block, h, "sum")
        return self.apply_func(rst)


class WeightedSAGEConv(nn.Module):
    """PinSAGE layer (reference pinsage.py:11-52):
    n = act(Q(drop(h_src))); n_v = sum w n_u / max(sum w, 1);
    z = act(W(drop([n_v, h_dst]))); z = z / ||z|| (norm 0 -> 1)."""

    def __init__(self, owner, name, input_dims, hidden_dims, output_dims, dropout, act):
        super().__init__()
        self.act = act
        self.Q = nn.Linear(input_dims, hidden_dims)
        self.W = nn.Linear(input_dims + hidden_dims, output_dims)
        self.dropout = nn.Dropout(dropout)
        self.input_dims, self.hidden_dims, self.output_dims = input_dims, hidden_dims, output_dims
        self.seg_q, self.seg_qb = f"{name}.Q", f"{name}.Qb"
        self.seg_w, self.seg_wb = f"{name}.W", f"{name}.Wb"
        owner.add_segment(self.seg_q, pad8(hidden_dims), input_dims)
        owner.add_segment(self.seg_qb, 1, hidden_dims)
        # W acts on [n_v | h_dst] laid out as hidden columns then input columns
        owner.add_segment(self.seg_w, pad8(output_dims), hidden_dims + input_dims)
        owner.add_segment(self.seg_wb, 1, output_dims)
        owner.bind(self.Q, "weight", self.seg_q, slice(0, hidden_dims), slice(0, input_dims))
        owner.bind(self.Q, "bias", self.seg_qb, 0, slice(0, hidden_dims))
        owner.bind(self.W, "weight", self.seg_w, slice(0, output_dims), slice(0, hidden_dims + input_dims))
        owner.bind(self.W, "bias", self.seg_wb, 0, slice(0, output_dims))

    def reset_parameters(self):
        xavier_uniform_(self.Q.weight, RELU_GAIN)
        xavier_uniform_(self.W.weight, RELU_GAIN)
        self.Q.bias.zero_()
        self.W.bias.zero_()

    def forward(self, block, h, weights):
        _cpu_only(h)
        h_src, h_dst = h if isinstance(h, tuple) else (h, h[: block.n_dst])
        n = self.act(self.Q(self.dropout(h_src)))
        nv = ref.aggregate(block, n, "weighted", edge_weight=weights.float())
        z = self.act(self.W(self.dropout(torch.cat([nv, h_dst], 1))))
        zn = z.norm(2, 1, keepdim=True)
        zn = torch.where(zn == 0, torch.ones_like(zn), zn)
        return z / zn
