"""Plain-PyTorch definitions of the layer math.

These are the CPU execution path (the gloo/CPU configurations train with them)
and the fp32 oracle that the sm_100a kernels are tested against.
"""
import torch

from grappa_b200 import _native


def aggregate(block, h, mode="mean", edge_weight=None, src_norm=None, dst_norm=None):
    """Aggregate source rows ``h`` [n_src, d] into [n_dst, d] over the block's edges.

    mean      1/deg_v * sum h_u               (SAGEConv 'mean'; 0 for deg 0)
    sum       sum h_u                          (GINConv 'sum')
    gcn       dnorm_v * sum snorm_u h_u        (GraphConv norm='both')
    weighted  sum w_e h_u / max(sum w_e, 1)    (PinSAGE)
    """
    u, v = block.edges()
    n_dst = block.n_dst
    msg = h[u]
    if mode == "gcn":
        msg = msg * src_norm[u].unsqueeze(1)
    elif mode == "weighted":
        msg = msg * edge_weight.unsqueeze(1)
    out = torch.zeros((n_dst, h.shape[1]), dtype=h.dtype, device=h.device).index_add_(0, v, msg)
    deg = block.in_degrees().to(h.dtype)
    if mode == "mean":
        out = out / deg.clamp(min=1).unsqueeze(1)
    elif mode == "gcn":
        dn = dst_norm if dst_norm is not None else deg.clamp(min=1).pow(-0.5)
        out = out * dn.unsqueeze(1)
    elif mode == "weighted":
        ws = torch.zeros(n_dst, dtype=h.dtype, device=h.device).index_add_(0, v, edge_weight.to(h.dtype))
        out = out / ws.clamp(min=1).unsqueeze(1)
    return out


def gcn_src_norm(block, dtype=torch.float32):
    return block.out_degrees().to(dtype).clamp(min=1).pow(-0.5)


def dropout(x, p, training, key=None, ld=None):
    """Dropout.  With ``key = (seed, epoch, step, salt)`` the keep-mask is the Philox
    mask that the GPU GEMM epilogue draws (bit-identical); otherwise torch's dropout."""
    if not training or p == 0.0:
        return x
    if key is None:
        return torch.nn.functional.dropout(x, p, True)
    seed, epoch, step, salt = key
    rows, cols = x.shape
    mask = _native.host().dropout_mask(seed, epoch, step, salt, rows, cols, ld or cols, p)
    mask = torch.from_numpy(mask).view(rows, cols).to(device=x.device, dtype=x.dtype)
    return x * mask / (1.0 - p)


def edge_softmax(block, e):
    """Softmax of edge scores e [E, H] over the in-edges of every dst node."""
    _, v = block.edges()
    n_dst = block.n_dst
    H = e.shape[1]
    emax = torch.full((n_dst, H), -float("inf"), dtype=e.dtype, device=e.device)
    emax = emax.scatter_reduce(0, v.unsqueeze(1).expand(-1, H), e, reduce="amax", include_self=True)
    ex = torch.exp(e - emax[v])
    den = torch.zeros((n_dst, H), dtype=e.dtype, device=e.device).index_add_(0, v, ex)
    return ex / den[v]
