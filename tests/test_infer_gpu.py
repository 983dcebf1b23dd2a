"""Layer-wise inference on the sm_100a kernels against the PyTorch layers (fp32 oracle)."""
import pytest
import torch

from grappa_b200.block import Block
from grappa_b200.infer import apply_layer
from grappa_b200.models import get_model

pytestmark = pytest.mark.gpu


def _block(n_dst, n_src, max_deg, seed, weights=False):
    g = torch.Generator().manual_seed(seed)
    deg = torch.randint(0, max_deg + 1, (n_dst,), generator=g)
    indptr = torch.zeros(n_dst + 1, dtype=torch.int64)
    indptr[1:] = torch.cumsum(deg, 0)
    indices = torch.randint(0, n_src, (int(indptr[-1]),), generator=g, dtype=torch.int64)
    w = torch.rand(indices.numel(), generator=g) * 3 if weights else None
    return Block(indptr, indices, torch.arange(n_src), n_dst, n_src, edge_weight=w)


@pytest.mark.parametrize("name", ["sage", "gcn", "gin", "gat", "pinsage"])
def test_infer_layer_matches_torch(name):
    torch.manual_seed(3)
    in_dim, hid, n_cls = 40, 64, 10
    model = get_model(name, in_dim, n_cls, num_hidden=hid, num_layers=2, dropout=0.0, n_heads=4)
    if name == "gin":
        for bn in list(model.batch_norms) + [layer.apply_func.batch_norm for layer in model.layers]:
            bn.running_mean.uniform_(-0.5, 0.5)
            bn.running_var.uniform_(0.5, 2.0)
    model.eval()
    dev = torch.device("cuda", 0)
    blk = _block(300, 1000, 12, 5, weights=(name == "pinsage"))
    h = torch.randn(1000, in_dim)
    with torch.no_grad():
        ref0 = apply_layer(model, 0, blk, h)
        got0 = apply_layer(model, 0, blk.to(dev), h.to(dev))
        blk1 = _block(120, 300, 8, 6, weights=(name == "pinsage"))
        ref1 = apply_layer(model, 1, blk1, ref0)
        got1 = apply_layer(model, 1, blk1.to(dev), ref0.to(dev))
    for ref, got in ((ref0, got0), (ref1, got1)):
        assert got.shape == ref.shape
        err = (got.cpu() - ref).abs().max().item() / max(1e-3, ref.abs().max().item())
        assert err < 3e-2, (name, err)
