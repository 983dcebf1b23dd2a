"""GNN models of the framework: GCN, GraphSAGE, GAT, GIN and PinSAGE.

Constructors, forward structure and state_dict keys follow the reference's
experiments/grappa/train/{gcn,graphsage,gat,gin,pinsage}.py (DGL 1.x modules), so
checkpoints keep the reference's format.  ``forward(blocks, x)`` is the PyTorch
path; ``grappa_b200.engine`` runs the same parameters on the sm_100a kernels.
"""
from contextlib import contextmanager

import torch
import torch.nn.functional as F
from torch import nn

from grappa_b200.models.flat import FlatModule, pad8
from grappa_b200.models.layers import GATConv, GINConv, GINMLP, GraphConv, SAGEConv, WeightedSAGEConv
from grappa_b200.ops import ref

__all__ = ["SAGE", "GCN", "GAT", "GIN", "PinSAGE", "get_model"]


class _Base(FlatModule):
    """Shared pieces: dropout keyed for GPU/CPU mask parity and a DDP-style join()."""

    dropout_key = None  # (seed, epoch, step): when set, dropout uses the GPU's Philox masks

    def _drop(self, h, salt, ld):
        if not self.training or self.dropout_p == 0.0:
            return h
        key = self.dropout_key
        if key is None:
            return F.dropout(h, self.dropout_p, True)
        return ref.dropout(h, self.dropout_p, True, key=(key[0], key[1], key[2], salt), ld=ld)

    @contextmanager
    def join(self):
        """dummy join for standalone"""
        yield


class SAGE(_Base):
    """GraphSAGE, mean aggregator (reference experiments/grappa/train/graphsage.py:11-42)."""

    def __init__(self, in_feats, n_hidden, n_classes, n_layers, activation=F.relu, dropout=0.5):
        super().__init__()
        self.name = "sage"
        self.n_layers, self.n_hidden, self.n_classes = n_layers, n_hidden, n_classes
        self.in_feats = in_feats
        dims = [in_feats] + [n_hidden] * (n_layers - 1) + [n_classes]
        self.layers = nn.ModuleList(
            [SAGEConv(self, f"layers.{i}", dims[i], dims[i + 1]) for i in range(n_layers)]
        )
        self.dropout = nn.Dropout(dropout)
        self.dropout_p = float(dropout)
        self.activation = activation
        self.finalize(self.reset_parameters)

    def reset_parameters(self):
        for layer in self.layers:
            layer.reset_parameters()

    def forward(self, blocks, x):
        h = x
        for l, (layer, block) in enumerate(zip(self.layers, blocks)):
            h = layer(block, h)
            if l != len(self.layers) - 1:
                h = self.activation(h)
                h = self._drop(h, l, pad8(layer.out_feats))
        return h


class GCN(_Base):
    """GCN with GraphConv(norm='both') (reference experiments/grappa/train/gcn.py:15-64)."""

    def __init__(self, in_feats, n_hidden, n_classes, n_layers, activation=F.relu, dropout=0.5):
        super().__init__()
        self.name = "gcn"
        self.n_layers, self.n_hidden, self.n_classes = n_layers, n_hidden, n_classes
        self.in_feats = in_feats
        dims = [in_feats] + [n_hidden] * (n_layers - 1) + [n_classes]
        self.layers = nn.ModuleList(
            [GraphConv(self, f"layers.{i}", dims[i], dims[i + 1], activation if i < n_layers - 1 else None)
             for i in range(n_layers)]
        )
        self.dropout = nn.Dropout(p=dropout)
        self.dropout_p = float(dropout)
        self.activation = activation
        self.finalize(self.reset_parameters)

    def reset_parameters(self):
        for layer in self.layers:
            layer.reset_parameters()

    def forward(self, blocks, features):
        h = features
        for i, layer in enumerate(self.layers):
            if i != 0:
                h = self._drop(h, i - 1, pad8(self.layers[i - 1].out_feats))
            g = blocks[i] if isinstance(blocks, (list, tuple)) else blocks
            h = layer(g, h)
        return h


class GAT(_Base):
    """GAT (reference experiments/grappa/train/gat.py:12-60): hidden layers flatten the
    heads, then ReLU and dropout; the last layer averages the heads."""

    def __init__(self, in_feats, n_hidden, n_classes, n_heads, n_layers, activation=F.relu, dropout=0.5):
        super().__init__()
        self.name = "gat"
        self.n_layers, self.n_hidden, self.n_classes, self.n_heads = n_layers, n_hidden, n_classes, n_heads
        self.in_feats = in_feats
        ins = [in_feats] + [n_hidden * n_heads] * (n_layers - 1)
        outs = [n_hidden] * (n_layers - 1) + [n_classes]
        self.layers = nn.ModuleList(
            [GATConv(self, f"layers.{i}", ins[i], outs[i], n_heads) for i in range(n_layers)]
        )
        self.dropout = nn.Dropout(dropout)
        self.dropout_p = float(dropout)
        self.activation = activation
        self.finalize(self.reset_parameters)

    def reset_parameters(self):
        for layer in self.layers:
            layer.reset_parameters()

    def forward(self, blocks, x):
        h = x
        for l, (layer, block) in enumerate(zip(self.layers, blocks)):
            h_dst = h[: block.num_dst_nodes()]
            if l < len(self.layers) - 1:
                h = layer(block, (h, h_dst)).flatten(1)
                h = self.activation(h)
                h = self._drop(h, l, pad8(layer.out_feats * layer.num_heads))
            else:
                h = layer(block, (h, h_dst)).mean(1)
        return h


class GIN(_Base):
    """GIN with 2-layer MLPs and sum aggregation; BatchNorm + ReLU after every layer
    (reference experiments/grappa/train/gin.py:40-124)."""

    def __init__(self, input_dim, hidden_dim, output_dim, num_layers=2):
        super().__init__()
        self.name = "gin"
        self.n_hidden, self.n_classes, self.n_layers = hidden_dim, output_dim, num_layers
        self.in_feats = input_dim
        self.dropout_p = 0.0
        self.layers = nn.ModuleList()
        self.batch_norms = nn.ModuleList()
        # layer i's segments (its MLP, then its output BatchNorm) are contiguous in the
        # flat buffer, so that a layer's gradient is one bucket of the all-reduce
        for layer in range(num_layers):
            last = layer == num_layers - 1
            mlp = GINMLP(self, f"layers.{layer}.mlp", input_dim if layer == 0 else hidden_dim, hidden_dim,
                         output_dim if last else hidden_dim)
            self.layers.append(GINConv(mlp, 0.0))
            bn = nn.BatchNorm1d(output_dim if last else hidden_dim)
            self.batch_norms.append(bn)
            self.add_segment(f"batch_norms.{layer}", 2, bn.num_features)
            self.bind(bn, "weight", f"batch_norms.{layer}", 0, slice(0, bn.num_features))
            self.bind(bn, "bias", f"batch_norms.{layer}", 1, slice(0, bn.num_features))
        self.finalize(self.reset_parameters)

    def reset_parameters(self):
        for layer in self.layers:
            layer.apply_func.reset_parameters()
        for bn in self.batch_norms:
            bn.weight.fill_(1.0)
            bn.bias.zero_()
            bn.reset_running_stats()

    def forward(self, blocks, h):
        for i, layer in enumerate(self.layers):
            g = blocks[i] if isinstance(blocks, (list, tuple)) else blocks
            h = layer(g, h)
            h = self.batch_norms[i](h)
            h = F.relu(h)
        return h


class PinSAGE(_Base):
    """PinSAGE with weighted (random-walk visit count) aggregation
    (reference experiments/grappa/train/pinsage.py:55-84)."""

    def __init__(self, in_feats, n_hidden, n_classes, n_layers, activation=F.relu, dropout=0.5):
        super().__init__()
        self.name = "pinsage"
        self.n_layers, self.n_hidden, self.n_classes = n_layers, n_hidden, n_classes
        self.in_feats = in_feats
        self.dropout_p = float(dropout)
        self.layers = nn.ModuleList()
        self.layers.append(WeightedSAGEConv(self, "layers.0", in_feats, n_hidden, n_hidden, dropout, activation))
        for i in range(1, n_layers - 1):
            self.layers.append(WeightedSAGEConv(self, f"layers.{i}", n_hidden, n_hidden, n_hidden, dropout, activation))
        self.layers.append(WeightedSAGEConv(self, f"layers.{n_layers - 1}", n_hidden, n_hidden, n_classes, dropout,
                                            activation))
        self.finalize(self.reset_parameters)

    def reset_parameters(self):
        for layer in self.layers:
            layer.reset_parameters()

    def forward(self, blocks, x):
        h = x
        for layer, block in zip(self.layers, blocks):
            h_dst = h[: block.num_dst_nodes()]
            w = block.edata.get("weights")
            if w is None:
                w = torch.ones(block.num_edges(), dtype=torch.float32, device=h.device)
            h = layer(block, (h, h_dst), w)
        return h


def get_model(name, n_feat_dim, n_class, num_hidden=128, num_layers=3, dropout=0.5, n_heads=4):
    """Model factory with the reference's argument mapping
    (experiments/grappa/train/t10n_train.py:52-101)."""
    if name == "sage":
        return SAGE(n_feat_dim, num_hidden, n_class, num_layers, F.relu, dropout)
    if name == "gat":
        return GAT(n_feat_dim, num_hidden, n_class, n_heads, num_layers, F.relu, dropout)
    if name == "gcn":
        return GCN(n_feat_dim, num_hidden, n_class, num_layers, F.relu, dropout)
    if name == "gin":
        return GIN(n_feat_dim, num_hidden, n_class, num_layers)
    if name == "pinsage":
        return PinSAGE(n_feat_dim, num_hidden, n_class, num_layers, F.relu, dropout)
    raise ValueError(f"unknown model {name}")
