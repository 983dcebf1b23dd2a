"""Block (message-flow graph) of one GNN layer.

A block has ``n_dst`` destination nodes and ``n_src`` source nodes; the first
``n_dst`` source nodes are the destination nodes themselves (DGL's ``to_block``
convention used by the reference, t10n/dgl_dsg/compliant.py:32-49).  Edges are
stored in CSR form by destination: the in-edges of dst ``v`` are
``indices[indptr[v]:indptr[v+1]]`` (local source indices).

``srcdata[NID]`` / ``dstdata[NID]`` give the graph ids of the nodes, as in DGL.
"""
import torch

NID = "_ID"


class Block:
    def __init__(self, indptr, indices, src_nid, n_dst, n_src=None, src_sampled=None, edge_weight=None):
        self.indptr = indptr
        self.indices = indices
        self.n_dst = int(n_dst)
        self.n_src = int(n_src if n_src is not None else src_nid.shape[0])
        self.srcdata = {NID: src_nid}
        self.dstdata = {NID: src_nid[: self.n_dst]}
        self.src_sampled = src_sampled
        self.edata = {}
        if edge_weight is not None:
            self.edata["weights"] = edge_weight

    # DGL-style accessors
    def num_dst_nodes(self):
        return self.n_dst

    def num_src_nodes(self):
        return self.n_src

    number_of_dst_nodes = num_dst_nodes
    number_of_src_nodes = num_src_nodes

    def num_edges(self):
        return int(self.indices.shape[0])

    def in_degrees(self):
        return self.indptr[1:] - self.indptr[:-1]

    def out_degrees(self):
        return torch.bincount(self.indices.long(), minlength=self.n_src)

    def dst_of_edges(self):
        deg = self.in_degrees().long()
        return torch.repeat_interleave(torch.arange(self.n_dst, device=deg.device), deg)

    def edges(self):
        """(u, v) local ids of every edge (u = src index, v = dst index)."""
        return self.indices.long(), self.dst_of_edges()

    @property
    def device(self):
        return self.indices.device

    def to(self, device):
        ew = self.edata.get("weights")
        return Block(self.indptr.to(device), self.indices.to(device), self.srcdata[NID].to(device), self.n_dst,
                     self.n_src, None if self.src_sampled is None else self.src_sampled.to(device),
                     None if ew is None else ew.to(device))

    def __repr__(self):
        return f"Block(num_src_nodes={self.n_src}, num_dst_nodes={self.n_dst}, num_edges={self.num_edges()})"


def blocks_from_host(batch_blocks):
    """Blocks (input layer first) from the host sampler's per-hop dicts (seed hop first)."""
    out = []
    for d in reversed(batch_blocks):
        out.append(
            Block(
                torch.from_numpy(d["indptr"]),
                torch.from_numpy(d["indices"]),
                torch.from_numpy(d["src_nid"]),
                d["n_dst"],
                d["n_src"],
                torch.from_numpy(d["src_sampled"]),
            )
        )
    return out
