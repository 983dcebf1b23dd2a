"""DGL-free counterparts of the reference's block samplers and its DGL compliance
helper (reference: t10n/dgl_dsg/sampler.py:22-366, t10n/dgl_dsg/compliant.py:10-50).

Each sampler has the BlockSampler call ``sample_blocks(g, seed_nodes)`` ->
``(input_nodes, output_nodes, blocks)`` with grappa_b200.block.Block objects
(input layer first), over a C++ ``HostGraph``:

  IsolatedSamplerOrCoarseCounter / IsolatedSamplerWithPreciseCounter
      neighbour sampling inside the working partition; the batch's coverage weight
      is handed to the loader (``set_coarse_count``).  The reference's coarse
      counter path never reports it (t10n/dgl_dsg/sampler.py:154-171); here both
      report the mean per-seed coverage ratio, the quantity the precise counter
      computes.
  XBorderSampler     cross-partition sampling through the owners (xbsampler)
  PinSAGESampler     random-walk neighbourhoods (pinsage_sampler)
  to_dgl_batch       per-hop (u, v) lists -> blocks, dst nodes first
"""
import numpy as np
import torch

from grappa_b200 import _native
from grappa_b200.block import blocks_from_host
from grappa_b200.pinsage_sampler import walk_block
from grappa_b200.xbsampler import HostXBBatchSampler, to_block


def to_dgl_batch(output_nodes, all_layers, all_inputs=None):
    """Blocks from [u_0, v_0, u_1, v_1, ...] (seed hop first, graph ids)."""
    assert torch.is_tensor(output_nodes), "only handle tensor input"
    blocks = []
    dst = output_nodes
    for i in range(len(all_layers) // 2):
        b = to_block(torch.as_tensor(all_layers[2 * i]), torch.as_tensor(all_layers[2 * i + 1]), dst)
        dst = b.srcdata["_ID"]
        blocks.insert(0, b)
    return dst, output_nodes, blocks


class IsolatedSamplerOrCoarseCounter:
    def __init__(self, fanouts, rank, nbr_idx, num_part, prefix_sum, device, device_allocator, loader, seed=0,
                 gideg=None):
        self.fanouts = [int(f) for f in fanouts]
        self.rank, self.nbr_idx, self.num_part, self.prefix_sum = rank, nbr_idx, num_part, prefix_sum
        self.device, self.da, self.loader = device, device_allocator, loader
        self.seed = int(seed)
        self.gideg = gideg  # callable: global ids -> global in-degrees (default: the loader's)
        self.step = 0
        self.epoch = 0

    def _gideg(self, seeds):
        if self.gideg is not None:
            return self.gideg(seeds)
        out = torch.zeros(seeds.shape[0], dtype=torch.int64)
        return self.loader.get_batch_gideg(out, seeds)

    def sample_blocks(self, g, seed_nodes, exclude_eids=None):
        seeds = torch.as_tensor(seed_nodes, dtype=torch.int64).cpu()
        gd = self._gideg(seeds)
        blocks, cs, cn = _native.host().graph.sample_batch(g, self.fanouts, seeds.numpy(), gd.numpy(), self.seed,
                                                           self.epoch, self.step, False)
        self.step += 1
        if self.loader is not None and hasattr(self.loader, "set_coarse_count"):
            self.loader.set_coarse_count(cs / cn if cn > 0 else 0.0)
        b = blocks_from_host(blocks)
        return b[0].srcdata["_ID"], seeds, b


IsolatedSamplerWithPreciseCounter = IsolatedSamplerOrCoarseCounter


class XBorderSampler:
    def __init__(self, fanouts, rank, num_part, prefix_sum, xb, device, device_allocator, seed=0):
        self.inner = HostXBBatchSampler(None, torch.zeros(0, dtype=torch.int64), fanouts, xb=xb, rank=rank,
                                        num_part=num_part, device_allocator=device_allocator, seed=seed)

    def sample_blocks(self, g, seed_nodes, exclude_eids=None):
        s = self.inner
        s.graph = g
        s.nodes = torch.as_tensor(seed_nodes, dtype=torch.int64).cpu()
        s.total_nodes_n = int(s.nodes.numel())
        s.batch_size = max(1, s.total_nodes_n)
        s.batch_idx = 0
        return s._next_batch()


class PinSAGESampler:
    def __init__(self, g, num_layer, random_walk_length=3, random_walk_restart_prob=0.5, num_random_walk=4,
                 num_neighbor=5, seed=0, **_):
        self.g = g
        self.num_layer = int(num_layer)
        self.length = int(random_walk_length)
        self.restart = float(random_walk_restart_prob)
        self.walks = int(num_random_walk)
        self.k = int(num_neighbor)
        self.seed = int(seed)
        self.step = 0

    def sample_blocks(self, _, seed_nodes, exclude_eids=None):
        output_nodes = torch.as_tensor(seed_nodes, dtype=torch.int64).cpu()
        seeds = output_nodes
        blocks = []
        for layer in range(self.num_layer):
            key = int(_native.host().graph.hop_key(self.seed, 0, self.step, layer))
            b = walk_block(self.g, seeds, self.length, self.restart, self.walks, self.k, key)
            seeds = b.srcdata["_ID"]
            blocks.insert(0, b)
        self.step += 1
        return seeds, output_nodes, blocks


def to_dgl_tensor(th_tensor):
    """Identity: blocks here hold torch tensors already (reference: sampler.py:18-20)."""
    return th_tensor if torch.is_tensor(th_tensor) else torch.as_tensor(np.asarray(th_tensor))
