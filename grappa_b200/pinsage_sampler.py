"""PinSAGE mini-batch sampler (reference: PinSAGESampler, t10n/dgl_dsg/sampler.py:323-366).

Every layer's block comes from random walks with restart over in-edges: per seed
``num_random_walk`` walks of at most ``random_walk_length`` steps (stop
probability ``random_walk_restart_prob`` before each step), the ``num_neighbor``
most visited nodes become its neighbours and the visit counts the edge weights
(``block.edata['weights']``).  The walks run in the C++ host engine
(grappa_b200/csrc/host/graph_host.cc, random_walk_topk) with the Philox streams
shared with the GPU walker.
"""
import torch

from grappa_b200 import _native
from grappa_b200.block import Block
from grappa_b200.sampler import BatchSampler


def walk_block(graph, seeds, length, restart_prob, num_walks, num_neighbors, key):
    d = _native.host().graph.random_walk_topk(graph, seeds.cpu().numpy(), length, restart_prob, num_walks,
                                              num_neighbors, key)
    return Block(torch.from_numpy(d["indptr"]), torch.from_numpy(d["indices"]), torch.from_numpy(d["src_nid"]),
                 d["n_dst"], d["n_src"], torch.from_numpy(d["src_sampled"]),
                 edge_weight=torch.from_numpy(d["weights"]))


class HostPinSAGESampler(BatchSampler):
    def __init__(self, graph, target_nodes, num_layer, batch_size=1, shuffle=False, use_batch_n=-1, seed=0,
                 random_walk_length=None, random_walk_restart_prob=0.5, num_random_walk=4, num_neighbor=5):
        super().__init__(target_nodes, batch_size, shuffle, use_batch_n, seed)
        self.graph = graph
        self.num_layer = int(num_layer)
        self.length = int(random_walk_length if random_walk_length is not None else num_layer)
        self.restart_prob = float(random_walk_restart_prob)
        self.num_walks = int(num_random_walk)
        self.num_neighbors = int(num_neighbor)

    def __iter__(self):
        self.epoch += 1
        self.nodes = self.target_nodes[self._order()]
        self.batch_idx = 0
        self.total_batch = self._n_batches()
        return self

    def sample_blocks(self, seeds):
        blocks = []
        cur = seeds
        for layer in range(self.num_layer):
            key = int(_native.host().graph.hop_key(self.seed, max(self.epoch, 0), self.batch_idx, layer))
            b = walk_block(self.graph, cur, self.length, self.restart_prob, self.num_walks, self.num_neighbors, key)
            cur = b.srcdata["_ID"]
            blocks.insert(0, b)
        return cur, blocks

    def __next__(self):
        if self.batch_idx >= self.total_batch:
            raise StopIteration
        seeds = self._cur_batch_opt_nodes(self.nodes)
        input_nodes, blocks = self.sample_blocks(seeds)
        self.batch_idx += 1
        return input_nodes, seeds, blocks

    def get_cur_resampling_cnt(self):
        return 1.0
