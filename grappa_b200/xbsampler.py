"""Cross-border sampler for inference (reference: t10n/xbsampler.py:17-142).

For a batch of target nodes, every hop groups the current frontier by owner,
sends each owner its nodes, the owner samples their in-neighbours on its own
working graph (which holds every in-edge of its nodes), and the sampled
(src, dst) pairs come back; the pairs are compacted into a block with the dst
nodes first.  With fanout INT64_MAX / -1 the sampling is full-neighbour, which is
what layer-wise inference uses.
"""
import numpy as np
import torch

from grappa_b200 import _native
from grappa_b200.block import Block
from grappa_b200.cl import t10n_all_to_all_1d_int64_nccl as t10n_all_to_all_1d_int64
from grappa_b200.sampler import BatchSampler
from grappa_b200.xborder import xb_group_by_partition


def to_block(u, v, dst_nodes):
    """Block with dst nodes first and the other sources in order of first appearance."""
    lid = {int(x): i for i, x in enumerate(dst_nodes.tolist())}
    src = list(dst_nodes.tolist())
    uu = u.tolist()
    local_u = np.empty(len(uu), dtype=np.int64)
    for k, x in enumerate(uu):
        j = lid.get(x)
        if j is None:
            j = len(src)
            lid[x] = j
            src.append(x)
        local_u[k] = j
    vloc = np.array([lid[int(x)] for x in v.tolist()], dtype=np.int64)
    order = np.argsort(vloc, kind="stable")
    n_dst = len(dst_nodes)
    indptr = np.zeros(n_dst + 1, dtype=np.int64)
    indptr[1:] = np.cumsum(np.bincount(vloc, minlength=n_dst))
    return Block(torch.from_numpy(indptr), torch.from_numpy(local_u[order]), torch.tensor(src, dtype=torch.int64),
                 n_dst, len(src))


class HostXBBatchSampler(BatchSampler):
    def __init__(self, graph, target_nodes, fan_outs, repeated=False, batch_size=1, shuffle=False, xb=None, rank=-1,
                 num_part=0, device_allocator=None, seed=0):
        super().__init__(target_nodes, batch_size, shuffle, -1, seed)
        self.graph = graph
        self.fan_outs = [-1 if int(f) >= np.iinfo(np.int64).max or int(f) < 0 else int(f) for f in fan_outs]
        self.xb, self.rank, self.num_part, self.da = xb, rank, num_part, device_allocator

    def __iter__(self):
        self.epoch += 1
        self.nodes = self.target_nodes[self._order()]
        self.batch_idx = 0
        self.total_batch = self._n_batches()
        return self

    def _comm_dev(self):
        return self.da.comm_dev() if self.da is not None else torch.device("cpu")

    def _next_batch(self):
        output_nodes = self._cur_batch_opt_nodes(self.nodes)
        seeds = output_nodes
        blocks = []
        for hop, fanout in enumerate(reversed(self.fan_outs)):
            groups, _ = xb_group_by_partition(self.xb, seeds, self.num_part)
            asked = t10n_all_to_all_1d_int64(groups, self.rank, self.num_part, device=self._comm_dev())
            src_list, dst_list = [], []
            for ids in asked:
                key = int(_native.host().graph.hop_key(self.seed, self.epoch, self.batch_idx, hop))
                uu, vv = _native.host().graph.sample_neighbors(self.graph, ids.cpu().numpy(), fanout, key)
                src_list.append(torch.from_numpy(uu))
                dst_list.append(torch.from_numpy(vv))
            all_u = torch.cat(t10n_all_to_all_1d_int64(src_list, self.rank, self.num_part, device=self._comm_dev()))
            all_v = torch.cat(t10n_all_to_all_1d_int64(dst_list, self.rank, self.num_part, device=self._comm_dev()))
            block = to_block(all_u.cpu(), all_v.cpu(), seeds)
            seeds = block.srcdata["_ID"]
            blocks.insert(0, block)
        self.batch_idx += 1
        return seeds, output_nodes, blocks

    def __next__(self):
        if self.batch_idx >= self.total_batch:
            raise StopIteration
        return self._next_batch()
