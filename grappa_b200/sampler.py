"""Mini-batch iterators (reference: t10n/sampler.py:14-191).

``HostBatchSampler`` / ``HostBatchSamplerWithCounter`` drive the C++ pipelined
host sampler (a worker thread keeps two batches ready) and yield
``(input_nodes, output_nodes, blocks)`` like the reference's DGL path, with
``grappa_b200.block.Block`` objects instead of DGL blocks (input layer first).
The with-counter variant also reports the batch's coverage weight c_r.

``GpuBatchSampler`` is the device version (the reference only declares it): the
sm_100a sampler of grappa_b200.sampler_gpu, materialising exact-size blocks.

Shuffling is a seeded permutation per epoch (a hash of (seed, epoch, id)), the
same on CPU and GPU; the reference uses an unseeded torch.randperm.
"""
import torch

from grappa_b200 import _native
from grappa_b200.block import blocks_from_host
from grappa_b200.dataset.synthetic import shuffle_keys


class BatchSampler:
    def __init__(self, target_nodes, batch_size=1, shuffle=False, use_batch_n=-1, seed=0):
        assert torch.is_tensor(target_nodes), "only handle tensor input"
        self.target_nodes = target_nodes.to(torch.int64).cpu()
        self.batch_size = int(batch_size)
        self.shuffle = bool(shuffle)
        self.use_batch_n = int(use_batch_n)
        self.seed = int(seed)
        self.total_nodes_n = int(self.target_nodes.shape[0])
        self.total_batch = 0
        self.batch_idx = 0
        self.epoch = -1

    def _order(self):
        if not self.shuffle:
            return torch.arange(self.total_nodes_n)
        return torch.argsort(shuffle_keys(self.target_nodes, self.seed, self.epoch), stable=True)

    def _n_batches(self):
        if self.use_batch_n <= 0:
            return (self.total_nodes_n + self.batch_size - 1) // self.batch_size
        return self.use_batch_n

    def _cur_batch_opt_nodes(self, nodes):
        lo = min(self.total_nodes_n, self.batch_idx * self.batch_size)
        return nodes[lo:min(self.total_nodes_n, lo + self.batch_size)]

    def __len__(self):
        return self._n_batches()


class HostBatchSampler(BatchSampler):
    def __init__(self, graph, target_nodes, fan_outs, repeated=False, batch_size=1, shuffle=False, use_batch_n=-1,
                 seed=0):
        super().__init__(target_nodes, batch_size, shuffle, use_batch_n, seed)
        self.graph = graph
        self.fan_outs = [int(f) for f in fan_outs]
        self.repeated = bool(repeated)
        self.host_sampler = _native.host().graph.HostSampler(graph, self.fan_outs, self.repeated, False, self.seed)

    def __iter__(self):
        self.epoch += 1
        self.nodes = self.target_nodes[self._order()]
        self.batch_idx = 0
        self.total_batch = self._n_batches()
        self.host_sampler.reinit(self.nodes.numpy(), None, self.batch_size, self.total_batch, self.epoch)
        return self

    def __next__(self):
        if self.batch_idx >= self.total_batch:
            raise StopIteration
        seeds, blocks, _, _ = self.host_sampler.next_batch()
        self.batch_idx += 1
        b = blocks_from_host(blocks)
        return b[0].srcdata["_ID"], torch.from_numpy(seeds), b


class HostBatchSamplerWithCounter(HostBatchSampler):
    def __init__(self, graph, target_nodes, fan_outs, repeated=False, batch_size=1, shuffle=False,
                 target_nodes_gideg=None, use_batch_n=-1, seed=0):
        BatchSampler.__init__(self, target_nodes, batch_size, shuffle, use_batch_n, seed)
        self.graph = graph
        self.fan_outs = [int(f) for f in fan_outs]
        self.repeated = bool(repeated)
        assert torch.is_tensor(target_nodes_gideg), "only handle tensor input"
        self.target_nodes_gideg = target_nodes_gideg.to(torch.int64).cpu()
        self.host_sampler = _native.host().graph.HostSampler(graph, self.fan_outs, self.repeated, True, self.seed)
        self.cur_resample_count = 0.0

    def __iter__(self):
        self.epoch += 1
        order = self._order()
        self.nodes = self.target_nodes[order]
        gideg = self.target_nodes_gideg[order]
        self.batch_idx = 0
        self.total_batch = self._n_batches()
        self.host_sampler.reinit(self.nodes.numpy(), gideg.numpy(), self.batch_size, self.total_batch, self.epoch)
        return self

    def __next__(self):
        if self.batch_idx >= self.total_batch:
            raise StopIteration
        seeds, blocks, cs, cn = self.host_sampler.next_batch()
        self.cur_resample_count = cs / cn if cn > 0 else 0.0
        self.batch_idx += 1
        b = blocks_from_host(blocks)
        return b[0].srcdata["_ID"], torch.from_numpy(seeds), b

    def get_cur_resampling_cnt(self):
        return self.cur_resample_count


class GpuBatchSampler(BatchSampler):
    """Device sampler over a CSC graph on the GPU (indptr int64, indices int32)."""

    def __init__(self, indptr, indices, target_nodes, fan_outs, batch_size=1, shuffle=False, seed=0, gideg=None,
                 replace=False):
        super().__init__(target_nodes, batch_size, shuffle, -1, seed)
        from grappa_b200.sampler_gpu import GpuNeighborSampler, new_counters

        self.indptr, self.indices = indptr, indices
        self.device = indptr.device
        self.sampler = GpuNeighborSampler(fan_outs, batch_size, indptr.numel() - 1, self.device, replace=replace)
        self.counters = new_counters(seed, self.device)
        self.gideg = gideg
        self.cov = torch.zeros(2, device=self.device)
        self.cur_resample_count = 0.0

    def __iter__(self):
        self.epoch += 1
        self.nodes = self.target_nodes[self._order()]
        self.batch_idx = 0
        self.total_batch = self._n_batches()
        self.counters[1] = self.epoch
        return self

    def __next__(self):
        if self.batch_idx >= self.total_batch:
            raise StopIteration
        seeds = self._cur_batch_opt_nodes(self.nodes)
        self.counters[2] = self.batch_idx
        self.cov.zero_()
        self.sampler.load_seeds(seeds)
        self.sampler.sample(self.indptr, self.indices, self.counters, gideg=self.gideg,
                            cov=self.cov if self.gideg is not None else None)
        _native.cuda().step_end(self.counters)  # fresh compaction tags for the next batch
        blocks = self.sampler.blocks()
        if self.gideg is not None:
            c = self.cov.cpu()
            self.cur_resample_count = float(c[0] / c[1]) if c[1] > 0 else 0.0
        self.batch_idx += 1
        return blocks[0].srcdata["_ID"], seeds.to(self.device), blocks

    def get_cur_resampling_cnt(self):
        return self.cur_resample_count
