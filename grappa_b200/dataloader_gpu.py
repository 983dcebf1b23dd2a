"""GPU-serving partition data loader (reference: IsolatedDataloaderGPU,
t10n/dataloader_gpu.py:27-799).

Same interface as grappa_b200.dataloader.IsolatedDataloader, with everything
resident in HBM: the own partition is loaded from the chunk files once
(graph_store.partition_from_chunks), the working graph (own + neighbour partition
+ halo rows) is rebuilt on every repartition by pulling the neighbour's CSR and
features straight out of the peers' HBM (graph_store.PartitionStore), mini-batches
are sampled on the GPU (sampler_gpu.GpuNeighborSampler) and features are gathered
on the GPU.  Blocks come out with global node ids in ``srcdata['_ID']`` (as the
CPU loader's), their CSR arrays on the device.

Training through this loader hands blocks to user code; the fused step
(grappa_b200.trainer.MiniBatchTrainer) keeps them inside the engine instead.
The reference's GPU loader reads the bridge ``v`` ids from the ``.u`` file and
the features as int64 (t10n/dataloader_gpu.py:209,226); this one reads them as
the chunk layout defines them.
"""
import torch

from grappa_b200 import _native
from grappa_b200.block import Block
from grappa_b200.dataset.meta import name_to_meta
from grappa_b200.dataset.synthetic import shuffle_keys
from grappa_b200.device_allocator import DeviceAllocGPUServing
from grappa_b200.graph_store import PartitionStore, next_neighbor, partition_from_chunks
from grappa_b200.sampler_gpu import C_EPOCH, C_STEP, GpuNeighborSampler, new_counters


class _GpuEpoch:
    """Iterator over one epoch of device-sampled mini-batches."""

    def __init__(self, loader, epoch):
        self.ld, self.epoch = loader, epoch
        ids = loader.train_local
        self.order = ids[torch.argsort(shuffle_keys(ids, loader.seed, epoch), stable=True)]
        self.step = 0

    def __iter__(self):
        return self

    def __next__(self):
        ld = self.ld
        if self.step >= ld.local_batch:
            raise StopIteration
        bs = ld.adjust_bs
        seeds = self.order[self.step * bs:(self.step + 1) * bs]
        ld.counters[C_EPOCH] = self.epoch
        ld.counters[C_STEP] = self.step
        ld.cov.zero_()
        ld.sampler.load_seeds(seeds)
        w = ld.store.working
        ld.sampler.sample(w.indptr, w.indices, ld.counters, gideg=ld.own.gideg, cov=ld.cov)
        _native.cuda().step_end(ld.counters)
        blocks = ld.sampler.blocks()
        for b in blocks:  # working ids -> global ids
            b.srcdata["_ID"] = ld.w2g[b.srcdata["_ID"].long()]
            b.dstdata["_ID"] = b.srcdata["_ID"][: b.n_dst]
        ld._last_cov = ld.cov
        self.step += 1
        off = ld.prefix_sum[ld.rank]
        return blocks[0].srcdata["_ID"], seeds.long() + off, blocks


class IsolatedDataloaderGPU:
    serving = DeviceAllocGPUServing

    def __init__(self, device, args, comm=None):
        import torch.distributed as dist

        meta = name_to_meta(args.graph_name)
        self.device = torch.device(device)
        self.da = self.serving(self.device, getattr(args, "backend", "nccl"))
        self.in_feats, self.n_classes = meta.n_dim, meta.n_label
        self.num_part = int(args.n_part)
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        self.world = dist.get_world_size() if dist.is_initialized() else 1
        self.seed = int(getattr(args, "seed", 0))
        self.fanouts = [int(f) for f in str(args.fan_out).split(",")]
        self.own = partition_from_chunks(args.data_path, args.graph_name, args.part_method, args.n_part, self.rank,
                                         meta.n_dim, self.device)
        self.prefix_sum = self.own.prefix
        if comm is None:
            from grappa_b200.parallel.comm import Comm

            comm = Comm()
        self.comm = comm
        self.store = PartitionStore(self.own, comm)
        self.train_local = torch.nonzero(self.own.train_mask).squeeze(1).to(torch.int64)
        n_batch = (self.train_local.numel() + int(args.batch_size) - 1) // int(args.batch_size)
        self.local_batch = int(comm.all_reduce_max([n_batch])[0]) if self.world > 1 else n_batch
        self.adjust_bs = max(1, (self.train_local.numel() + self.local_batch - 1) // max(self.local_batch, 1))
        self.sampler = GpuNeighborSampler(self.fanouts, self.adjust_bs, self.store.cap_nodes, self.device)
        self.counters = new_counters(self.seed, self.device)
        self.cov = torch.zeros(2, dtype=torch.float32, device=self.device)
        self._last_cov = None
        self.nbr_idx = self.rank
        self.max_coarse_count = int(args.batch_size) * float(self.fanouts[0])
        self.w2g = None
        self.g2w = None
        self.dataloader = None
        self.train_mask, self.valid_mask, self.test_mask = self.own.train_mask, self.own.val_mask, self.own.test_mask
        self.node_label = self.own.label

    # ------------------------------------------------------------------ working graph
    def load_nbr_chunk_v2(self, nbr_idx):
        w = self.store.repartition(nbr_idx)
        n_own, n_nbr = w.n_own, w.n_nbr
        n_halo = int(w.n_halo_dev.item()) if n_nbr else 0
        ps = self.prefix_sum
        parts = [torch.arange(ps[self.rank], ps[self.rank] + n_own, device=self.device)]
        if n_nbr:
            parts.append(torch.arange(ps[nbr_idx], ps[nbr_idx] + n_nbr, device=self.device))
            parts.append(self.store._halo_ids[:n_halo].to(torch.int64))
        self.w2g = torch.cat(parts)
        self.g2w = torch.full((ps[-1],), -1, dtype=torch.int64, device=self.device)
        self.g2w[self.w2g] = torch.arange(self.w2g.numel(), device=self.device)
        return w

    def get_cur_dataloader(self, args, epoch, overide_exp_mode=-1):
        if self.w2g is None or epoch % int(args.repart_every) == 0:
            self.nbr_idx = next_neighbor(self.nbr_idx, self.rank, self.world) if self.world > 1 else self.rank
            self.load_nbr_chunk_v2(self.nbr_idx)
        self.dataloader = _GpuEpoch(self, epoch)
        return self.dataloader

    # ------------------------------------------------------------------ batch data
    def get_coarse_count(self):
        if self._last_cov is None:
            return 0.0
        c = self._last_cov.cpu()
        return min(float(c[0] / c[1]) if c[1] > 0 else 0.0, self.max_coarse_count)

    def set_coarse_count(self, coarse_count):
        pass

    def get_batch_input(self, batch_input, input_nodes):
        rows = self.g2w[input_nodes.to(self.device).long()].to(torch.int32)
        out = torch.empty((rows.numel(), self.store.working.feat.shape[1]), dtype=torch.bfloat16, device=self.device)
        if rows.numel():
            _native.cuda().gather_rows(self.store.working.feat, rows, None, rows.numel(), rows.numel(),
                                       out.shape[1], out)
        batch_input.copy_(out[:, : batch_input.shape[1]].to(batch_input.dtype))
        return batch_input

    def get_batch_gideg(self, batch_input, input_nodes):
        g = input_nodes.to(self.device).long()
        own = (g >= self.prefix_sum[self.rank]) & (g < self.prefix_sum[self.rank + 1])
        batch_input.zero_()
        batch_input[own] = self.own.gideg[g[own] - self.prefix_sum[self.rank]].to(batch_input.dtype)
        return batch_input

    def get_batch_labels(self, seed):
        return self.node_label[(seed.to(self.device).long() - self.prefix_sum[self.rank])]

    def get_node_label(self):
        return self.node_label

    def get_rank(self):
        return self.rank

    def get_max_step(self):
        return self.local_batch

    def get_comm_dev(self):
        return self.da.comm_dev()

    def get_num_node(self):
        return self.own.n_nodes

    def get_nid_offset(self):
        return self.prefix_sum[self.rank]

    def get_node_subset(self, subset_tag):
        off = self.prefix_sum[self.rank]
        masks = {"train": self.train_mask, "valid": self.valid_mask, "test": self.test_mask}
        if subset_tag == "all":
            return torch.cat([torch.nonzero(masks[k]).squeeze(1) for k in ("train", "valid", "test")]) + off
        if subset_tag not in masks:
            raise ValueError(f"{subset_tag} is unknown")
        return torch.nonzero(masks[subset_tag]).squeeze(1) + off

    def full_neighbor_block(self, target_nodes):
        """One full-neighbour block over the working graph for global ``target_nodes``
        (the own rows' in-edges are complete there), for layer-wise inference."""
        w = self.store.working
        rows = self.g2w[target_nodes.to(self.device).long()]
        ip, ix = w.indptr, w.indices
        beg, end = ip[rows], ip[rows + 1]
        deg = end - beg
        indptr = torch.zeros(rows.numel() + 1, dtype=torch.int64, device=self.device)
        indptr[1:] = torch.cumsum(deg, 0)
        e = torch.arange(int(indptr[-1]), device=self.device)
        owner = torch.repeat_interleave(torch.arange(rows.numel(), device=self.device), deg)
        src_w = ix[(beg[owner] + e - indptr[owner])].long()
        uniq, inv = torch.unique(torch.cat([rows, src_w]), return_inverse=True)
        # dst rows first, then the other sources
        local = torch.full((uniq.numel(),), -1, dtype=torch.int64, device=self.device)
        local[inv[: rows.numel()]] = torch.arange(rows.numel(), device=self.device)
        rest = inv[rows.numel():]
        new = torch.unique(rest[local[rest] < 0], sorted=False)
        local[new] = torch.arange(rows.numel(), rows.numel() + new.numel(), device=self.device)
        src_ids = torch.empty(rows.numel() + new.numel(), dtype=torch.int64, device=self.device)
        src_ids[local] = uniq
        return Block(indptr, local[rest], self.w2g[src_ids], rows.numel(), src_ids.numel())

    def infer_train_mask_of(self, seeds):
        return self.train_mask[seeds.to(self.device).long() - self.prefix_sum[self.rank]]

    def infer_valid_mask_of(self, seeds):
        return self.valid_mask[seeds.to(self.device).long() - self.prefix_sum[self.rank]]

    def infer_test_mask_of(self, seeds):
        return self.test_mask[seeds.to(self.device).long() - self.prefix_sum[self.rank]]

    def close(self):
        self.store.close()
