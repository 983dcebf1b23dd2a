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


def to_block_device(dst, indptr, src):
    """Block of one hop on the device: ``dst`` (unique global ids, the block's first source
    nodes), the in-edges of dst[i] being ``src[indptr[i]:indptr[i+1]]`` (global ids).  The
    sources follow the destinations in order of first appearance in the edge list (the
    reference's to_block order, t10n/dgl_dsg/compliant.py:40-47)."""
    n_dst = int(dst.numel())
    allids = torch.cat([dst.long(), src.long()])
    uniq, inv = torch.unique(allids, return_inverse=True)
    first = torch.full((uniq.numel(),), allids.numel(), dtype=torch.int64, device=dst.device)
    first.scatter_reduce_(0, inv, torch.arange(allids.numel(), device=dst.device), reduce="amin")
    order = torch.argsort(first)
    pos = torch.empty_like(order)
    pos[order] = torch.arange(order.numel(), device=dst.device)
    local = pos[inv]
    return Block(indptr.to(torch.int64), local[n_dst:].to(torch.int32), uniq[order], n_dst, int(order.numel()))


def _segments(indptr, n):
    """(edge -> segment index, edge -> offset inside its segment) of a CSR indptr."""
    deg = (indptr[1:] - indptr[:-1]).long()
    seg = torch.repeat_interleave(torch.arange(n, device=indptr.device), deg)
    off = torch.arange(int(indptr[-1]), device=indptr.device) - indptr[:-1].long()[seg]
    return seg, off


class _XbLoader:
    """Cross-partition mini-batches over target nodes (reference: HostXBBatchSampler,
    t10n/xbsampler.py:61-128): per hop the frontier is grouped by owner, the ids go to
    their owners, every owner samples its requests on the GPU from its complete in-edge
    CSR, and the sampled neighbour lists come back (peer-memory all-to-all); the hop's
    block is built on the device.  Every rank runs the same number of batches."""

    def __init__(self, loader, targets, fanouts, batch_size, n_batches):
        self.ld, self.targets, self.fanouts = loader, targets, fanouts
        self.bs, self.n_batches = max(1, int(batch_size)), int(n_batches)
        self.i = 0

    def __iter__(self):
        self.i = 0
        return self

    def __len__(self):
        return self.n_batches

    def __next__(self):
        if self.i >= self.n_batches:
            raise StopIteration
        out = self.targets[self.i * self.bs:(self.i + 1) * self.bs]
        seeds, blocks = out, []
        for hop, fanout in enumerate(reversed(self.fanouts)):
            indptr, src = self.ld._xb_hop(seeds, int(fanout), hop, self.i)
            blk = to_block_device(seeds, indptr, src)
            seeds = blk.srcdata["_ID"]
            blocks.insert(0, blk)
        self.i += 1
        return seeds, out, blocks


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

    # ------------------------------------------------------------------ cross-border inference
    def _peer_a2a(self):
        if getattr(self, "_a2a", None) is None:
            from grappa_b200.cl import PeerAllToAll

            self._a2a = PeerAllToAll(self.comm, self.device)
        return self._a2a

    def _sample_own(self, gids, fanout, hop, batch):
        """In-neighbours (global ids) of own global ids ``gids``: all of them for fanout < 0,
        else ``fanout`` distinct ones drawn by the GPU sampling kernel (Philox keys from
        (seed, batch, hop)).  Returns (indptr int64 [n + 1], sources int64)."""
        cu = _native.cuda()
        n = int(gids.numel())
        lo = self.prefix_sum[self.rank]
        rows = (gids.long() - lo).to(torch.int32)
        deg = (self.own.indptr[1:] - self.own.indptr[:-1])[rows.long()] if n else rows.long()
        cap = int(deg.sum()) if fanout < 0 else int(torch.clamp(deg, max=fanout).sum())
        out_ip = torch.zeros(n + 1, dtype=torch.int32, device=self.device)
        out_nbr = torch.zeros(max(1, cap), dtype=torch.int32, device=self.device)
        n_e = torch.zeros(1, dtype=torch.int32, device=self.device)
        scratch = torch.zeros(cu.sample_scratch_words(max(1, n)), dtype=torch.int64, device=self.device)
        err = torch.zeros(1, dtype=torch.int32, device=self.device)
        ctr = new_counters(self.seed, self.device)
        ctr[C_EPOCH], ctr[C_STEP] = 1 << 20, batch  # draws apart from the training epochs
        cu.sample_hop(self.own.indptr, self.own.indices, rows, None, n, None, int(fanout), False, ctr, hop, None,
                      None, out_ip, out_nbr, n_e, scratch, err, max(1, n))
        if int(err.item()):
            raise RuntimeError(f"device error word {int(err.item()):#x} in cross-border sampling")
        return out_ip.to(torch.int64), out_nbr[: int(n_e.item())].to(torch.int64)

    def _xb_hop(self, seeds, fanout, hop, batch):
        """In-neighbours of arbitrary global ids, sampled by their owners."""
        from grappa_b200.xborder import _group_by_owner

        seeds = seeds.to(self.device).long()
        if self.world == 1:
            return self._sample_own(seeds, fanout, hop, batch)
        a2a = self._peer_a2a()
        sorted_ids, order, counts = _group_by_owner(seeds, self.prefix_sum, self.world)
        requests = a2a.exchange(list(torch.split(sorted_ids, counts)))
        sizes = [int(q.numel()) for q in requests]
        ip, nbr = self._sample_own(torch.cat(requests), fanout, hop, batch)
        deg = ip[1:] - ip[:-1]
        bounds = [0]
        for z in sizes:
            bounds.append(bounds[-1] + z)
        deg_parts = [deg[bounds[p]:bounds[p + 1]].contiguous() for p in range(self.world)]
        nbr_parts = [nbr[int(ip[bounds[p]]):int(ip[bounds[p + 1]])].contiguous() for p in range(self.world)]
        deg_back = torch.cat(a2a.exchange(deg_parts))      # degrees of sorted_ids
        nbr_back = torch.cat(a2a.exchange(nbr_parts))      # their neighbours, in sorted order
        n = int(seeds.numel())
        ip_sorted = torch.zeros(n + 1, dtype=torch.int64, device=self.device)
        ip_sorted[1:] = torch.cumsum(deg_back, 0)
        deg_orig = torch.empty_like(deg_back)
        deg_orig[order] = deg_back
        ip_orig = torch.zeros(n + 1, dtype=torch.int64, device=self.device)
        ip_orig[1:] = torch.cumsum(deg_orig, 0)
        inv_order = torch.empty_like(order)
        inv_order[order] = torch.arange(n, device=self.device)
        seg, off = _segments(ip_orig, n)
        src = nbr_back[ip_sorted[:-1][inv_order[seg]] + off]
        return ip_orig, src

    def _equal_batches(self, n_targets, batch_size):
        n_batch = (n_targets + batch_size - 1) // batch_size
        if self.world > 1:
            n_batch = int(self.comm.all_reduce_max([n_batch])[0])
        bs = max(1, (n_targets + n_batch - 1) // n_batch) if n_batch else 1
        return n_batch, bs

    def xb_dataloader(self, args, force_even=True, full_neighbor=False, subset_tag="all"):
        """Cross-partition sampled mini-batches over the own nodes of ``subset_tag`` (the
        training fanouts, or full neighbourhoods); yields (input_nodes, output_nodes,
        blocks) with global ids."""
        fanouts = [-1 if full_neighbor else int(f) for f in self.fanouts]
        target = self.get_node_subset(subset_tag).to(self.device)
        n_batch, bs = self._equal_batches(int(target.numel()), int(args.batch_size_eval))
        return _XbLoader(self, target, fanouts, bs, n_batch)

    def xb_dataloader_per_layer(self, args, subset_tag="all"):
        """One full-neighbour hop per batch of own target nodes, for layer-wise inference
        (the own in-edge lists are complete, so no exchange is needed)."""
        target = self.get_node_subset(subset_tag).to(self.device)
        n_batch, bs = self._equal_batches(int(target.numel()), int(args.batch_size_eval))
        return _XbLoader(self, target, [-1], bs, n_batch)

    def xb_get_batch_input(self, batch_input, target_nodes):
        """Features of arbitrary global ids, fetched from their owners."""
        return self.xb_get_batch_emb(batch_input, target_nodes, self.own.feat)

    def xb_get_batch_emb(self, batch_input, target_nodes, emb_self):
        """Rows of a per-rank table (``emb_self``: this rank's own nodes) for arbitrary
        global ids, fetched from their owners through peer memory."""
        from grappa_b200.xborder import xb_gather_peer

        if self.world == 1:
            rows = emb_self[(target_nodes.to(emb_self.device).long() - self.prefix_sum[self.rank])]
            cols = batch_input.shape[1]
            batch_input.copy_(rows[:, :cols].to(batch_input.device, batch_input.dtype))
            return batch_input
        return xb_gather_peer(self._peer_a2a(), batch_input, target_nodes, emb_self, self.rank, self.world,
                              self.prefix_sum)

    def xb_scatter_emb(self, emb, target_nodes, emb_self):
        """emb_self[id] = row of ``emb`` for own ids; other rows go to their owners."""
        from grappa_b200.xborder import _group_by_owner

        ids = target_nodes.to(self.device).long()
        lo = self.prefix_sum[self.rank]
        if self.world == 1:
            emb_self[ids - lo] = emb.to(emb_self.device, emb_self.dtype)
            return emb_self
        sorted_ids, order, counts = _group_by_owner(ids, self.prefix_sum, self.world)
        a2a = self._peer_a2a()
        got_ids = a2a.exchange(list(torch.split(sorted_ids, counts)))
        rows = emb.to(self.device, emb_self.dtype)[order]
        got_rows = a2a.exchange(list(torch.split(rows, counts)))
        for q, r_ in zip(got_ids, got_rows):
            if q.numel():
                emb_self[q.long() - lo] = r_
        return emb_self

    def infer_train_mask_of(self, seeds):
        return self.train_mask[seeds.to(self.device).long() - self.prefix_sum[self.rank]]

    def infer_valid_mask_of(self, seeds):
        return self.valid_mask[seeds.to(self.device).long() - self.prefix_sum[self.rank]]

    def infer_test_mask_of(self, seeds):
        return self.test_mask[seeds.to(self.device).long() - self.prefix_sum[self.rank]]

    def close(self):
        if getattr(self, "_a2a", None) is not None:
            self._a2a.close()
            self._a2a = None
        self.store.close()
