"""Partition-local data loader over the chunk files (reference: t10n/dataloader.py:27-842).

Every rank owns partition ``rank`` of a chunked dataset (layout:
grappa_b200.dataset.io_dist).  Every ``repart_every`` epochs the rank moves to the
next neighbour partition (round robin, skipping itself) and rebuilds its working
graph in the global id space (own ids offset by ``prefix_sum[rank]``):

  * every in-edge of the own and the neighbour partition: p{rank}, p{nbr} and the
    bridges b{j}_{rank}, b{j}_{nbr} of every other partition j;
  * the features and in-degrees of both partitions, plus a halo cache of the
    rows of every other source node those bridges reference, resolved by the
    C++ ``XBorder`` ad-hoc id map.

The sampler is the C++ pipelined host sampler with coverage counting
(``HostBatchSamplerWithCounter``) over the local train nodes; every rank runs the
same number of steps (max over ranks, batch size equalised), which is what the
coverage-weighted gradient all-reduce needs.  The DGL sampling path of the
reference (``--close_dd`` not given) has no counterpart: this loader always uses
the native sampler.

GPU serving (features and sampling on the device) is
grappa_b200.dataloader_gpu.IsolatedDataloaderGPU.
"""
import time

import numpy as np
import torch

from grappa_b200._native import host
from grappa_b200.dataset.io_dist import ChunkIO
from grappa_b200.dataset.meta import name_to_meta, t10n_chunk_path
from grappa_b200.device_allocator import DeviceAllocCPUServing, T10nDeviceAllocator
from grappa_b200.sampler import HostBatchSamplerWithCounter
from grappa_b200.util import pprint, set_py_affinity, timing
from grappa_b200.xborder import XBorder, xb_gather, xb_group_by_partition, xb_scatter
from grappa_b200.xbsampler import HostXBBatchSampler


def _dist():
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def _all_reduce_max(x, device):
    import torch.distributed as dist

    t = torch.tensor([int(x)], dtype=torch.int64, device=device)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return int(t.item())


class IsolatedDataloader:
    serving = DeviceAllocCPUServing

    def __init__(self, device, args):
        tic = time.time()
        meta = name_to_meta(args.graph_name)
        self.device = device
        self.da = self.serving(device, getattr(args, "backend", "gloo"))
        self.in_feats, self.n_classes = meta.n_dim, meta.n_label
        self.use_dgl_dsg_sampler = False
        self.model_name = getattr(args, "model", "sage")
        self.num_part = int(args.n_part)
        self.rank, self.world = _dist()
        assert self.world == self.num_part, "one partition per rank"
        # the host graph goes on the GPU's NUMA node, the process's CPUs there when
        # enabled (reference: t10n/dataloader.py:60-63)
        ta = T10nDeviceAllocator(getattr(args, "num_gpus", -1))
        self.node_id = ta.get_numa_affinity(ta.get_local_gpu_id(self.world, self.rank))
        set_py_affinity(self.node_id)
        self.nbr_idx = self.rank
        self.seed = int(getattr(args, "seed", 0))
        self.fanouts = [int(f) for f in str(args.fan_out).split(",")]
        self.max_coarse_count = int(args.batch_size) * float(self.fanouts[0])
        self.data_path = f"{args.data_path}/{t10n_chunk_path(args.graph_name, args.part_method, args.n_part)}"
        self.io = ChunkIO(self.data_path, self.num_part, self.in_feats)
        self.part_num_node = self.io.counts
        self.prefix_sum = self.io.prefix
        self.xb = XBorder(self.rank, self.num_part, self.prefix_sum)

        r = self.rank
        self.p0_u = torch.from_numpy(self.io.part(r, "u"))
        self.p0_v = torch.from_numpy(self.io.part(r, "v"))
        self.feat_0 = torch.from_numpy(self.io.part(r, "nfeat"))
        self.label_0 = torch.from_numpy(self.io.part(r, "label"))
        ideg = self.io.part(r, "ideg")
        self.ideg_0 = torch.from_numpy(ideg) if ideg is not None else torch.ones(self.label_0.shape[0],
                                                                                 dtype=torch.int64)
        self.train_mask = torch.from_numpy(self.io.part(r, "train"))
        self.valid_mask = torch.from_numpy(self.io.part(r, "valid"))
        self.test_mask = torch.from_numpy(self.io.part(r, "test"))
        off = self.prefix_sum[r]
        self.train_nid = torch.nonzero(self.train_mask).flatten() + off
        self.valid_nid = torch.nonzero(self.valid_mask).flatten() + off
        self.test_nid = torch.nonzero(self.test_mask).flatten() + off
        self.node_label = self.label_0
        self.feat_n = [None] * self.num_part
        self.ideg_n = [None] * self.num_part
        self.feat_n[r], self.ideg_n[r] = self.feat_0, self.ideg_0

        n_batch = (self.train_nid.shape[0] + int(args.batch_size) - 1) // int(args.batch_size)
        self.local_batch = _all_reduce_max(n_batch, self.da.comm_dev())
        self.adjust_bs = max(1, (self.train_nid.shape[0] + self.local_batch - 1) // self.local_batch)
        self.explore_mode = 1 if self.num_part == 1 else 2
        self.batch_coarse_count = 1.0
        self.dataloader = None
        self.cur_g = None
        self._pp(f"rank:{r:02d} INIT_LOAD: {time.time() - tic:.2f} s")
        self._pp(f"rank:{r:02d} NUM_BATCH: {self.local_batch}")
        self._pp(f"rank:{r:02d} bs       : {self.adjust_bs}")
        self._pp(f"rank:{r:02d} N_TRAIN  : {self.train_nid.shape[0]}")
        self._pp(f"rank:{r:02d} N_VALID  : {self.valid_nid.shape[0]}")
        self._pp(f"rank:{r:02d} N_TEST   : {self.test_nid.shape[0]}")

    def _pp(self, *a):
        pprint(self.rank, *a)

    # ------------------------------------------------------------------ working graph
    def load_nbr_chunk_v2(self, nbr_idx):
        """Edges, features and halo cache of the working partition (own + ``nbr_idx``)."""
        tic = time.time()
        r, P, ps = self.rank, self.num_part, self.prefix_sum
        self.xb.ad_hoc_clear()
        self.xb.set_nbr_idx(nbr_idx)
        self.feat_n = [None] * P
        self.ideg_n = [None] * P
        self.feat_n[r], self.ideg_n[r] = self.feat_0, self.ideg_0
        srcs = [self.p0_u + ps[r]]
        dsts = [self.p0_v + ps[r]]
        if nbr_idx != r:
            srcs.append(torch.from_numpy(self.io.part(nbr_idx, "u")) + ps[nbr_idx])
            dsts.append(torch.from_numpy(self.io.part(nbr_idx, "v")) + ps[nbr_idx])
            self.feat_n[nbr_idx] = torch.from_numpy(self.io.part(nbr_idx, "nfeat"))
            ideg = self.io.part(nbr_idx, "ideg")
            self.ideg_n[nbr_idx] = torch.from_numpy(ideg) if ideg is not None else None
        halo = []
        for j in range(P):
            for prim in {r, nbr_idx}:
                if j == prim:
                    continue
                bu, bv = self.io.bridge(j, prim)  # in-edges of `prim` from partition j
                if bu is None:
                    continue
                bu = torch.from_numpy(bu) + ps[j]
                srcs.append(bu)
                dsts.append(torch.from_numpy(bv) + ps[prim])
                if j not in (r, nbr_idx):
                    halo.append(bu)
        if halo:
            uniq = torch.unique(torch.cat(halo))
            groups, _ = xb_group_by_partition(self.xb, uniq, P)
            for j in range(P):
                if j in (r, nbr_idx) or groups[j].numel() == 0:
                    continue
                ids = torch.sort(groups[j])[0]
                rows = (ids - ps[j]).numpy()
                self.feat_n[j] = torch.from_numpy(np.ascontiguousarray(self.io.part(j, "nfeat", mmap=True)[rows]))
                ideg = self.io.part(j, "ideg", mmap=True)
                self.ideg_n[j] = torch.from_numpy(np.ascontiguousarray(ideg[rows])) if ideg is not None else None
                self.xb.ad_hoc_build_id_mapping(j, ids.numpy())
            self._pp(f"rank:{r:02d}  NUM_HALO: {uniq.shape[0]}")
        self.part_src = torch.cat(srcs)
        self.part_dst = torch.cat(dsts)
        self._pp(f"rank:{r:02d} RELOADING: {time.time() - tic:.2f} s")

    def build_partition_v2_t10n(self):
        tic = time.time()
        self.cur_g = host().graph.HostGraph(self.part_src.numpy(), self.part_dst.numpy(), self.prefix_sum[-1],
                                            self.node_id)
        self._pp(f"rank:{self.rank:02d} NUM_EDGES: {self.part_src.shape[0]}")
        self._pp(f"rank:{self.rank:02d} BLD_GRAPH: {time.time() - tic:.2f} s")

    def load_nbr_chunk(self, nbr_idx):
        """The reference's first working-set form (t10n/dataloader.py:452-490): this
        partition and ``nbr_idx``'s in local numbering (own nodes [0, n0), the
        neighbour's [n0, n0 + n1)), with only the bridges from the neighbour into this
        partition; no halo.  Sets p1_u/p1_v, b01_u/b01_v, feat_1 and label_1."""
        n0 = int(self.label_0.shape[0])
        u = self.io.part(nbr_idx, "u")
        v = self.io.part(nbr_idx, "v")
        self.p1_u = torch.from_numpy(u) + n0
        self.p1_v = torch.from_numpy(v) + n0
        bu, bv = self.io.bridge(nbr_idx, self.rank)
        if bu is None:
            self.b01_u = torch.empty(0, dtype=torch.int64)
            self.b01_v = torch.empty(0, dtype=torch.int64)
        else:
            self.b01_u = torch.from_numpy(bu) + n0
            self.b01_v = torch.from_numpy(bv)
        self.feat_1 = torch.from_numpy(self.io.part(nbr_idx, "nfeat"))
        self.label_1 = torch.from_numpy(self.io.part(nbr_idx, "label"))
        self.nbr_idx = nbr_idx

    def build_partition(self):
        """Host graph of the first working-set form (own intra edges, bridges from the
        neighbour, the neighbour's intra edges; local ids) and its feature rows
        (t10n/dataloader.py:492-502)."""
        n = int(self.label_0.shape[0] + self.label_1.shape[0])
        src = torch.cat([self.p0_u, self.b01_u, self.p1_u])
        dst = torch.cat([self.p0_v, self.b01_v, self.p1_v])
        self.cur_g = host().graph.HostGraph(src.numpy(), dst.numpy(), n, self.node_id)
        self.cur_node_feat = torch.cat([self.feat_0, self.feat_1], 0)
        self._pp(f"rank:{self.rank:02d} NUM_EDGES_v1: {src.shape[0]}")

    def build_partition_v2(self):
        """The working graph of load_nbr_chunk_v2 (global ids), as a host graph."""
        self.build_partition_v2_t10n()

    def next_nbr(self):
        nbr = (self.nbr_idx + 1) % self.world
        if nbr == self.rank:
            nbr = (nbr + 1) % self.world
        return nbr

    def get_cur_dataloader(self, args, epoch, overide_exp_mode=-1):
        if self.dataloader is None or epoch % int(args.repart_every) == 0:
            self.nbr_idx = self.next_nbr() if self.world > 1 else self.rank
            self.load_nbr_chunk_v2(self.nbr_idx)
            self.build_partition_v2_t10n()
            self.dataloader = self._make_sampler(args)
        return self.dataloader

    def _make_sampler(self, args):
        if self.model_name == "pinsage":
            from grappa_b200.pinsage_sampler import HostPinSAGESampler

            return HostPinSAGESampler(self.cur_g, self.train_nid, int(args.num_layers), batch_size=self.adjust_bs,
                                      shuffle=True, use_batch_n=self.get_max_step(), seed=self.seed)
        gideg = self.ideg_0[self.train_nid - self.prefix_sum[self.rank]]
        return HostBatchSamplerWithCounter(self.cur_g, self.train_nid, self.fanouts, repeated=False,
                                           batch_size=self.adjust_bs, shuffle=True, target_nodes_gideg=gideg,
                                           use_batch_n=self.get_max_step(), seed=self.seed)

    # ------------------------------------------------------------------ batch data
    def set_coarse_count(self, coarse_count):
        self.batch_coarse_count = coarse_count

    def get_coarse_count(self):
        if isinstance(self.dataloader, HostBatchSamplerWithCounter):
            return min(float(self.dataloader.get_cur_resampling_cnt()), self.max_coarse_count)
        return 0.0

    def get_batch_input(self, batch_input, input_nodes):
        tables = [None if t is None else t.numpy() for t in self.feat_n]
        self.xb.ad_hoc_fill_batch_feat(batch_input.numpy(), tables, input_nodes.cpu().numpy())
        return batch_input

    def get_batch_gideg(self, batch_input, input_nodes):
        tables = [None if t is None else t.numpy() for t in self.ideg_n]
        self.xb.ad_hoc_fill_batch_ideg(batch_input.numpy(), tables, input_nodes.cpu().numpy())
        return batch_input

    def get_batch_labels(self, seed):
        return self.node_label[seed.cpu() - self.prefix_sum[self.rank]]

    def get_node_label(self):
        return self.node_label

    def get_rank(self):
        return self.rank

    def get_max_step(self):
        return self.local_batch

    def get_comm_dev(self):
        return self.da.comm_dev()

    def get_num_node(self):
        return self.part_num_node[self.rank]

    def get_nid_offset(self):
        return self.prefix_sum[self.rank]

    def get_node_subset(self, subset_tag):
        if subset_tag == "all":
            return torch.cat((self.train_nid, self.valid_nid, self.test_nid))
        if subset_tag == "train":
            return self.train_nid
        if subset_tag == "valid":
            return self.valid_nid
        if subset_tag == "test":
            return self.test_nid
        raise ValueError(f"{subset_tag} is unknown")

    # ------------------------------------------------------------------ cross-border inference
    def xb_dataloader(self, args, force_even=True, full_neighbor=False, subset_tag="all"):
        fanouts = [-1 if full_neighbor else f for f in self.fanouts]
        return HostXBBatchSampler(self.cur_g, self.get_node_subset(subset_tag), fanouts,
                                  batch_size=int(args.batch_size_eval), shuffle=False, xb=self.xb, rank=self.rank,
                                  num_part=self.num_part, device_allocator=self.da, seed=self.seed)

    def xb_dataloader_per_layer(self, args, subset_tag="all"):
        target = self.get_node_subset(subset_tag)
        n_batch = (target.shape[0] + int(args.batch_size_eval) - 1) // int(args.batch_size_eval)
        max_batch = _all_reduce_max(n_batch, self.da.comm_dev())
        # every rank runs the same number of all-to-all rounds: pad with empty batches
        bs = max(1, (target.shape[0] + max_batch - 1) // max_batch) if max_batch else 1
        loader = HostXBBatchSampler(self.cur_g, target, [np.iinfo(np.int64).max], batch_size=bs, shuffle=False,
                                    xb=self.xb, rank=self.rank, num_part=self.num_part, device_allocator=self.da,
                                    seed=self.seed)
        loader.use_batch_n = max_batch
        return loader

    @timing
    def xb_get_batch_input(self, batch_input, target_nodes):
        return xb_gather(self.xb, self.da.comm_dev(), batch_input, target_nodes, self.feat_0, self.rank,
                         self.num_part, self.prefix_sum)

    def xb_get_batch_emb(self, batch_input, target_nodes, emb_self):
        return xb_gather(self.xb, self.da.comm_dev(), batch_input, target_nodes, emb_self, self.rank, self.num_part,
                         self.prefix_sum)

    def xb_scatter_emb(self, emb, target_nodes, emb_self):
        return xb_scatter(self.xb, self.da.comm_dev(), emb, target_nodes, emb_self, self.rank, self.num_part,
                          self.prefix_sum)

    def infer_train_mask_of(self, seeds):
        return self.train_mask[seeds.cpu() - self.prefix_sum[self.rank]]

    def infer_valid_mask_of(self, seeds):
        return self.valid_mask[seeds.cpu() - self.prefix_sum[self.rank]]

    def infer_test_mask_of(self, seeds):
        return self.test_mask[seeds.cpu() - self.prefix_sum[self.rank]]
