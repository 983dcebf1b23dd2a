"""Device neighbour sampler: multi-hop sampling + block compaction on the GPU.

The reference declares GpuSampler / GpuBatchSampler but leaves them empty
(csrc/python/py_graph.h:117-122, t10n/sampler.py:182-191) and samples on the
host.  ``GpuNeighborSampler`` is the working device version with the same
semantics as the host sampler (csrc/graph/sampling_h.h, csrc/python/py_graph.cc):
per hop it runs the S1 sampling kernel and the three S2 compaction kernels with
static, capacity-sized buffers and device-side counts, so it never synchronises
with the host and can be captured in a CUDA graph.
"""
import torch

from grappa_b200 import _native
from grappa_b200.block import Block

# counters layout shared with the engine: [seed, epoch, step_in_epoch, global_step, gen, adam_t]
C_SEED, C_EPOCH, C_STEP, C_GLOBAL, C_GEN, C_ADAM = range(6)


def new_counters(seed, device):
    c = torch.zeros(6, dtype=torch.int64, device=device)
    c[C_SEED] = int(seed)
    return c


def hop_capacities(batch_size, fanouts, n_nodes_cap):
    """Capacities (dst, edges, src) of every hop, seed hop first; fanouts are given input
    layer first as in the reference (the seed hop uses fanouts[-1])."""
    L = len(fanouts)
    cap_dst, cap_e, cap_src = [], [], []
    d = int(batch_size)
    for h in range(L):
        f = int(fanouts[L - 1 - h])
        if f < 0:
            raise ValueError("full-neighbour hops need an explicit edge capacity")
        e = d * f
        s = min(d + e, int(n_nodes_cap))
        cap_dst.append(d)
        cap_e.append(max(1, e))
        cap_src.append(max(s, d))
        d = cap_src[-1]
    return cap_dst, cap_e, cap_src


class GpuNeighborSampler:
    def __init__(self, fanouts, batch_size, n_nodes_cap, device, cu=None, replace=False, transpose_hops=()):
        self.cu = cu if cu is not None else _native.cuda()
        self.fanouts = [int(f) for f in fanouts]
        self.L = len(self.fanouts)
        self.B = int(batch_size)
        self.replace = bool(replace)
        self.device = torch.device(device)
        self.n_nodes_cap = int(n_nodes_cap)
        dev = self.device
        i32 = dict(dtype=torch.int32, device=dev)
        L = self.L
        self.cap_dst, self.cap_e, self.cap_src = hop_capacities(self.B, self.fanouts, self.n_nodes_cap)
        self.cnt = torch.zeros(1 + 3 * L, **i32)  # [n_seeds, (n_edges, n_src, spare) per hop]
        self.seeds = torch.zeros(self.B, **i32)
        self.seed_gideg = torch.zeros(self.B, dtype=torch.int64, device=dev)
        self.indptr = [torch.zeros(self.cap_dst[h] + 1, **i32) for h in range(L)]
        self.nbr = [torch.zeros(self.cap_e[h], **i32) for h in range(L)]
        self.indices = [torch.zeros(self.cap_e[h], **i32) for h in range(L)]
        self.src = [torch.zeros(self.cap_src[h], **i32) for h in range(L)]
        self.sampled = [torch.zeros(self.cap_src[h], dtype=torch.uint8, device=dev) for h in range(L)]
        self.sscr = [torch.zeros(self.cu.sample_scratch_words(self.cap_dst[h]), dtype=torch.int64, device=dev)
                     for h in range(L)]
        self.cscr = [torch.zeros(self.cu.compact_scratch_words(self.cap_e[h]), dtype=torch.int64, device=dev)
                     for h in range(L)]
        # dense tagged id map of the compaction (never cleared: tags decrease call to call)
        self.map = torch.full((self.n_nodes_cap,), -1, dtype=torch.int64, device=dev)
        self.err = torch.zeros(1, **i32)
        # blocks also kept grouped by source (CSR by local src) for the gathered backward
        self.transpose_hops = tuple(int(h) for h in transpose_hops)
        self.t_cnt, self.t_rank, self.tptr, self.tdst = {}, {}, {}, {}
        for h in self.transpose_hops:
            self.t_cnt[h] = torch.zeros(self.cap_src[h], **i32)
            self.t_rank[h] = torch.zeros(self.cap_e[h], **i32)
            self.tptr[h] = torch.zeros(self.cap_src[h] + 1, **i32)
            self.tdst[h] = torch.zeros(self.cap_e[h], **i32)

    # device counters ------------------------------------------------------------------
    def n_seeds(self):
        return self.cnt[0:1]

    def n_edges(self, h):
        return self.cnt[1 + 3 * h:2 + 3 * h]

    def n_src(self, h):
        return self.cnt[2 + 3 * h:3 + 3 * h]

    def n_dst(self, h):
        return self.n_seeds() if h == 0 else self.n_src(h - 1)

    def dst(self, h):
        return self.seeds if h == 0 else self.src[h - 1]

    # sampling --------------------------------------------------------------------------
    def sample(self, indptr, indices, counters, gideg=None, cov=None, err=None, seed_gideg_ready=False):
        """Sample every hop from ``self.seeds[:cnt[0]]`` on the graph (indptr int64 [n+1],
        indices int32).  ``counters`` (device int64 [6]) supplies seed/epoch/step for the
        Philox keys and the compaction tag generation; gideg (per node, int64) and cov
        (float [2]) enable the coverage counter of the seed hop; ``seed_gideg_ready`` says
        that the seeds' in-degrees are already in ``seed_gideg`` (the engine's step
        prologue gathers them)."""
        cu = self.cu
        err = self.err if err is None else err
        if indptr.numel() - 1 > self.n_nodes_cap:
            raise ValueError("graph larger than the sampler's node capacity")
        if gideg is not None and not seed_gideg_ready:
            cu.gather_scalar(gideg, self.seeds, self.n_seeds(), 0, self.B, self.seed_gideg)
        for h in range(self.L):
            dst = self.dst(h)
            front = None if h == 0 else self.sampled[h - 1]
            # the hop kernel also does the compaction's first pass (map entries of the
            # block's nodes), so the compaction starts at its scan
            cu.sample_hop(indptr, indices, dst, self.n_dst(h), 0, front, self.fanouts[self.L - 1 - h], self.replace,
                          counters, h, self.seed_gideg if (h == 0 and gideg is not None) else None,
                          cov if h == 0 else None, self.indptr[h], self.nbr[h], self.n_edges(h), self.sscr[h], err,
                          self.cap_dst[h], self.map, self.src[h], self.sampled[h])
            tr = h in self.t_cnt
            # without block transposes every hop's edge rewrite (K3) waits for one launch
            # after the last hop (compact_edges): the next hop needs only K2's outputs
            cu.compact(dst, self.n_dst(h), self.nbr[h], self.n_edges(h), self.map, self.src[h], self.sampled[h],
                       self.indices[h], self.n_src(h), self.cscr[h], err, self.cap_dst[h], self.cap_e[h], counters, h,
                       True, self.t_cnt.get(h), self.t_rank.get(h), run_k3=tr)
            if tr:
                cu.block_transpose(self.indptr[h], self.indices[h], self.n_dst(h), self.n_src(h), self.t_cnt[h],
                                   self.t_rank[h], self.tptr[h], self.tdst[h], err)
        # the hops without a transpose get their edge rewrite here, in one launch
        late = [h for h in range(self.L) if h not in self.t_cnt]
        if late:
            cu.compact_edges([self.nbr[h] for h in late], [self.n_edges(h) for h in late],
                             [self.indices[h] for h in late], [self.cap_src[h] for h in late], self.map)

    def blocks(self):
        """Materialise the sampled blocks (input layer first) with exact sizes (host sync)."""
        cnt = self.cnt.cpu().tolist()
        out = []
        for h in range(self.L - 1, -1, -1):
            nd = cnt[0] if h == 0 else cnt[2 + 3 * (h - 1)]
            ne, ns = cnt[1 + 3 * h], cnt[2 + 3 * h]
            out.append(Block(self.indptr[h][: nd + 1].clone(), self.indices[h][:ne].clone(), self.src[h][:ns].clone(),
                             nd, ns, self.sampled[h][:ns].clone()))
        return out

    def load_seeds(self, seeds):
        """Eager helper: seeds (int tensor on any device) -> static buffer + count."""
        n = int(seeds.numel())
        if n > self.B:
            raise ValueError("more seeds than the batch capacity")
        self.seeds[:n].copy_(seeds.to(self.device, torch.int32))
        self.cnt[0] = n
