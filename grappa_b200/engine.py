"""Mini-batch and full-graph training engines on the sm_100a kernels.

One training step of a block GNN, entirely on the device:

  for hop h = 0..L-1 (seed hop first, fanouts reversed as in the reference):
      S1  sample_hop / walk_hop  pick counts + look-back scan + Philox picks (or the
                                 PinSAGE random walks + top-k visited)
      S2  compact                dst-first relabelling with a dense tagged id map
  layer l = 0..L-1 (input layer first, on hop h = L-1-l): the model's layer kernels
  backward, last layer first: the transposed kernels, fp32 reductions
  K-AR   coverage-weighted all-reduce + Adam over NVLink peer memory (W > 1), or Adam

Layer programs (kernels in grappa_b200/csrc/cuda):
  SAGE     aggregate [h_dst | mean h_src] -> tcgen05 GEMM (+bias, ReLU, dropout; or the
           fused softmax cross-entropy of the last layer)
  GCN      in <= out: aggregate (sym. norm) -> GEMM;  in > out: GEMM over the source
           rows -> aggregate with the bias/ReLU/dropout epilogue (DGL's order)
  GIN      aggregate (sum + self) -> GEMM -> BatchNorm+ReLU -> GEMM -> BatchNorm+ReLU
  GAT      GEMM over the source rows -> attention logits -> fused edge softmax +
           weighted sum (+ReLU, dropout; head mean on the last layer)
  PinSAGE  dropout -> GEMM (+bias, ReLU) over the sources -> weighted mean over the
           random-walk neighbours -> [agg | h_dst] -> GEMM (+bias, ReLU) -> L2 norm

Every buffer is allocated once at its capacity (batch size times the fanout
products); the kernels read the live sizes from device counters, so the step has
no host synchronisation and is captured once into a CUDA graph and replayed.
Full-graph training uses the same engines with ``FullGraphBlocks`` (the working
graph as a fixed block for every layer) in place of the sampler.
"""
import math
import os

import torch

from grappa_b200 import _native
from grappa_b200.models.flat import pad8
from grappa_b200.sampler_gpu import C_EPOCH, C_STEP, GpuNeighborSampler, new_counters

GEMM_STORE_BF16, GEMM_STORE_F32, GEMM_ATOMIC_F32, GEMM_CROSS_ENTROPY = 0, 1, 2, 3
AGG_MEAN, AGG_SUM, AGG_GCN, AGG_WEIGHTED = 0, 1, 2, 3
# GAT input layer.  "x": attention on the input rows, projection after the aggregation
# (el = x.wl, y_v[h] = sum a_uv x_u, out = y Wbd^T: no per-source z = x W^T and no
# per-source dz, but H * in instead of H * F multiply-adds per edge); "bwd": z = x W^T
# forward, dW from attention-weighted input rows in the backward; "auto" (default): "x"
# when in <= F, else "bwd" (4 heads x 64 on 128 input columns measured 1.18 s/epoch
# with "x" against 0.93 with "bwd"); "0": the plain z / dz path (for comparisons)
GAT_INPUT_MODE = os.environ.get("GRAPPA_GAT_INPUT", os.environ.get("GRAPPA_GAT_INPUT_BWD", "auto"))
GAT_INPUT_LAYER_BWD = GAT_INPUT_MODE != "0"
# GAT attention logits el / er reduced in the epilogue of the z = x W^T GEMM (1) or by
# a separate pass over z (0, the default: the longer GEMM epilogue measured 0.977
# s/epoch on the 111M-node workload against 0.923 with the separate pass)
GAT_FUSED_LOGITS = os.environ.get("GRAPPA_GAT_FUSED_LOGITS", "0") != "0"
# GraphSAGE backward gathered by source over the block transpose (1) or scattered with
# fp32 reductions plus a separate activation pass (0, the default: the transposes add
# two kernels per hop to the sampling stream, which measured slower overall)
# "0" (default), "1" (every hop) or "inner" (the hops the fused output layer does not
# cover; measured 0.0366 against 0.0358 s/epoch with the default)
SAGE_GATHER_BWD = os.environ.get("GRAPPA_SAGE_GATHER_BWD", "0")
# output tiles per SM the GEMM tile width aims for (gemm_bn)
GEMM_CTAS_PER_SM = float(os.environ.get("GRAPPA_GEMM_TILES_PER_SM", "2"))
# GraphSAGE output layer (aggregation, logits, cross-entropy, dlogits and dX) as one
# CUDA-core kernel (csrc/cuda/head.cu) instead of an aggregation, a tensor-core GEMM
# with a cross-entropy epilogue on a handful of SMs and a dX GEMM
SAGE_FUSED_HEAD = os.environ.get("GRAPPA_SAGE_HEAD", "1") != "0"
# hidden GraphSAGE layers after the first as 16-row MMA tile kernels (aggregation +
# projection forward; projection transpose + aggregation backward) instead of an
# aggregation and a tcgen05 GEMM each way.  Off by default: at 3250 rows x 256 x 512
# they are 408 CTAs that each load a 133 KB slice of W (one CTA per SM, three waves),
# and the epoch measured 0.0397 s against 0.0362 with the tcgen05 path
SAGE_TILE_LAYERS = os.environ.get("GRAPPA_SAGE_TILE_LAYERS", "0") != "0"
# stream priorities inside the step graphs: the layer chain, the weight gradients and
# the updates at the highest priority, the next step's sampling at the lowest
STREAM_PRIORITY = os.environ.get("GRAPPA_STREAM_PRIORITY", "1") != "0"
# one rank: Adam per layer on the comm stream during the backward pass (1, the default)
# or one Adam pass after it (0)
ADAM_PER_LAYER = os.environ.get("GRAPPA_ADAM_PER_LAYER", "1") != "0"


def _stream(device, high):
    if not STREAM_PRIORITY:
        return torch.cuda.Stream(device=device)
    lo, hi = torch.cuda.Stream.priority_range()
    return torch.cuda.Stream(device=device, priority=hi if high else lo)

# kernels launched by each binding (memsets excluded)
KERNELS_PER_CALL = {
    "sample_hop": 1, "walk_hop": 1, "compact": 3, "gemm": 1, "aggregate": 1, "aggregate_bwd": 1, "act_bwd": 1,
    "gather_scalar": 1, "gather_rows": 1, "adam": 1, "step_end": 1, "src_norm": 2,
    "pull_rows": 1, "csr_merge": 1, "mark_ids": 1, "iota_map": 1, "mark_compact": 1, "peer_copy": 1, "a2a_pull": 1, "peer_barrier": 1,
    "shuffle_keys": 1, "sample_prologue": 1, "cross_entropy": 1, "batchnorm_fwd": 2, "batchnorm_bwd": 2, "l2norm_fwd": 1,
    "l2norm_bwd": 1, "dropout_rows": 1, "dropout_grad": 1, "f32_to_bf16_rows": 1, "add_bf16_rows": 1,
    "gat_scores": 1, "gat_fwd": 1, "gat_bwd": 2, "gat_bwd_input": 2, "gat_dw_combine": 1, "sampler_counters": 1,
    "gat_in_scores": 1, "gat_in_fwd": 1, "gat_in_bwd": 2, "gat_in_prep": 1, "gat_in_dw": 1, "col_sum_bf16": 1,
    "block_transpose": 2, "aggregate_bwd_gather": 1, "sage_head": 1, "compact_edges": 1, "sage_layer_fwd": 1,
    "sage_layer_bwd": 1,
}


class LaunchCounter:
    """Proxy of the kernel module that counts the kernels each call launches."""

    def __init__(self, mod):
        self._mod = mod
        self.count = 0
        # a list: every counted call appends (name, start event, end event) recorded on
        # the current stream around it (eager steps only: events cannot be recorded
        # inside a graph capture and read back per launch)
        self.timer = None

    def __getattr__(self, name):
        f = getattr(self._mod, name)
        k = KERNELS_PER_CALL.get(name, 0)
        if not k:
            return f

        def wrapped(*a, **kw):
            n = k
            if name == "compact" and ((len(a) > 15 and a[15]) or kw.get("k1_done")):
                n -= 1  # the first pass ran inside the sampling kernel
            if name == "compact" and kw.get("run_k3") is False:
                n -= 1  # the edge rewrite runs in compact_edges
            self.count += n
            if self.timer is None:
                return f(*a, **kw)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            r = f(*a, **kw)
            e1.record()
            self.timer.append((name, e0, e1))
            return r

        return wrapped


def bn_for(n, mn_major=False):
    """Tile width of the GEMM for an output width n (48 only with K-major B)."""
    if n == 48 and not mn_major:
        return 48
    if n <= 64:
        return 64
    if n <= 128:
        return 128
    return 256


def gemm_bn(M_cap, N, mn_major=False, sms=148):
    """Tile width for an M_cap x N output: the widest tile (fewest B re-reads, longest
    rows per epilogue thread) that still gives about two CTAs per SM, assuming a third
    of the row capacity is live (block sizes are a fraction of their capacity)."""
    bn = bn_for(N, mn_major)
    if bn == 48:
        return bn
    mt = math.ceil(max(1, M_cap // 3) / 128)
    while bn > 64 and mt * math.ceil(N / bn) < GEMM_CTAS_PER_SM * sms:
        bn //= 2
    return bn


def dropout_scale(p):
    """Scale of the kept values of the kernels' dropout masks: the probability is
    quantised to t / 256 (byte-resolution masks, grappa/rng.h), t = round(256 p)."""
    if p <= 0:
        return 1.0
    t = min(255, max(0, int(p * 256.0 + 0.5)))
    return 256.0 / (256 - t)


def split_k(rows, n_tiles, sms=148, min_kblocks=8):
    """Number of split-K slices for a dW GEMM over ``rows`` reduction rows."""
    kblocks = max(1, math.ceil(rows / 64))
    by_work = max(1, kblocks // min_kblocks)
    by_sms = max(1, (2 * sms) // max(1, n_tiles))
    return max(1, min(by_work, by_sms))


# ---------------------------------------------------------------------- block sources
class FullGraphBlocks:
    """The working graph's own + neighbour rows as one fixed block used by every layer
    (isolated full-graph training, reference experiments/grappa/train/
    t10n_fullgraph_train.py:163-205): dst = src = rows [0, n), edges = in-edges among
    them.  Same interface as GpuNeighborSampler; ``sample`` does nothing."""

    def __init__(self, indptr, indices, n_layers, device, labels, train_rows, cov=None, cap_nodes=0, cap_edges=0):
        dev = torch.device(device)
        self.device = dev
        self.L = int(n_layers)
        n, E = int(indptr.numel() - 1), int(indices.numel())
        # buffers sized for the largest working graph a repartition can produce, so that
        # ``refill`` keeps every pointer (and the engine's captured step graph) valid
        cap_n, cap_e = max(n, int(cap_nodes)), max(1, E, int(cap_edges))
        self.B = cap_n
        i32 = dict(dtype=torch.int32, device=dev)
        self.cnt = torch.zeros(1 + 3 * self.L, **i32)
        self.seeds = torch.arange(cap_n, **i32)
        ip = torch.zeros(cap_n + 1, **i32)
        ix = torch.zeros(cap_e, **i32)
        self.indptr = [ip] * self.L
        self.indices = [ix] * self.L
        self.src = [self.seeds] * self.L
        self.cap_dst = [cap_n] * self.L
        self.cap_src = [cap_n] * self.L
        self.cap_e = [cap_e] * self.L
        self.w = [None] * self.L
        self.labels = torch.zeros(cap_n, **i32)
        self.row_mask = torch.zeros(cap_n, dtype=torch.uint8, device=dev)
        self.n_sel = torch.zeros(1, **i32)
        # [coverage sum, count] of the partition's training rows (weight 1 when not given)
        self.cov = torch.ones(2, dtype=torch.float32, device=dev)
        self.full_graph = True
        self.refill(indptr, indices, labels, train_rows, cov)

    def refill(self, indptr, indices, labels, train_rows, cov=None):
        """Load another working graph into the same buffers (False when it does not fit):
        rows [0, n) and the n + 1 row pointers, the edges, labels, training rows and
        coverage; the live sizes go to the device counters the kernels read."""
        n, E = int(indptr.numel() - 1), int(indices.numel())
        if n > self.cap_dst[0] or E > self.cap_e[0]:
            return False
        self.n = n
        ip, ix = self.indptr[0], self.indices[0]
        ip[: n + 1].copy_(indptr)
        ip[n + 1:].fill_(E)
        ix[:E].copy_(indices)
        self.labels[:n].copy_(labels)
        self.row_mask.zero_()
        self.row_mask[:n].copy_(train_rows)
        self.n_sel.copy_(self.row_mask.sum().to(torch.int32).view(1))
        if cov is None:
            self.cov.fill_(1.0)
        else:
            self.cov.copy_(cov)
        self.cnt.copy_(torch.tensor([n] + [E, n, 0] * self.L, dtype=torch.int32))
        return True

    def n_seeds(self):
        return self.cnt[0:1]

    def n_edges(self, h):
        return self.cnt[1 + 3 * h:2 + 3 * h]

    def n_src(self, h):
        return self.cnt[2 + 3 * h:3 + 3 * h]

    def n_dst(self, h):
        return self.n_seeds() if h == 0 else self.n_src(h - 1)

    def sample(self, *args, **kwargs):
        return None


class GpuWalkSampler(GpuNeighborSampler):
    """PinSAGE sampler on the GPU: per hop walk_hop (random walks + top-k visited,
    grappa_b200/csrc/cuda/walk.cu) then the S2 compaction; the visit counts are the
    edge weights ``w[h]`` in the block's edge order."""

    def __init__(self, n_layers, batch_size, n_nodes_cap, device, cu=None, length=None, restart_prob=0.5,
                 num_walks=4, num_neighbors=5):
        super().__init__([num_neighbors] * int(n_layers), batch_size, n_nodes_cap, device, cu=cu)
        self.length = int(length if length is not None else n_layers)
        self.restart_prob = float(restart_prob)
        self.num_walks = int(num_walks)
        self.num_neighbors = int(num_neighbors)
        self.w = [torch.zeros(self.cap_e[h], dtype=torch.float32, device=self.device) for h in range(self.L)]
        self.wscr = [torch.zeros(self.cu.walk_scratch_words(self.cap_dst[h]), dtype=torch.int64, device=self.device)
                     for h in range(self.L)]

    def sample(self, indptr, indices, counters, gideg=None, cov=None, err=None, seed_gideg_ready=False):
        cu = self.cu
        err = self.err if err is None else err
        for h in range(self.L):
            dst = self.dst(h)
            cu.walk_hop(indptr, indices, dst, self.n_dst(h), 0, self.length, self.restart_prob, self.num_walks,
                        self.num_neighbors, counters, h, self.indptr[h], self.nbr[h], self.w[h], self.n_edges(h),
                        self.wscr[h], err, self.cap_dst[h])
            cu.compact(dst, self.n_dst(h), self.nbr[h], self.n_edges(h), self.map, self.src[h], self.sampled[h],
                       self.indices[h], self.n_src(h), self.cscr[h], err, self.cap_dst[h], self.cap_e[h], counters, h)

    def blocks(self):
        out = super().blocks()
        cnt = self.cnt.cpu().tolist()
        for b, h in zip(out, range(self.L - 1, -1, -1)):
            b.edata["weights"] = self.w[h][: cnt[1 + 3 * h]].clone()
        return out


# ---------------------------------------------------------------------- engines
class BlockEngine:
    """Shared parts: parameters (flat fp32 master, bf16 working copy, gradient, Adam
    moments), device counters, the block source, the optimizer step, CUDA-graph
    capture.  Subclasses implement ``_alloc_layers``, ``_forward`` and ``_backward``."""

    model_name = None

    def __init__(self, model, n_nodes_cap, fanouts, batch_size, device, lr=3e-3, comm=None, seed=0,
                 fused_allreduce=True, use_cuda_graph=True, betas=(0.9, 0.999), eps=1e-8, blocks=None,
                 overlap_sampling=True, overlap_allreduce=True, ar_mode=None):
        if getattr(model, "name", None) != self.model_name:
            raise ValueError(f"{type(self).__name__} trains {self.model_name} models")
        self.cu = LaunchCounter(_native.cuda())
        self.launches_per_step = 0
        self.model = model
        self.comm = comm
        self.world = 1 if comm is None else comm.world
        self.rank = 0 if comm is None else comm.rank
        self.fanouts = [int(f) for f in fanouts]
        self.L = len(model.layers)
        if blocks is None and len(self.fanouts) != self.L:
            raise ValueError("one fanout per layer")
        self.lr, self.betas, self.eps = float(lr), betas, float(eps)
        self.p = float(getattr(model, "dropout_p", 0.0))
        self.device = torch.device(device)
        self.seed = int(seed)
        self.use_cuda_graph = use_cuda_graph
        self.fused_allreduce = fused_allreduce and self.world > 1
        dev = self.device

        model.place(dev)
        self.allreduce = None
        self._ar_by_layer = False
        if self.fused_allreduce:
            # gradient and fp32 master weights in peer-mapped buffers; one bucket per layer
            # (launched as the backward pass completes the layer) when the layers' segments
            # are contiguous, else one bucket after the backward pass
            from grappa_b200.parallel.allreduce import FusedAllReduceAdam

            buckets = model.layer_buckets(self.L) if overlap_allreduce else None
            self._ar_by_layer = buckets is not None
            nb = 1 if buckets is None else len(buckets)
            modes = None if ar_mode is None else [{"one_shot": 0, "shard": 1}[ar_mode]] * nb
            self.allreduce = FusedAllReduceAdam(comm, model.flat.numel(), buckets, modes=modes)
            self.allreduce.adopt_params(model)
            self.grad = self.allreduce.grad
        else:
            self.grad = torch.zeros_like(model.flat)
        self.flat = model.flat
        self.wbf = self.flat.to(torch.bfloat16)
        self.m = torch.zeros_like(self.flat)
        self.v = torch.zeros_like(self.flat)

        self.counters = new_counters(self.seed, dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.fstats = torch.zeros(4, dtype=torch.float32, device=dev)  # cov_sum, cov_n, loss_sum, spare
        self.istats = torch.zeros(2, dtype=torch.int32, device=dev)   # correct, spare
        self._ce_dummy = torch.zeros((1, 1), dtype=torch.float32, device=dev)
        # device slots read by the step graphs: [address of the epoch's seed table (0 =
        # seeds loaded by the host), address of the per-step loss ring (0 = none)]
        self._slots = torch.zeros(2, dtype=torch.int64, device=dev)
        self._count_table = torch.zeros(1, dtype=torch.int32, device=dev)
        self._seed_table = None
        if self.allreduce is not None:
            self.allreduce.bind(self.counters, self.m, self.v, self.wbf, self.lr, self.betas, self.eps, self.err)
        # one rank: Adam per layer on the comm stream as soon as the layer's gradient is
        # complete (the same overlap as the per-layer all-reduce)
        self._adam_slices = None
        self._launched = set()
        if self.world == 1 and overlap_allreduce and ADAM_PER_LAYER:
            buckets = model.layer_buckets(self.L)
            if buckets is not None:
                self._adam_slices = [tuple(t[lo:hi] for t in (self.flat, self.m, self.v, self.grad, self.wbf))
                                     for lo, hi in buckets]

        # block sources: with CUDA graphs two samplers alternate, so that the next
        # step's sampling (a side stream inside the step graph) overlaps this step's
        # layers; the eager path uses the first one only
        if blocks is None:
            n = 2 if (use_cuda_graph and overlap_sampling) else 1
            samplers = [self._make_sampler(int(batch_size), int(n_nodes_cap), dev) for _ in range(n)]
        else:
            samplers = [blocks]
        self.n_classes = model.n_classes
        self._working = None
        self._set_samplers(samplers)

    def _set_samplers(self, samplers):
        dev = self.device
        self.samplers = samplers
        self.full_graph = getattr(samplers[0], "full_graph", False)
        self.B = samplers[0].B
        self.scnt = [new_counters(self.seed, dev) for _ in samplers]      # per-sampler draw counters
        self.covs = [torch.zeros(2, dtype=torch.float32, device=dev) for _ in samplers]
        self.seed_labels = [torch.zeros(self.B, dtype=torch.int32, device=dev) for _ in samplers]
        self._select(0)
        self.lay = []
        self._alloc_layers()
        self._graph = None
        self._graphs = {}

    def _select(self, p):
        """Make sampler p the one whose blocks the layers run on."""
        self.p_cur = p
        self.sm = self.samplers[p]
        self.seeds = self.sm.seeds
        self.seed_label = self.seed_labels[p]
        self.cov_cur = self.covs[p]

    def _make_sampler(self, batch_size, n_nodes_cap, dev):
        return GpuNeighborSampler(self.fanouts, batch_size, n_nodes_cap, dev, cu=self.cu)

    def set_blocks(self, blocks):
        """Replace a fixed block source (full-graph training after a repartition) and
        re-size the layer buffers; parameters and optimizer state are kept."""
        self._set_samplers([blocks])

    # ------------------------------------------------------------------ helpers
    def _seg(self, name, buf=None):
        return self.model.segment(name).view(self.flat if buf is None else buf)

    def _n_dst(self, h):
        return self.sm.n_dst(h)

    def _input(self, l):
        """(rows, src_map) that layer l aggregates from."""
        h = self.L - 1 - l
        if l == 0:
            return self._working.feat, (None if self.full_graph else self.sm.src[h])
        return self.lay[l - 1]["H"], None

    def _gathered_input(self, l, s):
        """Source rows of layer l as a contiguous GEMM operand."""
        h = self.L - 1 - l
        if l > 0:
            return self.lay[l - 1]["H"]
        if self.full_graph:
            return self._working.feat
        self.cu.gather_rows(self._working.feat, self.sm.src[h], self.sm.n_src(h), 0, self.sm.cap_src[h], s["ip"],
                            s["Xg"])
        return s["Xg"]

    def _labels_rows(self):
        if self.full_graph:
            return self.sm.labels, self.sm.row_mask, self.sm.n_sel
        return self.seed_label, None, None

    def _ce(self, logits, C, dl, dbias, h):
        labels, mask, n_sel = self._labels_rows()
        self.cu.cross_entropy(logits, C, labels, self._n_dst(h), self.sm.cap_dst[h], mask, n_sel, dl, dbias,
                              self.fstats[2:3], self.istats[0:1])

    def _gemm(self, A, a_mn, B, b_mn, M_cap, M_dev, N, K_cap, K_dev, splits, C, mode, bias=None, act=0, p=0.0,
              salt=0, bn=None, act_mask=None, mask_scale=1.0, zero_tail_rows=0, att=None):
        """``att`` = (att_l, att_r, el, er, heads, feat, n_dst): GAT attention logits of
        the stored bf16 rows reduced into el / er (zeroed by the caller) in the epilogue."""
        bn = bn or gemm_bn(M_cap, N, b_mn)
        kw = {}
        if att is not None:
            kw = dict(att_l=att[0], att_r=att[1], att_el=att[2], att_er=att[3], att_heads=att[4], att_feat=att[5],
                      att_n_dst=att[6])
        self.cu.gemm(A, a_mn, B, b_mn, M_cap, M_dev, N, K_cap, K_dev, splits, C, mode, bias, act, p,
                     self.counters if p > 0 else None, salt, None, 0, None, None, None, None, None, None, self.err, bn,
                     act_mask, mask_scale, zero_tail_rows, **kw)

    def _dw(self, A, B, M, N, K_cap, K_dev, gW):
        """gW[M, N] += A^T B with A [K, M], B [K, N] (both MN-major), split-K over rows.
        Runs on the auxiliary stream (forked here, joined before the optimizer step), so
        the weight gradients overlap the input-gradient chain of the backward pass."""
        n_tiles = math.ceil(M / 128) * math.ceil(N / 256)
        main = torch.cuda.current_stream(self.device)
        aux = self._aux_stream()
        aux.wait_stream(main)
        with torch.cuda.stream(aux):
            self._gemm(A, True, B, True, M, None, N, K_cap, K_dev, split_k(K_cap, n_tiles), gW, GEMM_ATOMIC_F32,
                       bn=256)
        self._aux_used = True

    def _aux_stream(self):
        if getattr(self, "_aux", None) is None:
            self._aux = _stream(self.device, True)
        return self._aux

    def _join_aux(self):
        if getattr(self, "_aux_used", False):
            torch.cuda.current_stream(self.device).wait_stream(self._aux)
            self._aux_used = False

    def _comm_stream(self):
        if getattr(self, "_comm", None) is None:
            self._comm = _stream(self.device, True)
        return self._comm

    def _grad_ready(self, l):
        """Layer l's gradient is complete and no later kernel of the backward pass reads
        its parameters: reduce its bucket (all-reduce + Adam) on the comm stream while
        the backward pass goes on with the layers before it (the reference's DDP buckets
        reduced by the comm hook as autograd produces them)."""
        if not (self._ar_by_layer or self._adam_slices):
            return
        comm = self._comm_stream()
        comm.wait_stream(torch.cuda.current_stream(self.device))
        if getattr(self, "_aux", None) is not None:
            comm.wait_stream(self._aux)
        with torch.cuda.stream(comm):
            self._launch_update(l)
        self._launched.add(l)
        self._comm_used = True

    def _launch_update(self, l):
        """All-reduce + Adam (or Adam alone) of layer l's parameters on the current stream."""
        if self._ar_by_layer:
            self.allreduce.launch(l, self._cov())
            self.cu.count += 1
        else:
            p, m, v, g, w = self._adam_slices[l]
            b1, b2 = self.betas
            self.cu.adam(p, m, v, g, w, self.lr, b1, b2, self.eps, 0.0, self.counters, 1.0, None, True)

    def _backward(self, update=False):
        """The backward pass; with ``update`` every layer's update is launched on the comm
        stream as soon as its gradient is complete (else ``_update`` runs them all)."""
        for l in range(self.L - 1, -1, -1):
            self._backward_layer(l)
            if update:
                self._grad_ready(l)

    def _backward_layer(self, l):
        raise NotImplementedError

    # ------------------------------------------------------------------ binding
    def bind_working(self, working, labels, gideg):
        """Point the engine at a working graph (after a repartition)."""
        if not self.full_graph and working.indptr.numel() - 1 > self.sm.n_nodes_cap:
            raise ValueError("working graph larger than the engine's node capacity")
        self._working = working
        self.labels = labels
        self.gideg = gideg
        # the captured graphs hold these pointers and sizes; the partition store rebuilds
        # the working graph in place, so a repartition usually keeps them all and the
        # graphs stay valid
        sig = tuple((t.data_ptr(), tuple(t.shape)) if t is not None else None
                    for t in (working.indptr, working.indices, working.feat, labels, gideg))
        if sig != getattr(self, "_working_sig", None):
            self._graph = None  # pointers changed: capture again
            self._graphs = {}
        self._working_sig = sig

    def set_epoch(self, epoch):
        self.counters[C_EPOCH] = int(epoch)
        self.counters[C_STEP] = 0

    # ------------------------------------------------------------------ the step
    def _cov(self):
        """[coverage sum, count] of the step: the sampler's for mini-batches; the block
        source's, computed once per repartition from the kept in-degrees, for full-graph
        training."""
        return self.sm.cov if self.full_graph else self.cov_cur

    def _sample_into(self, q, step_offset):
        """Sample the blocks of the step ``step_offset`` ahead of the main counters into
        sampler q (its own draw counters, coverage and seed labels)."""
        if self.full_graph:
            return
        w = self._working
        sm = self.samplers[q]
        # one prologue kernel: the sampler's counters, its coverage sums cleared, the
        # step's seeds from the epoch table (when one is bound), their labels and degrees
        self.cu.sample_prologue(self.counters, self.scnt[q], step_offset, self.covs[q], self._slots[0:1],
                                self._count_table, sm.seeds, sm.cnt[0:1], self.labels, self.seed_labels[q],
                                self.gideg, sm.seed_gideg if self.gideg is not None else None)
        sm.sample(w.indptr, w.indices, self.scnt[q], gideg=self.gideg, cov=self.covs[q], err=self.err,
                  seed_gideg_ready=True)

    def _sample(self):
        self._sample_into(self.p_cur, 0)

    def _forward(self, training=True):
        raise NotImplementedError

    def _update(self):
        self._join_aux()
        cu = self.cu
        b1, b2 = self.betas
        if self._ar_by_layer or self._adam_slices:
            # per-layer updates: those not launched during the backward pass run here,
            # then the comm stream joins
            for l in range(self.L - 1, -1, -1):
                if l not in self._launched:
                    self._launch_update(l)
            self._launched = set()
            if getattr(self, "_comm_used", False):
                torch.cuda.current_stream(self.device).wait_stream(self._comm)
                self._comm_used = False
        elif self.fused_allreduce:
            self.allreduce.launch_all(self._cov())
            self.cu.count += len(self.allreduce.buckets)
        elif self.world > 1:
            # the reference's path (t10n/grad.py:6-24): scale by c_r / W, NCCL SUM all-reduce, Adam
            import torch.distributed as dist

            cov = self._cov()
            c = cov[0:1] / cov[1:2].clamp(min=1.0)
            self.grad.mul_(c / self.world)
            dist.all_reduce(self.grad)
            cu.adam(self.flat, self.m, self.v, self.grad, self.wbf, self.lr, b1, b2, self.eps, 0.0, self.counters,
                    1.0, None, True)
        else:
            cu.adam(self.flat, self.m, self.v, self.grad, self.wbf, self.lr, b1, b2, self.eps, 0.0, self.counters,
                    1.0, None, True)

    def _step_body(self):
        self.cu.zero_(self.fstats)
        self.cu.zero_(self.istats)
        self._sample()
        self._forward(True)
        self._backward(update=True)
        self._update()
        self.cu.step_end(self.counters)

    def _capture(self, body):
        s = _stream(self.device, True)
        s.wait_stream(torch.cuda.current_stream(self.device))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                body()
        torch.cuda.current_stream(self.device).wait_stream(s)
        return g

    def capture(self):
        """Capture the single-sampler step into a CUDA graph (after one eager step has run)."""
        self._select(0)
        self._graph = self._capture(self._step_body)

    def _overlapped_step_body(self, p, prefetch):
        """Layers of the step on sampler p; with ``prefetch`` the next step is sampled
        into the other sampler on a side stream that joins before the counters advance.
        The step's loss goes to the bound ring and the statistics are cleared for the
        next step by step_end (the graphs start with them cleared)."""
        self._select(p)
        main = torch.cuda.current_stream(self.device)
        if prefetch:
            side = _stream(self.device, False)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                self._sample_into(1 - p, 1)
        self._forward(True)
        self._backward(update=True)
        self._update()
        if prefetch:
            main.wait_stream(side)
        self.cu.step_end(self.counters, self._slots[1:2], self.fstats, self.istats)

    def _graph_for(self, key):
        g = self._graphs.get(key)
        if g is None:
            torch.cuda.synchronize(self.device)
            if key[0] == "epoch":
                nb = key[1]

                def body():
                    # one epoch: the first step's sampling, then every step with the next
                    # step's sampling on the side stream; seeds come from the bound table
                    self.cu.zero_(self.fstats)
                    self.cu.zero_(self.istats)
                    self._select(0)
                    self._sample_into(0, 0)
                    p = 0
                    for s_ in range(nb):
                        self._overlapped_step_body(p, s_ + 1 < nb)
                        p ^= 1
                    self._select(0)

                g = self._capture(body)
            elif key[0] == "sample":
                p = key[1]

                def body():
                    self._select(p)
                    self._sample_into(p, 0)

                g = self._capture(body)
            else:
                g = self._capture(lambda: self._overlapped_step_body(key[1], key[2]))
            self._graphs[key] = g
        return g

    def _load_into(self, q, seeds, count):
        sm = self.samplers[q]
        sm.seeds.copy_(seeds, non_blocking=True)
        sm.cnt[0:1].copy_(count, non_blocking=True)

    def run_epoch(self, seeds, counts, ring=None):
        """Run the mini-batches ``seeds[s]`` / ``counts[s]`` of one epoch (the counters'
        epoch must be set).  With CUDA graphs and two samplers every step graph samples
        the next step's blocks while it computes.  ``ring[s]`` receives step s's loss."""
        nb = int(seeds.shape[0])
        if not (self.use_cuda_graph and len(self.samplers) > 1):
            for s in range(nb):
                self.step(seeds[s], counts[s])
                if ring is not None:
                    ring[s:s + 1].copy_(self.fstats[2:3], non_blocking=True)
            return
        self._bind_epoch(seeds, counts, ring)
        self._graph_for(("epoch", nb)).replay()
        self._slots.zero_()  # eager steps after the epoch load their own seeds
        self._select(0)

    def _bind_epoch(self, seeds, counts, ring):
        """Point the epoch graph at this epoch's seed table and loss ring.  Seeds in pinned
        host memory are read by the step prologue straight over PCIe (the host -> device
        copy of each step's seeds), device seeds are copied into a fixed table first; the
        loss ring (pinned host memory) is written by step_end (device -> host)."""
        nb, B = int(seeds.shape[0]), int(seeds.shape[1])
        if B != self.B:
            raise ValueError("seed table width differs from the batch capacity")
        if self._count_table.numel() != nb:
            # the captured graphs hold the table's address: capture again
            torch.cuda.synchronize(self.device)
            self._count_table = torch.zeros(nb, dtype=torch.int32, device=self.device)
            self._graphs = {}
            self._graph = None
        self._count_table.copy_(counts.view(-1), non_blocking=True)
        if seeds.is_cuda:
            if self._seed_table is None or tuple(self._seed_table.shape) != (nb, B):
                self._seed_table = torch.zeros((nb, B), dtype=torch.int32, device=self.device)
            self._seed_table.copy_(seeds, non_blocking=True)
            table = self._seed_table.data_ptr()
        else:
            if not seeds.is_pinned():
                raise ValueError("host seed tables must be pinned (read by the device over PCIe)")
            table = seeds.data_ptr()
        if ring is not None and not ring.is_pinned():
            raise ValueError("the loss ring must be pinned host memory")
        self._slots[0].fill_(table)
        self._slots[1].fill_(0 if ring is None else ring.data_ptr())

    def load_seeds(self, seeds, count):
        """Copy this step's seeds ([B] int32) and seed count ([1] int32) into the static
        buffers.  Both may live in device memory or in pinned host memory; they are
        plain copies (no kernels) and must stay unchanged until the step has run."""
        if self.full_graph:
            return
        self.seeds.copy_(seeds, non_blocking=True)
        self.sm.cnt[0:1].copy_(count, non_blocking=True)

    def step(self, seeds=None, count=None):
        self._select(0)
        if seeds is not None:
            self.load_seeds(seeds, count)
        if self.use_cuda_graph and self._graph is not None:
            self._graph.replay()
        else:
            c0 = self.cu.count
            self._step_body()
            self.launches_per_step = self.cu.count - c0

    def prepare(self):
        """Capture the step graph (call after an eager step so that attributes and tensor
        maps are initialised)."""
        if self.use_cuda_graph and self._graph is None:
            torch.cuda.synchronize(self.device)
            self.capture()

    def predict(self, seeds, count):
        """Forward only (eval mode) for the given seeds; returns (correct, loss) on the device."""
        self._select(0)
        self.load_seeds(seeds, count)
        self.cu.zero_(self.fstats)
        self.cu.zero_(self.istats)
        self._sample()
        self._forward(training=False)
        return self.istats[0:1], self.fstats[2:3]

    def time_phases(self, seeds, counts, n_steps=None):
        """Device time per phase of eager steps (CUDA events on the launching stream,
        one synchronisation at the end): {'sample', 'forward', 'backward', 'update'} in
        ms per step, averaged over the steps.  NVTX ranges mark the same phases."""
        import torch.cuda.nvtx as nvtx

        n = int(seeds.shape[0]) if n_steps is None else int(n_steps)
        names = ("sample", "forward", "backward", "update")
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(n)]
        self._select(0)
        for s in range(n):
            self.load_seeds(seeds[s % seeds.shape[0]], counts[s % counts.shape[0]])
            self.cu.zero_(self.fstats)
            self.cu.zero_(self.istats)
            e = ev[s]
            e[0].record()
            for k, fn in enumerate((self._sample, lambda: self._forward(True), lambda: self._backward(update=True),
                                    self._update)):
                nvtx.range_push(names[k])
                fn()
                nvtx.range_pop()
                e[k + 1].record()
            self.cu.step_end(self.counters)
        torch.cuda.synchronize(self.device)
        return {name: sum(ev[s][k].elapsed_time(ev[s][k + 1]) for s in range(n)) / n for k, name in enumerate(names)}

    def check_errors(self):
        e = int(self.err.item())
        if e:
            raise RuntimeError(f"device error word {e:#x} (bits: grappa_b200/csrc/cuda/common.cuh kErr*)")

    # checkpoint helpers --------------------------------------------------------------
    def optimizer_state_dict(self):
        """torch.optim.Adam-compatible state of the fused optimizer (one entry per
        model parameter, views of the flat moments)."""
        if self.allreduce is not None:
            self.allreduce.sync_moments(self.m, self.v)  # collective: sharded moments to every rank
        state, ids = {}, []
        t = torch.tensor(float(self.counters[5].item()))
        for i, (name, p) in enumerate(self.model.named_parameters()):
            mv = self._param_view(p, self.m)
            vv = self._param_view(p, self.v)
            state[i] = {"step": t.clone(), "exp_avg": mv.detach().clone().cpu(), "exp_avg_sq": vv.detach().clone().cpu()}
            ids.append(i)
        b1, b2 = self.betas
        group = {"lr": self.lr, "betas": (b1, b2), "eps": self.eps, "weight_decay": 0, "amsgrad": False,
                 "maximize": False, "foreach": None, "capturable": False, "differentiable": False, "fused": None,
                 "params": ids}
        return {"state": state, "param_groups": [group]}

    def _param_view(self, p, buf):
        off = (p.data_ptr() - self.flat.data_ptr()) // 4
        return torch.as_strided(buf, p.shape, p.stride(), off)

    def load_optimizer_state_dict(self, sd):
        with torch.no_grad():
            for i, (name, p) in enumerate(self.model.named_parameters()):
                st = sd["state"].get(i)
                if st is None:
                    continue
                self._param_view(p, self.m).copy_(st["exp_avg"])
                self._param_view(p, self.v).copy_(st["exp_avg_sq"])
                self.counters[5] = int(float(st["step"]))
            self.wbf.copy_(self.flat)


class SageEngine(BlockEngine):
    """GraphSAGE (mean): [h_dst | mean h_src] . [W_self | W_neigh]^T + b in one GEMM.
    The backward of every inner hop runs gathered by source over the block's transpose
    (built by the sampler on its side stream), with the previous layer's ReLU/dropout
    backward fused: no fp32 gradient rows and no separate activation pass."""

    model_name = "sage"

    def _make_sampler(self, batch_size, n_nodes_cap, dev):
        # hops 0 .. L-2 feed a backward aggregation (the input layer's hop does not);
        # "inner" leaves hop 0 to the fused output layer's scatter
        if SAGE_GATHER_BWD == "1":
            hops = tuple(range(self.L - 1))
        elif SAGE_GATHER_BWD == "inner" and SAGE_FUSED_HEAD:  # mini-batch samplers only
            hops = tuple(range(1, self.L - 1))
        else:
            hops = ()
        return GpuNeighborSampler(self.fanouts, batch_size, n_nodes_cap, dev, cu=self.cu, transpose_hops=hops)

    def _alloc_layers(self):
        dev = self.device
        for l, layer in enumerate(self.model.layers):
            h = self.L - 1 - l
            ip, op = pad8(layer.in_feats), pad8(layer.out_feats)
            K = 2 * ip
            rows = self.sm.cap_dst[h]
            spec = dict(h=h, ip=ip, op=op, K=K, rows=rows,
                        W=self._seg(layer.seg_w, self.wbf), bias=self._seg(layer.seg_b)[0],
                        gW=self._seg(layer.seg_w, self.grad), gb=self._seg(layer.seg_b, self.grad)[0],
                        X=torch.zeros((rows, K), dtype=torch.bfloat16, device=dev),
                        dY=torch.zeros((rows, op), dtype=torch.bfloat16, device=dev))
            if l < self.L - 1:
                spec["H"] = torch.zeros((rows, op), dtype=torch.bfloat16, device=dev)
                # fp32 gradient rows unless the next layer's hop (L-2-l) has a block
                # transpose (gathered backward with the activation backward fused)
                if self.full_graph or (self.L - 2 - l) not in (getattr(self.sm, "tptr", None) or {}):
                    spec["dH"] = torch.zeros((rows, op), dtype=torch.float32, device=dev)
            else:
                spec["ce_fused"] = op <= 64
                spec["head"] = (SAGE_FUSED_HEAD and l > 0 and not self.full_graph
                                and self.cu.sage_head_supported(ip, self.n_classes))
                # the previous layer keeps fp32 gradient rows (scatter backward): the head
                # kernel reduces into them itself
                spec["head_bwd"] = bool(spec["head"] and self.cu.sage_head_fused_bwd()
                                        and "dH" in self.lay[l - 1])
                if not spec["ce_fused"]:
                    spec["logits"] = torch.zeros((rows, op), dtype=torch.bfloat16, device=dev)
            if l > 0:
                spec["dX"] = torch.zeros((rows, K), dtype=torch.bfloat16, device=dev)
            spec["tile"] = bool(SAGE_TILE_LAYERS and 0 < l < self.L - 1 and not self.full_graph
                                and "dH" in self.lay[l - 1] and self.cu.sage_layer_tile_supported(ip, op))
            self.lay.append(spec)

    def _forward(self, training=True):
        cu, sm = self.cu, self.sm
        L = self.L
        for l, s in enumerate(self.lay):
            h = s["h"]
            src, src_map = self._input(l)
            if s.get("head"):
                # aggregation, logits, loss, dlogits (dY) and dX of the output layer; with
                # the tile kernel also the aggregation's backward into the previous layer's
                # fp32 gradient rows (no dX written)
                labels, _, _ = self._labels_rows()
                fused_bwd = training and s["head_bwd"]
                cu.sage_head(sm.indptr[h], sm.indices[h], self._n_dst(h), sm.cap_dst[h], src, s["ip"], s["W"],
                             s["bias"], self.n_classes, labels, s["X"], s["dY"],
                             s["dX"] if training and not fused_bwd else None, self.fstats[2:3], self.istats[0:1],
                             s["gb"] if training else None, dsrc=self.lay[l - 1]["dH"] if fused_bwd else None)
                continue
            if s.get("tile"):
                p = self.p if training else 0.0
                cu.sage_layer_fwd(sm.indptr[h], sm.indices[h], self._n_dst(h), sm.cap_dst[h], src, s["ip"], s["W"],
                                  s["op"], s["bias"], 1, p, self.counters if p > 0 else None, l, s["X"], s["H"])
                continue
            cu.aggregate(sm.indptr[h], sm.indices[h], self._n_dst(h), 0, sm.cap_dst[h], src, src_map,
                         s["ip"], AGG_MEAN, None, None, None, s["X"], s["ip"], 0, 0.0, 0, self.err)
            if l < L - 1:
                self._gemm(s["X"], False, s["W"], False, s["rows"], self._n_dst(h), s["op"], s["K"], None, 1,
                           s["H"], GEMM_STORE_BF16, s["bias"], 1, self.p if training else 0.0, l)
            elif s["ce_fused"]:
                labels, _, _ = self._labels_rows()
                cu.gemm(s["X"], False, s["W"], False, s["rows"], self._n_dst(h), s["op"], s["K"], None, 1,
                        self._ce_dummy, GEMM_CROSS_ENTROPY, s["bias"], 0, 0.0, None, 0, labels,
                        self.n_classes, s["dY"], self.fstats[2:3], self.istats[0:1], None, self._n_dst(h),
                        s["gb"] if training else None, self.err, bn_for(s["op"]))
            else:
                self._gemm(s["X"], False, s["W"], False, s["rows"], self._n_dst(h), s["op"], s["K"], None, 1,
                           s["logits"], GEMM_STORE_BF16, s["bias"])
                self._ce(s["logits"], self.n_classes, s["dY"], s["gb"] if training else None, h)

    def _backward_layer(self, l):
        cu, sm = self.cu, self.sm
        scale = dropout_scale(self.p)
        s = self.lay[l]
        h = s["h"]
        # dW += dY^T X (split-K over the block's rows, fp32 reductions into the gradient)
        self._dw(s["dY"], s["X"], s["op"], s["K"], s["rows"], self._n_dst(h), s["gW"])
        if l == 0:
            return
        if s.get("tile"):
            # dY W reduced into the previous layer's fp32 rows through the aggregation's
            # transpose, then the previous layer's activation backward
            prev = self.lay[l - 1]
            cu.sage_layer_bwd(sm.indptr[h], sm.indices[h], self._n_dst(h), sm.cap_dst[h], s["dY"], s["ip"], s["W"],
                              s["op"], prev["dH"])
            cu.act_bwd(prev["dH"], prev["H"], prev["dY"], self._n_dst(prev["h"]), 0, prev["op"], scale, prev["gb"],
                       prev["rows"])
            return
        # dX = dY W (W read MN-major; the fused output layer wrote it in the forward pass)
        if not s.get("head"):
            self._gemm(s["dY"], False, s["W"], True, s["rows"], self._n_dst(h), s["K"], s["op"], None, 1, s["dX"],
                       GEMM_STORE_BF16)
        prev = self.lay[l - 1]
        if "dH" not in prev:
            # gathered by source over the block's transpose, activation backward fused
            cu.aggregate_bwd_gather(sm.indptr[h], sm.tptr[h], sm.tdst[h], self._n_dst(h), sm.n_src(h), s["dX"], 0,
                                    s["ip"], s["ip"], prev["H"], scale, prev["dY"], prev["gb"], self.err)
            return
        # transpose aggregation: d(self) -> dst rows, d(agg) -> sources (done by the
        # fused output layer in the forward pass)
        if not s.get("head_bwd"):
            cu.aggregate_bwd(sm.indptr[h], sm.indices[h], self._n_dst(h), 0, sm.cap_dst[h], s["dX"],
                             s["ip"], 0, 0.0, s["ip"], AGG_MEAN, None, None, None, prev["dH"], self.err)
        cu.act_bwd(prev["dH"], prev["H"], prev["dY"], self._n_dst(prev["h"]), 0, prev["op"], scale, prev["gb"],
                   prev["rows"])


class GcnEngine(BlockEngine):
    """GCN (GraphConv norm='both'): D_dst^-1/2 A D_src^-1/2 h W + b.  The projection
    runs first when it narrows the rows (in > out), as DGL does."""

    model_name = "gcn"

    def _alloc_layers(self):
        dev = self.device
        z = dict(dtype=torch.bfloat16, device=dev)
        for l, layer in enumerate(self.model.layers):
            h = self.L - 1 - l
            ip, op = pad8(layer.in_feats), pad8(layer.out_feats)
            rows, srows = self.sm.cap_dst[h], self.sm.cap_src[h]
            last = l == self.L - 1
            s = dict(h=h, ip=ip, op=op, rows=rows, srows=srows, last=last, first_proj=layer.in_feats > layer.out_feats,
                     W=self._seg(layer.seg_w, self.wbf), bias=self._seg(layer.seg_b)[0],
                     gW=self._seg(layer.seg_w, self.grad), gb=self._seg(layer.seg_b, self.grad)[0],
                     snorm=torch.zeros(srows, dtype=torch.float32, device=dev),
                     degs=torch.zeros(srows, dtype=torch.float32, device=dev),
                     dY=torch.zeros((rows, op), **z))
            s["H"] = torch.zeros((rows, op), **z)  # hidden output, or the logits of the last layer
            if not last:
                s["dH"] = torch.zeros((rows, op), dtype=torch.float32, device=dev)
            if s["first_proj"]:
                if l == 0 and not self.full_graph:
                    s["Xg"] = torch.zeros((srows, ip), **z)
                s["Z"] = torch.zeros((srows, op), **z)
                s["dZ32"] = torch.zeros((srows, op), dtype=torch.float32, device=dev)
                s["dZ"] = torch.zeros((srows, op), **z)
            else:
                s["X"] = torch.zeros((rows, ip), **z)
                if l > 0:
                    s["dX"] = torch.zeros((rows, ip), **z)
            self.lay.append(s)

    def _forward(self, training=True):
        cu, sm = self.cu, self.sm
        for l, s in enumerate(self.lay):
            h = s["h"]
            p = self.p if (training and not s["last"]) else 0.0
            act = 0 if s["last"] else 1
            cu.src_norm(sm.indices[h], sm.n_edges(h), sm.cap_e[h], sm.n_src(h), sm.cap_src[h], s["degs"], s["snorm"])
            if s["first_proj"]:
                A = self._gathered_input(l, s)
                self._gemm(A, False, s["W"], True, s["srows"], sm.n_src(h), s["op"], s["ip"], None, 1, s["Z"],
                           GEMM_STORE_BF16)
                cu.aggregate(sm.indptr[h], sm.indices[h], self._n_dst(h), 0, sm.cap_dst[h], s["Z"], None, s["op"],
                             AGG_GCN, None, s["snorm"], None, s["H"], 0, -1, 0.0, 64, self.err, bias=s["bias"],
                             act=act, dropout_p=p, counters=self.counters if p > 0 else None, dropout_salt=l)
            else:
                src, src_map = self._input(l)
                cu.aggregate(sm.indptr[h], sm.indices[h], self._n_dst(h), 0, sm.cap_dst[h], src, src_map, s["ip"],
                             AGG_GCN, None, s["snorm"], None, s["X"], 0, -1, 0.0, 64, self.err)
                self._gemm(s["X"], False, s["W"], True, s["rows"], self._n_dst(h), s["op"], s["ip"], None, 1, s["H"],
                           GEMM_STORE_BF16, s["bias"], act, p, l)
            if s["last"]:
                self._ce(s["H"], self.n_classes, s["dY"], s["gb"] if training else None, h)

    def _backward_layer(self, l):
        cu, sm = self.cu, self.sm
        scale = dropout_scale(self.p)
        s = self.lay[l]
        h = s["h"]
        if not s["last"]:
            cu.act_bwd(s["dH"], s["H"], s["dY"], self._n_dst(h), 0, s["op"], scale, s["gb"], s["rows"])
        prev = self.lay[l - 1] if l > 0 else None
        if s["first_proj"]:
            cu.aggregate_bwd(sm.indptr[h], sm.indices[h], self._n_dst(h), 0, sm.cap_dst[h], s["dY"], 0, -1, 0.0,
                             s["op"], AGG_GCN, None, s["snorm"], None, s["dZ32"], self.err)
            cu.f32_to_bf16_rows(s["dZ32"], s["dZ"], s["op"], sm.n_src(h), s["srows"], True, 64)
            A = s["Xg"] if "Xg" in s else (self._working.feat if l == 0 else prev["H"])
            self._dw(A, s["dZ"], s["ip"], s["op"], s["srows"], sm.n_src(h), s["gW"])
            if prev is not None:
                self._gemm(s["dZ"], False, s["W"], False, s["srows"], sm.n_src(h), s["ip"], s["op"], None, 1,
                           prev["dH"], GEMM_STORE_F32)
        else:
            self._dw(s["X"], s["dY"], s["ip"], s["op"], s["rows"], self._n_dst(h), s["gW"])
            if prev is not None:
                self._gemm(s["dY"], False, s["W"], False, s["rows"], self._n_dst(h), s["ip"], s["op"], None, 1,
                           s["dX"], GEMM_STORE_BF16)
                cu.aggregate_bwd(sm.indptr[h], sm.indices[h], self._n_dst(h), 0, sm.cap_dst[h], s["dX"], 0, -1,
                                 0.0, s["ip"], AGG_GCN, None, s["snorm"], None, prev["dH"], self.err)


class GinEngine(BlockEngine):
    """GIN: MLP((1 + eps) h_dst + sum h_src) with Linear -> BatchNorm+ReLU -> Linear,
    then the model's BatchNorm+ReLU (training-mode batch statistics)."""

    model_name = "gin"

    def _alloc_layers(self):
        dev = self.device
        z = dict(dtype=torch.bfloat16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        m = self.model
        for l, conv in enumerate(m.layers):
            h = self.L - 1 - l
            mlp = conv.apply_func
            lin0, lin1 = mlp.linears
            ip, hp, op = pad8(lin0.in_features), pad8(lin0.out_features), pad8(lin1.out_features)
            rows = self.sm.cap_dst[h]
            bn_mlp, bn_out = mlp.batch_norm, m.batch_norms[l]
            seg_bn_out = f"batch_norms.{l}"
            s = dict(h=h, ip=ip, hp=hp, op=op, rows=rows, last=l == self.L - 1, eps=float(conv.eps.item()),
                     W0=self._seg(mlp.seg_w0, self.wbf), W1=self._seg(mlp.seg_w1, self.wbf),
                     gW0=self._seg(mlp.seg_w0, self.grad), gW1=self._seg(mlp.seg_w1, self.grad),
                     g_mlp=self._seg(mlp.seg_bn)[0], b_mlp=self._seg(mlp.seg_bn)[1],
                     dg_mlp=self._seg(mlp.seg_bn, self.grad)[0], db_mlp=self._seg(mlp.seg_bn, self.grad)[1],
                     g_out=self._seg(seg_bn_out)[0], b_out=self._seg(seg_bn_out)[1],
                     dg_out=self._seg(seg_bn_out, self.grad)[0], db_out=self._seg(seg_bn_out, self.grad)[1],
                     bn_mlp=bn_mlp, bn_out=bn_out,
                     X=torch.zeros((rows, ip), **z), T0=torch.zeros((rows, hp), **z), U=torch.zeros((rows, hp), **z),
                     T1=torch.zeros((rows, op), **z), H=torch.zeros((rows, op), **z),
                     s_mlp=torch.zeros(2 * hp, **f32), s_out=torch.zeros(2 * op, **f32),
                     bs_mlp=torch.zeros(2 * hp, **f32), bs_out=torch.zeros(2 * op, **f32),
                     dU=torch.zeros((rows, hp), **f32), dT0=torch.zeros((rows, hp), **z),
                     dT1=torch.zeros((rows, op), **z))
            if s["last"]:
                s["dl"] = torch.zeros((rows, op), **z)
            else:
                s["dH"] = torch.zeros((rows, op), **f32)
            if l > 0:
                s["dX"] = torch.zeros((rows, ip), **z)
            self.lay.append(s)

    def _bn(self, x, dim, n, cap, sums, gamma, beta, mod, training, y):
        cu = self.cu
        if training:
            cu.zero_(sums)
        cu.batchnorm_fwd(x, dim, n, cap, sums, gamma, beta, mod.running_mean, mod.running_var,
                         mod.num_batches_tracked if training else None, mod.momentum, mod.eps, training, 1, y)

    def _forward(self, training=True):
        cu, sm = self.cu, self.sm
        for l, s in enumerate(self.lay):
            h = s["h"]
            n = self._n_dst(h)
            src, src_map = self._input(l)
            cu.aggregate(sm.indptr[h], sm.indices[h], n, 0, sm.cap_dst[h], src, src_map, s["ip"], AGG_SUM, None,
                         None, None, s["X"], 0, -1, 1.0 + s["eps"], 64, self.err)
            self._gemm(s["X"], False, s["W0"], False, s["rows"], n, s["hp"], s["ip"], None, 1, s["T0"],
                       GEMM_STORE_BF16)
            self._bn(s["T0"], s["hp"], n, s["rows"], s["s_mlp"], s["g_mlp"], s["b_mlp"], s["bn_mlp"], training, s["U"])
            self._gemm(s["U"], False, s["W1"], False, s["rows"], n, s["op"], s["hp"], None, 1, s["T1"],
                       GEMM_STORE_BF16)
            self._bn(s["T1"], s["op"], n, s["rows"], s["s_out"], s["g_out"], s["b_out"], s["bn_out"], training, s["H"])
            if s["last"]:
                self._ce(s["H"], self.n_classes, s["dl"], None, h)

    def _backward_layer(self, l):
        cu, sm = self.cu, self.sm
        s = self.lay[l]
        h = s["h"]
        n = self._n_dst(h)
        dy = s["dl"] if s["last"] else s["dH"]
        cu.zero_(s["bs_out"])
        cu.batchnorm_bwd(s["T1"], s["H"], dy, True, s["op"], n, s["rows"], s["s_out"], s["bs_out"], s["g_out"],
                         s["dg_out"], s["db_out"], s["bn_out"].eps, s["dT1"])
        self._dw(s["dT1"], s["U"], s["op"], s["hp"], s["rows"], n, s["gW1"])
        self._gemm(s["dT1"], False, s["W1"], True, s["rows"], n, s["hp"], s["op"], None, 1, s["dU"],
                   GEMM_STORE_F32)
        cu.zero_(s["bs_mlp"])
        cu.batchnorm_bwd(s["T0"], s["U"], s["dU"], True, s["hp"], n, s["rows"], s["s_mlp"], s["bs_mlp"],
                         s["g_mlp"], s["dg_mlp"], s["db_mlp"], s["bn_mlp"].eps, s["dT0"])
        self._dw(s["dT0"], s["X"], s["hp"], s["ip"], s["rows"], n, s["gW0"])
        if l == 0:
            return
        prev = self.lay[l - 1]
        self._gemm(s["dT0"], False, s["W0"], True, s["rows"], n, s["ip"], s["hp"], None, 1, s["dX"],
                   GEMM_STORE_BF16)
        cu.aggregate_bwd(sm.indptr[h], sm.indices[h], n, 0, sm.cap_dst[h], s["dX"], 0, -1, 1.0 + s["eps"],
                         s["ip"], AGG_SUM, None, None, None, prev["dH"], self.err)


class GatEngine(BlockEngine):
    """GAT: z = fc(h_src) (GEMM) -> attention logits -> fused edge softmax + weighted sum
    (+bias; ReLU + dropout on hidden layers, mean over heads on the last)."""

    model_name = "gat"

    def _alloc_layers(self):
        dev = self.device
        z = dict(dtype=torch.bfloat16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        for l, layer in enumerate(self.model.layers):
            h = self.L - 1 - l
            H, F = layer.num_heads, layer.out_feats
            HF = H * F
            ip, hfp = pad8(layer.in_feats), pad8(HF)
            rows, srows, ecap = self.sm.cap_dst[h], self.sm.cap_src[h], self.sm.cap_e[h]
            last = l == self.L - 1
            A = self._seg(layer.seg_a)
            gA = self._seg(layer.seg_a, self.grad)
            # input layer without a per-source dz (gat.cu): attention on x with the
            # projection after the aggregation ("x"), or dW from attention-weighted
            # input rows ("bwd")
            in_ok = GAT_INPUT_LAYER_BWD and l == 0 and not last and H * ip <= 1024
            in_x = in_ok and (GAT_INPUT_MODE == "x" or (GAT_INPUT_MODE == "auto" and ip <= F))
            in_fast = in_ok and not in_x
            s = dict(h=h, H=H, F=F, HF=HF, ip=ip, hfp=hfp, rows=rows, srows=srows, last=last, in_fast=in_fast,
                     in_x=in_x, W=self._seg(layer.seg_w, self.wbf), W32=self._seg(layer.seg_w),
                     gW=self._seg(layer.seg_w, self.grad), al=A[0], ar=A[1], gal=gA[0], gar=gA[1],
                     bias=self._seg(layer.seg_b)[0], gb=self._seg(layer.seg_b, self.grad)[0],
                     Z=None if in_x else torch.zeros((srows, hfp), **z), el=torch.zeros(srows * H, **f32),
                     er=torch.zeros(rows * H, **f32), smax=torch.zeros(rows * H, **f32),
                     ssum=torch.zeros(rows * H, **f32), escr=torch.zeros(ecap * H, **f32),
                     del_=torch.zeros(srows * H, **f32), der=torch.zeros(rows * H, **f32))
            if in_x:
                hin = H * ip
                s["Yin"] = torch.zeros((rows, hin), **z)   # y_v[h] = sum_u a_uvh x_u
                s["G"] = torch.zeros((rows, hin), **z)     # dL/dy = dout Wbd
                s["Wbd"] = torch.zeros((hfp, hin), **z)    # block-diagonal W (row hF+f: W[hF+f] at columns h*ip)
                s["wlr"] = torch.zeros(2 * hin, **f32)     # wl[h] = sum_f a_l[h,f] W[hF+f], wr
                s["T"] = torch.zeros((hfp, hin), **f32)
                s["xlr"] = torch.zeros(2 * hin, **f32)
            elif in_fast:
                s["Yin"] = torch.zeros((rows, H * ip), **z)
                s["T"] = torch.zeros((hfp, H * ip), **f32)
                s["xlr"] = torch.zeros(2 * H * ip, **f32)
            else:
                s["dz"] = torch.zeros((srows, hfp), **f32)
                s["dzb"] = torch.zeros((srows, hfp), **z)
            if l == 0 and not self.full_graph:
                s["Xg"] = torch.zeros((srows, ip), **z)
            if last:
                s["fo"] = pad8(F)
                s["H_out"] = torch.zeros((rows, s["fo"]), **z)
                s["dl"] = torch.zeros((rows, s["fo"]), **z)
            else:
                s["H_out"] = torch.zeros((rows, hfp), **z)
                # written by the next layer's dX GEMM with the ReLU/dropout backward fused
                # into its epilogue (no fp32 gradient rows, no separate activation pass)
                s["dY"] = torch.zeros((rows, hfp), **z)
            self.lay.append(s)

    def _A(self, l, s):
        if l > 0:
            return self.lay[l - 1]["H_out"]
        return s["Xg"] if "Xg" in s else self._working.feat

    def _forward(self, training=True):
        cu, sm = self.cu, self.sm
        for l, s in enumerate(self.lay):
            h = s["h"]
            if l == 0:
                A = self._gathered_input(0, s) if "Xg" in s else self._working.feat
            else:
                A = self.lay[l - 1]["H_out"]
            p = self.p if (training and not s["last"]) else 0.0
            if s["in_x"]:
                self._input_layer_fwd(s, h, A, p, l)
                continue
            args = (sm.indptr[h], sm.indices[h], self._n_dst(h), s["rows"], sm.n_src(h), s["srows"], s["H"], s["F"],
                    s["Z"], s["al"], s["ar"], s["el"], s["er"], s["smax"], s["ssum"], 0.2)
            if GAT_FUSED_LOGITS:
                # z = x W^T with the attention logits el / er reduced in the GEMM epilogue
                cu.zero_(s["el"])
                cu.zero_(s["er"])
                self._gemm(A, False, s["W"], False, s["srows"], sm.n_src(h), s["HF"], s["ip"], None, 1, s["Z"],
                           GEMM_STORE_BF16, att=(s["al"], s["ar"], s["el"], s["er"], s["H"], s["F"], self._n_dst(h)))
            else:
                self._gemm(A, False, s["W"], False, s["srows"], sm.n_src(h), s["HF"], s["ip"], None, 1, s["Z"],
                           GEMM_STORE_BF16)
                cu.gat_scores(*args)
            cu.gat_fwd(*args, s["bias"], s["last"], 0 if s["last"] else 1, p, self.counters if p > 0 else None,
                       l, s["H_out"])
            if s["last"]:
                self._ce(s["H_out"], self.n_classes, s["dl"], None, h)

    def _backward_layer(self, l):
        cu, sm = self.cu, self.sm
        scale = dropout_scale(self.p)
        s = self.lay[l]
        h = s["h"]
        # a hidden layer's dY was written by the layer above's dX GEMM (activation backward
        # fused into its epilogue)
        dout = s["dl"] if s["last"] else s["dY"]
        A = self._A(l, s)
        if s["in_x"]:
            self._input_layer_bwd_x(s, h, dout, A)
            return
        if s["in_fast"]:
            self._input_layer_bwd(s, h, dout, A)
            return
        cu.gat_bwd(sm.indptr[h], sm.indices[h], self._n_dst(h), s["rows"], sm.n_src(h), s["srows"], s["H"],
                   s["F"], s["Z"], s["al"], s["ar"], s["el"], s["er"], s["smax"], s["ssum"], 0.2, s["last"], dout,
                   s["escr"], s["del_"], s["der"], s["dz"], s["gb"], s["gal"], s["gar"], s["dzb"], self.err)
        self._dw(s["dzb"], A, s["HF"], s["ip"], s["srows"], sm.n_src(h), s["gW"])
        if l > 0:
            # dX = dz W, then the previous layer's ReLU + dropout backward, in one GEMM
            prev = self.lay[l - 1]
            self._gemm(s["dzb"], False, s["W"], True, s["srows"], sm.n_src(h), s["ip"], s["HF"], None, 1,
                       prev["dY"], GEMM_STORE_BF16, act_mask=prev["H_out"], mask_scale=scale, zero_tail_rows=64)


    def _input_layer_fwd(self, s, h, X, p, l):
        """Input layer with the projection after the aggregation: the logits are
        el_u = x_u . wl[h] (wl[h] = sum_f a_l[h,f] W[hF+f]), the softmax-weighted sum runs
        over the input rows (y_v[h] = sum_u a_uvh x_u, [rows, H*in]) and one GEMM against
        the block-diagonal W (bias, ReLU and dropout in its epilogue) gives the layer's
        output.  Equal to W x then attention (the weights are linear in x); it reads in
        columns per edge instead of H*F and needs no projection of every source row."""
        cu, sm = self.cu, self.sm
        H, ip = s["H"], s["ip"]
        hin = H * ip
        wl, wr = s["wlr"][:hin], s["wlr"][hin:]
        cu.gat_in_prep(s["W"], s["al"], s["ar"], H, s["F"], ip, wl, wr, s["Wbd"])
        args = (sm.indptr[h], sm.indices[h], self._n_dst(h), s["rows"], sm.n_src(h), s["srows"], H, ip, X, wl, wr,
                s["el"], s["er"], s["smax"], s["ssum"], 0.2)
        cu.gat_in_scores(*args)
        cu.gat_in_fwd(*args, s["Yin"])
        self._gemm(s["Yin"], False, s["Wbd"], False, s["rows"], self._n_dst(h), s["HF"], hin, None, 1, s["H_out"],
                   GEMM_STORE_BF16, bias=s["bias"], act=1, p=p, salt=l, zero_tail_rows=64)

    def _input_layer_bwd_x(self, s, h, dout, X):
        """Backward of ``_input_layer_fwd``: G = dout Wbd (dL/dy), the attention backward
        over the input rows gives xl[h] = sum_u del[u,h] x_u and xr[h]; then
        dW[hF+f] = (dout^T y)[hF+f, h-block] + a_l[h,f] xl[h] + a_r[h,f] xr[h],
        da_l[h,f] = W[hF+f] . xl[h] (same for a_r) and db = column sums of dout.  The
        dout^T y GEMM and the bias sums run on the auxiliary stream."""
        cu, sm = self.cu, self.sm
        H, ip = s["H"], s["ip"]
        hin = H * ip
        wl, wr = s["wlr"][:hin], s["wlr"][hin:]
        xl, xr = s["xlr"][:hin], s["xlr"][hin:]
        main = torch.cuda.current_stream(self.device)
        aux = self._aux_stream()
        aux.wait_stream(main)
        n_tiles = math.ceil(s["hfp"] / 128) * math.ceil(hin / 256)
        with torch.cuda.stream(aux):
            cu.zero_(s["T"])
            self._gemm(dout, True, s["Yin"], True, s["hfp"], None, hin, s["rows"], self._n_dst(h),
                       split_k(s["rows"], n_tiles), s["T"], GEMM_ATOMIC_F32, bn=256)
            cu.col_sum_bf16(dout, self._n_dst(h), s["HF"], s["gb"])
        self._gemm(dout, False, s["Wbd"], True, s["rows"], self._n_dst(h), hin, s["HF"], None, 1, s["G"],
                   GEMM_STORE_BF16)
        cu.zero_(s["xlr"])
        cu.gat_in_bwd(sm.indptr[h], sm.indices[h], self._n_dst(h), s["rows"], sm.n_src(h), s["srows"], H, ip, X, wl,
                      wr, s["el"], s["er"], s["smax"], s["ssum"], 0.2, s["G"], s["escr"], s["del_"], s["der"], xl, xr,
                      self.err)
        aux.wait_stream(main)
        with torch.cuda.stream(aux):
            cu.gat_in_dw(s["T"], xl, xr, s["al"], s["ar"], s["W32"], H, s["F"], ip, s["gW"], s["gal"], s["gar"])
        self._aux_used = True

    def _input_layer_bwd(self, s, h, dout, A):
        """dW of the input layer as dout^T y plus two rank-1 terms (y = attention-weighted
        input rows per destination), with no per-source dz: the GEMM and the combine run
        on the auxiliary stream like the other weight gradients."""
        cu, sm = self.cu, self.sm
        Hh, ip = s["H"], s["ip"]
        xl, xr = s["xlr"][:Hh * ip], s["xlr"][Hh * ip:]
        cu.zero_(s["xlr"])
        # no attention-vector gradients here: da_l[hF+f] = sum_u del[u,h] z_u[hF+f] =
        # W[hF+f] . xl[h], formed by gat_in_dw (the node pass then reads no z rows)
        cu.gat_bwd_input(sm.indptr[h], sm.indices[h], self._n_dst(h), s["rows"], sm.n_src(h), s["srows"], Hh,
                         s["F"], s["Z"], s["al"], s["ar"], s["el"], s["er"], s["smax"], s["ssum"], 0.2, dout,
                         s["escr"], s["del_"], s["der"], s["gb"], None, None, A, ip, s["Yin"], xl, xr, self.err)
        main = torch.cuda.current_stream(self.device)
        aux = self._aux_stream()
        aux.wait_stream(main)
        n_tiles = math.ceil(s["hfp"] / 128) * math.ceil(Hh * ip / 256)
        with torch.cuda.stream(aux):
            cu.zero_(s["T"])
            self._gemm(dout, True, s["Yin"], True, s["hfp"], None, Hh * ip, s["rows"], self._n_dst(h),
                       split_k(s["rows"], n_tiles), s["T"], GEMM_ATOMIC_F32, bn=256)
            cu.gat_in_dw(s["T"], xl, xr, s["al"], s["ar"], s["W32"], Hh, s["F"], ip, s["gW"], s["gal"], s["gar"])
        self._aux_used = True


class PinSageEngine(BlockEngine):
    """PinSAGE (WeightedSAGEConv): n = ReLU(Q drop(h_src) + q); n_v = sum w n_u / max(sum w, 1);
    z = ReLU(W drop([n_v | h_dst]) + b); out = z / |z|, on random-walk blocks."""

    model_name = "pinsage"

    def __init__(self, *args, walk_length=None, restart_prob=0.5, num_walks=4, num_neighbors=5, **kw):
        self._walk = dict(length=walk_length, restart_prob=restart_prob, num_walks=num_walks,
                          num_neighbors=num_neighbors)
        super().__init__(*args, **kw)

    def _make_sampler(self, batch_size, n_nodes_cap, dev):
        wk = self._walk
        return GpuWalkSampler(self.L, batch_size, n_nodes_cap, dev, cu=self.cu,
                              length=wk["length"] if wk["length"] is not None else self.L,
                              restart_prob=wk["restart_prob"], num_walks=wk["num_walks"],
                              num_neighbors=wk["num_neighbors"])

    def _alloc_layers(self):
        dev = self.device
        z = dict(dtype=torch.bfloat16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        for l, layer in enumerate(self.model.layers):
            h = self.L - 1 - l
            if layer.hidden_dims % 8 != 0:
                raise ValueError("PinSAGE engine: hidden width must be a multiple of 8")
            ip, hid, op = pad8(layer.input_dims), layer.hidden_dims, pad8(layer.output_dims)
            kw = pad8(hid + layer.input_dims)
            rows, srows = self.sm.cap_dst[h], self.sm.cap_src[h]
            last = l == self.L - 1
            s = dict(h=h, ip=ip, hid=hid, op=op, kw=kw, rows=rows, srows=srows, last=last,
                     Q=self._seg(layer.seg_q, self.wbf), gQ=self._seg(layer.seg_q, self.grad),
                     qb=self._seg(layer.seg_qb)[0], gqb=self._seg(layer.seg_qb, self.grad)[0],
                     W=self._seg(layer.seg_w, self.wbf), gW=self._seg(layer.seg_w, self.grad),
                     wb=self._seg(layer.seg_wb)[0], gwb=self._seg(layer.seg_wb, self.grad)[0],
                     Hd=torch.zeros((srows, ip), **z), N=torch.zeros((srows, hid), **z),
                     X=torch.zeros((rows, kw), **z), Z=torch.zeros((rows, op), **z), H=torch.zeros((rows, op), **z),
                     norms=torch.zeros(rows, **f32), dZ32=torch.zeros((rows, op), **f32),
                     dZ=torch.zeros((rows, op), **z), dX=torch.zeros((rows, kw), **z),
                     dN32=torch.zeros((srows, hid), **f32), dN=torch.zeros((srows, hid), **z))
            if l == 0 and not self.full_graph:
                s["Xg"] = torch.zeros((srows, ip), **z)
            if last:
                s["dl"] = torch.zeros((rows, op), **z)
            else:
                s["dH"] = torch.zeros((rows, op), **f32)
            self.lay.append(s)

    def _A(self, l, s):
        if l > 0:
            return self.lay[l - 1]["H"]
        return s["Xg"] if "Xg" in s else self._working.feat

    def _forward(self, training=True):
        cu, sm = self.cu, self.sm
        p = self.p if training else 0.0
        for l, s in enumerate(self.lay):
            h = s["h"]
            n = self._n_dst(h)
            A = self._gathered_input(l, s) if l == 0 else self._A(l, s)
            cu.dropout_rows(A, s["Hd"], s["ip"], s["ip"], sm.n_src(h), s["srows"], p, self.counters, 8 * l + 1)
            self._gemm(s["Hd"], False, s["Q"], False, s["srows"], sm.n_src(h), s["hid"], s["ip"], None, 1, s["N"],
                       GEMM_STORE_BF16, s["qb"], 1)
            cu.aggregate(sm.indptr[h], sm.indices[h], n, 0, sm.cap_dst[h], s["N"], None, s["hid"], AGG_WEIGHTED,
                         sm.w[h], None, None, s["X"], 0, -1, 0.0, 64, self.err, dropout_p=p,
                         counters=self.counters if p > 0 else None, dropout_salt=8 * l + 2)
            cu.dropout_rows(A, s["X"][:, s["hid"]:s["hid"] + s["ip"]], s["ip"], s["kw"], n, s["rows"], p,
                            self.counters, 8 * l + 3)
            self._gemm(s["X"], False, s["W"], False, s["rows"], n, s["op"], s["kw"], None, 1, s["Z"],
                       GEMM_STORE_BF16, s["wb"], 1)
            cu.l2norm_fwd(s["Z"], s["op"], n, s["rows"], s["H"], s["norms"])
            if s["last"]:
                self._ce(s["H"], self.n_classes, s["dl"], None, h)

    def _backward_layer(self, l):
        cu, sm = self.cu, self.sm
        p = self.p
        s = self.lay[l]
        h = s["h"]
        n = self._n_dst(h)
        cu.l2norm_bwd(s["H"], s["dl"] if s["last"] else s["dH"], s["norms"], s["op"], n, s["rows"], s["dZ32"])
        cu.act_bwd(s["dZ32"], s["Z"], s["dZ"], n, 0, s["op"], 1.0, s["gwb"], s["rows"])
        self._dw(s["dZ"], s["X"], s["op"], s["kw"], s["rows"], n, s["gW"])
        self._gemm(s["dZ"], False, s["W"], True, s["rows"], n, s["kw"], s["op"], None, 1, s["dX"],
                   GEMM_STORE_BF16)
        hid, ip = s["hid"], s["ip"]
        dnv, dhd = s["dX"][:, :hid], s["dX"][:, hid:hid + ip]
        cu.dropout_rows(dnv, dnv, hid, s["kw"], n, s["rows"], p, self.counters, 8 * l + 2)
        cu.aggregate_bwd(sm.indptr[h], sm.indices[h], n, 0, sm.cap_dst[h], s["dX"], 0, -1, 0.0, hid,
                         AGG_WEIGHTED, sm.w[h], None, None, s["dN32"], self.err)
        cu.act_bwd(s["dN32"], s["N"], s["dN"], sm.n_src(h), 0, hid, 1.0, s["gqb"], s["srows"])
        self._dw(s["dN"], s["Hd"], hid, ip, s["srows"], sm.n_src(h), s["gQ"])
        if l == 0:
            return
        prev = self.lay[l - 1]
        cu.dropout_rows(dhd, dhd, ip, s["kw"], n, s["rows"], p, self.counters, 8 * l + 3)
        self._gemm(s["dN"], False, s["Q"], True, s["srows"], sm.n_src(h), ip, hid, None, 1, prev["dH"],
                   GEMM_STORE_F32)
        cu.dropout_grad(prev["dH"], ip, ip, sm.n_src(h), s["srows"], p, self.counters, 8 * l + 1)
        cu.add_bf16_rows(prev["dH"], dhd, ip, n, s["rows"])


ENGINES = {"sage": SageEngine, "gcn": GcnEngine, "gin": GinEngine, "gat": GatEngine, "pinsage": PinSageEngine}


def make_engine(model, *args, **kwargs):
    """The engine class of ``model.name`` (sage, gcn, gin, gat, pinsage)."""
    try:
        cls = ENGINES[model.name]
    except KeyError:
        raise ValueError(f"no GPU engine for model {getattr(model, 'name', None)}") from None
    return cls(model, *args, **kwargs)
