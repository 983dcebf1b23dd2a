"""Mini-batch training engine on the sm_100a kernels.

One training step of a sampled-block GNN, entirely on the device:

  for hop h = 0..L-1 (seed hop first, fanouts reversed as in the reference):
      S1  sample_hop      pick counts + look-back scan + Philox picks (+ coverage of the seeds)
      S2  compact         dst-first relabelling with a dense tagged id map (3 kernels)
  layer l = 0..L-1 (input layer first, on hop h = L-1-l):
      K-SpMM  aggregate   [h_dst | mean h_src] (layer 0 reads the resident feature table
                          through the block's source ids, so no gathered copy is made)
      K-GEMM  tcgen05     [h_dst | agg] . [W_self | W_neigh]^T + b, ReLU, dropout (hidden)
                          or the fused softmax cross-entropy + its gradient (last layer)
  backward, last layer first:
      K-GEMM  dW += dY^T X  (split-K, fp32 reductions straight into the flat gradient)
      K-GEMM  dX  = dY W    (MN-major operand, no transposes)
      K-SpMM  transpose aggregation into fp32 accumulators
      act_bwd ReLU/dropout mask from the stored activation, bias gradient, clears the accumulator
  K-AR   coverage-weighted all-reduce + Adam over NVLink peer memory (W > 1), or Adam (W = 1)

Every buffer is allocated once at its capacity (batch size times the fanout
products); the kernels read the live sizes from device counters, so the step has
no host synchronisation and is captured once into a CUDA graph and replayed.
"""
import math

import torch

from grappa_b200 import _native
from grappa_b200.models.flat import pad8
from grappa_b200.sampler_gpu import C_ADAM, C_EPOCH, C_SEED, C_STEP, GpuNeighborSampler, new_counters

GEMM_STORE_BF16, GEMM_STORE_F32, GEMM_ATOMIC_F32, GEMM_CROSS_ENTROPY = 0, 1, 2, 3
AGG_MEAN, AGG_SUM, AGG_GCN, AGG_WEIGHTED = 0, 1, 2, 3

# kernels launched by each binding (memsets excluded)
KERNELS_PER_CALL = {
    "sample_hop": 1, "compact": 3, "gemm": 1, "aggregate": 1, "aggregate_bwd": 1, "act_bwd": 1,
    "gather_scalar": 1, "gather_rows": 1, "adam": 1, "allreduce_adam": 1, "step_end": 1, "src_norm": 2,
    "pull_rows": 1, "csr_merge": 1, "mark_ids": 1, "iota_map": 1, "mark_compact": 1, "peer_copy": 1,
    "shuffle_keys": 1,
}


class LaunchCounter:
    """Proxy of the kernel module that counts the kernels each call launches."""

    def __init__(self, mod):
        self._mod = mod
        self.count = 0

    def __getattr__(self, name):
        f = getattr(self._mod, name)
        k = KERNELS_PER_CALL.get(name, 0)
        if not k:
            return f

        def wrapped(*a, **kw):
            self.count += k
            return f(*a, **kw)

        return wrapped


def bn_for(n):
    """Tile width of the GEMM for an output width n (K-major operands)."""
    if n == 48:
        return 48
    if n <= 64:
        return 64
    if n <= 128:
        return 128
    return 256


def split_k(rows, n_tiles, sms=148, min_kblocks=8):
    """Number of split-K slices for a dW GEMM over ``rows`` reduction rows."""
    kblocks = max(1, math.ceil(rows / 64))
    by_work = max(1, kblocks // min_kblocks)
    by_sms = max(1, (2 * sms) // max(1, n_tiles))
    return max(1, min(by_work, by_sms))


class SageEngine:
    """GraphSAGE (mean) mini-batch training on one rank's working graph."""

    def __init__(self, model, n_nodes_cap, fanouts, batch_size, device, lr=3e-3, comm=None, seed=0,
                 fused_allreduce=True, use_cuda_graph=True, betas=(0.9, 0.999), eps=1e-8):
        if getattr(model, "name", None) != "sage":
            raise ValueError("SageEngine trains GraphSAGE models")
        self.cu = LaunchCounter(_native.cuda())
        self.launches_per_step = 0
        self.model = model
        self.comm = comm
        self.world = 1 if comm is None else comm.world
        self.rank = 0 if comm is None else comm.rank
        self.fanouts = [int(f) for f in fanouts]
        self.L = len(self.fanouts)
        if self.L != model.n_layers:
            raise ValueError("one fanout per layer")
        self.B = int(batch_size)
        self.lr, self.betas, self.eps = float(lr), betas, float(eps)
        self.p = float(model.dropout_p)
        self.device = torch.device(device)
        self.seed = int(seed)
        self.use_cuda_graph = use_cuda_graph
        self.fused_allreduce = fused_allreduce and self.world > 1
        dev = self.device

        # parameters: flat fp32 master, bf16 working copy, gradient, Adam moments
        model.place(dev)
        self.flat = model.flat
        self.wbf = self.flat.to(torch.bfloat16)
        self.grad = torch.zeros_like(self.flat)
        self.m = torch.zeros_like(self.flat)
        self.v = torch.zeros_like(self.flat)

        # device scalars
        self.counters = new_counters(self.seed, dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.fstats = torch.zeros(4, dtype=torch.float32, device=dev)  # cov_sum, cov_n, loss_sum, spare
        self.istats = torch.zeros(2, dtype=torch.int32, device=dev)   # correct, spare
        self._ce_dummy = torch.zeros((1, 1), dtype=torch.float32, device=dev)
        self.allreduce = FusedAllReduceAdam(comm, self.flat.numel()) if self.fused_allreduce else None

        self.sm = GpuNeighborSampler(self.fanouts, self.B, n_nodes_cap, dev, cu=self.cu)
        self.seeds = self.sm.seeds
        self.seed_label = torch.zeros(self.B, dtype=torch.int32, device=dev)
        self._alloc_layers()
        self._working = None
        self._graph = None

    # ------------------------------------------------------------------ buffers
    def _alloc_layers(self):
        dev = self.device
        L, model = self.L, self.model
        self.lay = []
        for l, layer in enumerate(model.layers):
            h = L - 1 - l
            ip, op = pad8(layer.in_feats), pad8(layer.out_feats)
            K = 2 * ip
            rows = self.sm.cap_dst[h]
            seg_w = model.segment(layer.seg_w)
            seg_b = model.segment(layer.seg_b)
            spec = dict(h=h, ip=ip, op=op, K=K, rows=rows,
                        W=seg_w.view(self.wbf), bias=seg_b.view(self.flat)[0],
                        gW=seg_w.view(self.grad), gb=seg_b.view(self.grad)[0],
                        X=torch.zeros((rows, K), dtype=torch.bfloat16, device=dev),
                        dY=torch.zeros((rows, op), dtype=torch.bfloat16, device=dev))
            if l < L - 1:
                spec["H"] = torch.zeros((rows, op), dtype=torch.bfloat16, device=dev)
                spec["dH"] = torch.zeros((rows, op), dtype=torch.float32, device=dev)
            if l > 0:
                spec["dX"] = torch.zeros((rows, K), dtype=torch.bfloat16, device=dev)
            self.lay.append(spec)
        self.n_classes = model.n_classes

    # ------------------------------------------------------------------ graph binding
    def bind_working(self, working, labels, gideg):
        """Point the engine at a working graph (after a repartition)."""
        if working.indptr.numel() - 1 > self.sm.n_nodes_cap:
            raise ValueError("working graph larger than the engine's node capacity")
        self._working = working
        self.labels = labels
        self.gideg = gideg
        self._graph = None  # pointers may have changed: capture again

    def set_epoch(self, epoch):
        self.counters[C_EPOCH] = int(epoch)
        self.counters[C_STEP] = 0

    # ------------------------------------------------------------------ the step
    def _n_dst(self, h):
        return self.sm.n_dst(h)

    def _sample(self):
        w = self._working
        self.cu.gather_scalar(self.labels, self.sm.seeds, self.sm.n_seeds(), 0, self.B, self.seed_label)
        self.sm.sample(w.indptr, w.indices, self.counters, gideg=self.gideg, cov=self.fstats[0:2], err=self.err)

    def _forward(self, training=True):
        cu, w, sm = self.cu, self._working, self.sm
        L = self.L
        for l, s in enumerate(self.lay):
            h = s["h"]
            if l == 0:
                src, src_map = w.feat, sm.src[h]
            else:
                src, src_map = self.lay[l - 1]["H"], None
            cu.aggregate(sm.indptr[h], sm.indices[h], self._n_dst(h), 0, sm.cap_dst[h], src, src_map,
                         s["ip"], AGG_MEAN, None, None, None, s["X"], s["ip"], 0, 0.0, 0, self.err)
            bn = bn_for(s["op"])
            if l < L - 1:
                cu.gemm(s["X"], False, s["W"], False, s["rows"], self._n_dst(h), s["op"], s["K"], None, 1,
                        s["H"], GEMM_STORE_BF16, s["bias"], 1, self.p if training else 0.0,
                        self.counters, l, None, 0, None, None, None, None, None, None, self.err, bn)
            else:
                cu.gemm(s["X"], False, s["W"], False, s["rows"], self._n_dst(h), s["op"], s["K"], None, 1,
                        self._ce_dummy, GEMM_CROSS_ENTROPY, s["bias"], 0, 0.0, None, 0, self.seed_label,
                        self.n_classes, s["dY"], self.fstats[2:3], self.istats[0:1], None, self.sm.n_seeds(),
                        s["gb"] if training else None, self.err, bn)

    def _backward(self):
        cu, sm = self.cu, self.sm
        L = self.L
        scale = 1.0 / (1.0 - self.p) if self.p > 0 else 1.0
        for l in range(L - 1, -1, -1):
            s = self.lay[l]
            h = s["h"]
            n_tiles = math.ceil(s["op"] / 128) * math.ceil(s["K"] / 256)
            # dW += dY^T X (split-K over the block's rows, fp32 reductions into the gradient)
            cu.gemm(s["dY"], True, s["X"], True, s["op"], None, s["K"], s["rows"], self._n_dst(h),
                    split_k(s["rows"], n_tiles), s["gW"], GEMM_ATOMIC_F32, None, 0, 0.0, None, 0, None, 0,
                    None, None, None, None, None, None, self.err, 256)
            if l == 0:
                break
            # dX = dY W (W read MN-major)
            cu.gemm(s["dY"], False, s["W"], True, s["rows"], self._n_dst(h), s["K"], s["op"], None, 1, s["dX"],
                    GEMM_STORE_BF16, None, 0, 0.0, None, 0, None, 0, None, None, None, None, None, None, self.err,
                    256)
            prev = self.lay[l - 1]
            # transpose aggregation: d(self) -> dst rows, d(agg) -> sources
            cu.aggregate_bwd(sm.indptr[h], sm.indices[h], self._n_dst(h), 0, sm.cap_dst[h], s["dX"],
                             s["ip"], 0, 0.0, s["ip"], AGG_MEAN, None, None, None, prev["dH"], self.err)
            cu.act_bwd(prev["dH"], prev["H"], prev["dY"], self._n_dst(prev["h"]), 0, prev["op"], scale, prev["gb"],
                       prev["rows"])

    def _update(self):
        cu = self.cu
        b1, b2 = self.betas
        if self.fused_allreduce:
            self.allreduce.step(self.grad, self.fstats[0:2], self.counters, self.flat, self.m, self.v, self.wbf,
                                self.lr, b1, b2, self.eps, self.err, cu=cu)
        elif self.world > 1:
            # the reference's path (t10n/grad.py:6-24): scale by c_r / W, NCCL SUM all-reduce, Adam
            import torch.distributed as dist

            c = self.fstats[0:1] / self.fstats[1:2].clamp(min=1.0)
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
        self._backward()
        self._update()
        self.cu.step_end(self.counters)

    def capture(self):
        """Capture the step into a CUDA graph (after one eager step has run)."""
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self._step_body()
        torch.cuda.current_stream(self.device).wait_stream(s)
        self._graph = g

    def load_seeds(self, seeds, count):
        """Copy this step's seeds ([B] int32) and seed count ([1] int32) into the static
        buffers.  Both may live in device memory or in pinned host memory; they are
        plain copies (no kernels) and must stay unchanged until the step has run."""
        self.seeds.copy_(seeds, non_blocking=True)
        self.sm.cnt[0:1].copy_(count, non_blocking=True)

    def step(self, seeds=None, count=None):
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
        """Forward only (dropout off) for the given seeds; returns (correct, loss) on the device."""
        self.load_seeds(seeds, count)
        self.cu.zero_(self.fstats)
        self.cu.zero_(self.istats)
        self._sample()
        self._forward(training=False)
        return self.istats[0:1], self.fstats[2:3]

    def check_errors(self):
        e = int(self.err.item())
        if e:
            raise RuntimeError(f"device error word {e:#x} (bits: grappa_b200/csrc/cuda/common.cuh kErr*)")


class FusedAllReduceAdam:
    """Coverage-weighted gradient all-reduce fused with Adam (peer memory, one kernel)."""

    def __init__(self, comm, n, chunk=4096, timeout_s=30.0):
        from grappa_b200.parallel.comm import PeerBuffer

        self.comm = comm
        self.n = int(n)
        self.chunk = int(chunk)
        self.n_chunks = (self.n + self.chunk - 1) // self.chunk
        W = comm.world
        half = (self.n * 4 + 255) // 256 * 256
        flag_bytes = (W * self.n_chunks * 4 + 255) // 256 * 256
        self.buf = PeerBuffer(comm, 2 * half + flag_bytes)
        me = comm.rank
        self.send_local = [self.buf.ptrs[me], self.buf.ptrs[me] + half]
        self.send_peer = []
        for p in range(W):
            self.send_peer += [self.buf.ptrs[p], self.buf.ptrs[p] + half]
        self.flags_local = self.buf.ptrs[me] + 2 * half
        self.flags_peer = [self.buf.ptrs[p] + 2 * half for p in range(W)]
        self.timeout_ns = int(timeout_s * 1e9)
        torch.cuda.synchronize()
        comm.barrier()

    def step(self, grad, cov, counters, param, m, v, wbf, lr, b1, b2, eps, err, grid=0, cu=None):
        cu = cu or _native.cuda()
        cu.allreduce_adam(self.comm.rank, self.comm.world, grad, self.chunk, self.send_local, self.send_peer,
                          self.flags_local, self.flags_peer, cov, counters, param, m, v, wbf, lr, b1, b2, eps, 0.0,
                          True, None, err, grid, self.timeout_ns)

    def reduce(self, grad, cov, counters, out, err, grid=0):
        """All-reduce only (no Adam): out = sum_r c_r grad_r / W."""
        _native.cuda().allreduce_adam(self.comm.rank, self.comm.world, grad, self.chunk, self.send_local,
                                      self.send_peer, self.flags_local, self.flags_peer, cov, counters, None, None,
                                      None, None, 0.0, 0.9, 0.999, 1e-8, 0.0, False, out, err, grid, self.timeout_ns)

    def close(self):
        self.buf.close()
