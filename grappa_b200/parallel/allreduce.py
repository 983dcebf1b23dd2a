"""K-AR: coverage-weighted gradient all-reduce fused with Adam over NVLink peer memory.

The reference aggregates gradients with a DDP comm hook that scales each bucket by
the rank's coverage weight c_r and divides by W before an NCCL SUM all-reduce, then
steps torch.optim.Adam (t10n/grad.py:6-24; registered at
experiments/grappa/train/t10n_train.py:103-114,160-162; optimizer step at :248).
DDP reduces a bucket as soon as autograd has produced it.

Here the gradient, the fp32 master weights and the send slots live in buffers that
every rank maps (CUDA IPC), and one sm_100a kernel per gradient bucket
(grappa_b200/csrc/cuda/allreduce.cu) scales, casts (bf16 gradients), reduces and
applies Adam:

  * one-shot: publish a scaled fp32 copy, one flag round trip, every rank reads all W
    copies and updates the whole bucket (small buckets: lowest latency);
  * shard: reduce-scatter (the owner of each shard reads it straight from every rank's
    gradient buffer), Adam on the owned shard, all-gather of the updated fp32 master
    weights (large buckets: (W-1)/W of the gradient and of the parameters cross NVLink
    per rank, 1/W of the Adam work).  The Adam moments of a shard are kept by its
    owner only; ``sync_moments`` gathers them (checkpoints).

Buckets are contiguous element ranges of the flat parameter buffer (one per model
layer in the engines), launched in the order the backward pass completes them, so
that a bucket's reduction overlaps the backward of the layers before it.
"""
import math

import torch

from grappa_b200 import _native

ONE_SHOT, SHARD = 0, 1
_FLAG_PAGE = 2 * 8 * 160 * 4  # ready[rank][cta] + done[rank][cta] words (allreduce.h kFlagPageBytes)
_MAX_CTAS = 148


def _r256(n):
    return (int(n) + 255) // 256 * 256


class FusedAllReduceAdam:
    """Per-bucket fused all-reduce + Adam for one data-parallel group (one rank per GPU).

    ``grad`` ([n], fp32 or bf16) and ``param`` ([n] fp32) are tensors over this rank's
    peer-mapped buffers: the caller accumulates gradients into ``grad`` and uses
    ``param`` as the fp32 master weights (``adopt_params`` re-homes a model's flat
    buffer there).  ``bind`` fixes the remaining arguments; ``launch(k)`` enqueues bucket
    k's kernel on the current stream.  Every rank must create the object with the same
    n, buckets and modes, and launch the same buckets in the same order every step;
    the step tag is counters[3] (global step), so a bucket runs at most once per step.

    Mode per bucket: one-shot when the bucket is at most ``one_shot_max_bytes(W)`` of
    gradient, otherwise shard (``modes`` overrides).
    """

    @staticmethod
    def one_shot_max_bytes(world):
        # one-shot reads W-1 peer copies against 2 (W-1)/W for the shard mode, but pays
        # one flag round trip instead of two.  Measured crossovers (fp32): W = 2 between
        # 4 and 16 MB, W = 4 at 4 MB (41.0 vs 41.8 us), W = 8 between 1 MB (36.2 vs
        # 54.8 us) and 4 MB (82.7 vs 60.3 us)
        if world <= 2:
            return 8 << 20
        if world <= 4:
            return 4 << 20
        return 2 << 20

    def __init__(self, comm, n, buckets=None, grad_dtype=torch.float32, modes=None, timeout_s=30.0, grids=None):
        from grappa_b200.parallel.comm import PeerBuffer

        self.comm = comm
        self.W, self.rank = comm.world, comm.rank
        self.n = int(n)
        self.buckets = [(0, self.n)] if buckets is None else [(int(a), int(b)) for a, b in buckets]
        prev = 0
        for lo, hi in self.buckets:
            if lo % 8 or lo < prev or hi < lo or hi > self.n:
                raise ValueError(f"bucket ({lo}, {hi}) must start on a multiple of 8, in order, inside [0, {self.n})")
            prev = hi
        if grad_dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("gradients are fp32 or bf16")
        self.grad_dtype = grad_dtype
        esz = 4 if grad_dtype == torch.float32 else 2
        if modes is None:
            lim = self.one_shot_max_bytes(self.W)
            modes = [ONE_SHOT if (hi - lo) * esz <= lim else SHARD for lo, hi in self.buckets]
        self.modes = [int(m) for m in modes]
        if len(self.modes) != len(self.buckets):
            raise ValueError("one mode per bucket")
        self.grids = list(grids) if grids is not None else [self._grid(lo, hi, m, esz)
                                                            for (lo, hi), m in zip(self.buckets, self.modes)]
        self.timeout_ns = int(timeout_s * 1e9)
        nb = len(self.buckets)
        self._gbuf = PeerBuffer(comm, _r256(self.n * esz))
        self._pbuf = PeerBuffer(comm, _r256(self.n * 4))
        self._sbuf = PeerBuffer(comm, 2 * _r256(self.n * 4)) if ONE_SHOT in self.modes else None
        self._cbuf = PeerBuffer(comm, nb * _FLAG_PAGE + _r256(nb * 2 * 4))
        self.grad = self._gbuf.tensor(grad_dtype, [self.n])
        self.param = self._pbuf.tensor(torch.float32, [self.n])
        self.plan = None
        self._model = None
        torch.cuda.synchronize()
        comm.barrier()

    def _grid(self, lo, hi, mode, esz):
        """CTAs of a bucket's launch: about 64 KB of peer reads or 256 KB of local Adam
        traffic per CTA, whichever asks for more, 8 at least (the flag round trips
        dominate small buckets) and one per SM at most.  The local traffic is 30 bytes
        per updated element (fp32 master, both moments, bf16 copy) plus the one-shot
        mode's published copy and its W reads."""
        n = hi - lo
        W = self.W
        if mode == ONE_SHOT:
            peer, local = n * 4 * (W - 1), n * (30 + 4 * (W + 1))
        else:
            peer, local = n * esz * (W - 1) / W, n * (30.0 / W + 2 * esz)
        want = max(math.ceil(peer / 65536), math.ceil(local / 262144))
        return int(max(8, min(_MAX_CTAS, want)))

    # ---------------------------------------------------------------------- binding
    def adopt_params(self, model):
        """Copy ``model.flat`` into the peer-mapped master buffer and re-bind the model's
        parameter views to it (``release_params`` moves them back to ordinary memory)."""
        if model.flat.numel() != self.n:
            raise ValueError("model size differs from the all-reduce buffer")
        self.param.copy_(model.flat)
        model._rebind(self.param)
        self._model = model

    def release_params(self):
        if self._model is not None:
            self._model._rebind(self.param.clone())
            self._model = None

    def bind(self, counters, m, v, wbf, lr, betas=(0.9, 0.999), eps=1e-8, err=None, weight_decay=0.0, cov=None,
             do_adam=True, grad_out=None):
        """Build the launch plan: Adam state (m, v, wbf on this rank, each [n]), the device
        counters ([seed, epoch, step, global_step, gen, adam_t]), the error word and the
        default coverage tensor ([sum, count], None for weight 1)."""
        cu = _native.cuda()
        W, r = self.W, self.rank
        plan = cu.ArPlan()
        nb = len(self.buckets)
        scale_base = [self._cbuf.ptrs[p] + nb * _FLAG_PAGE for p in range(W)]
        for k, ((lo, hi), mode) in enumerate(zip(self.buckets, self.modes)):
            page = [self._cbuf.ptrs[p] + k * _FLAG_PAGE for p in range(W)]
            scales = [scale_base[p] + k * 8 for p in range(W)]
            if mode == ONE_SHOT:
                half = _r256(self.n * 4)
                slot_local = [self._sbuf.local, self._sbuf.local + half]
                slot_peer = []
                for p in range(W):
                    slot_peer += [self._sbuf.ptrs[p], self._sbuf.ptrs[p] + half]
            else:
                slot_local, slot_peer = [], []
            plan.add(rank=r, world=W, mode=mode, grad_bf16=self.grad_dtype == torch.bfloat16, lo=lo, hi=hi,
                     grad=self._gbuf.local, grad_peer=list(self._gbuf.ptrs) if mode == SHARD else [],
                     slot_local=slot_local, slot_peer=slot_peer, param=self._pbuf.local,
                     param_peer=list(self._pbuf.ptrs) if mode == SHARD else [], m=m, v=v, wbf=wbf,
                     scale_local=scales[r], scale_peer=scales if mode == SHARD else [], flags_local=page[r],
                     flags_peer=page, cov=cov, counters=counters, lr=float(lr), b1=float(betas[0]),
                     b2=float(betas[1]), eps=float(eps), wd=float(weight_decay), do_adam=do_adam,
                     grad_out=grad_out, err=err, grid=self.grids[k], timeout_ns=self.timeout_ns)
        self.plan = plan
        return self

    def launch(self, k, cov=None):
        """Enqueue bucket k on the current stream (``cov`` overrides the bound coverage)."""
        self.plan.launch(int(k), cov)

    def launch_all(self, cov=None):
        for k in range(len(self.buckets)):
            self.launch(k, cov)

    # ---------------------------------------------------------------------- moments
    def shard_range(self, k, s):
        """Element range of shard s of bucket k (the kernel's split)."""
        lo, hi = self.buckets[k]
        S = (math.ceil((hi - lo) / self.W) + 7) // 8 * 8
        a = min(hi, lo + s * S)
        return a, min(hi, a + S)

    def sync_moments(self, m, v):
        """Gather the Adam moments of every sharded bucket from the shard owners (a
        collective: every rank calls it), so that m and v are complete on every rank."""
        import torch.distributed as dist

        if self.W == 1 or SHARD not in self.modes:
            return
        for k, mode in enumerate(self.modes):
            if mode != SHARD:
                continue
            for buf in (m, v):
                parts = []
                for s in range(self.W):
                    a, b = self.shard_range(k, s)
                    parts.append(buf[a:b].clone())
                for s in range(self.W):
                    dist.broadcast(parts[s], src=s)
                for s in range(self.W):
                    a, b = self.shard_range(k, s)
                    buf[a:b].copy_(parts[s])

    def close(self):
        self.release_params()
        self.plan = None
        for b in (self._gbuf, self._pbuf, self._sbuf, self._cbuf):
            if b is not None:
                b.close()
