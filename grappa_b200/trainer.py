"""Public training API: isolated partition training with periodic repartitioning.

``MiniBatchTrainer`` reproduces the reference's epoch structure
(experiments/grappa/train/t10n_train.py:148-350 with t10n/dataloader.py):
  * every rank trains on its own training nodes; the number of steps per epoch is
    equalised across ranks (all-reduce MAX of the local batch counts, batch size
    re-adjusted to ceil(n_train / n_batches), t10n/dataloader.py:200-213);
  * every ``repart_every`` epochs (starting at epoch 0) the rank switches to the next
    neighbour partition of the round-robin schedule (t10n/dataloader.py:547-553);
  * seeds are reshuffled every epoch;
  * gradients are aggregated with the coverage-corrected all-reduce.

Seeds can be fed from device memory (``host_feed=False``) or, as a user with data
on the host would, from pinned host memory with the loss read back every step
(``host_feed=True``).
"""
import math
import time

import torch

from grappa_b200.dataset.synthetic import shuffle_keys
from grappa_b200.engine import make_engine
from grappa_b200.graph_store import PartitionStore, next_neighbor


class MiniBatchTrainer:
    def __init__(self, model, own, fanouts, batch_size, lr=3e-3, repart_every=10, comm=None, seed=0,
                 fused_allreduce=True, use_cuda_graph=True, ar_mode=None, overlap_allreduce=True):
        self.model = model
        self.own = own
        self.comm = comm
        self.rank = own.rank
        self.world = own.world
        self.repart_every = max(1, int(repart_every))
        self.seed = int(seed)
        self.device = own.indices.device
        self.store = PartitionStore(own, comm)
        self.nbr_idx = self.rank
        self._last_repart = None
        self.repart_seconds = []
        tr = torch.nonzero(own.train_mask).squeeze(1)
        self.train_ids = tr.to(torch.int64)
        n_local = int(tr.numel())
        nb = max(1, math.ceil(n_local / batch_size))
        if comm is not None and comm.world > 1:
            nb = int(comm.all_reduce_max([nb])[0])
        self.n_batches = nb
        self.batch_size = max(1, math.ceil(n_local / nb))  # reference: adjust_bs
        self.engine = make_engine(model, self.store.cap_nodes, fanouts, self.batch_size, self.device, lr=lr,
                                 comm=comm, seed=seed, fused_allreduce=fused_allreduce,
                                 use_cuda_graph=use_cuda_graph, ar_mode=ar_mode,
                                 overlap_allreduce=overlap_allreduce)
        self._maybe_repartition(0)
        self._warm = False

    # ------------------------------------------------------------------ schedule
    def epoch_seeds(self, epoch, on_host):
        """Shuffled seeds of an epoch as [n_batches, B] int32 plus counts [n_batches, 1]."""
        B, nb = self.batch_size, self.n_batches
        if on_host:
            ids = self.train_ids.cpu()
            perm = ids[torch.argsort(shuffle_keys(ids, self.seed, epoch), stable=True)].to(torch.int32)
            seeds = torch.zeros((nb, B), dtype=torch.int32).pin_memory()
            counts = torch.zeros((nb, 1), dtype=torch.int32).pin_memory()
        else:
            ids = self.train_ids
            perm = ids[torch.argsort(shuffle_keys(ids, self.seed, epoch), stable=True)].to(torch.int32)
            seeds = torch.zeros((nb, B), dtype=torch.int32, device=self.device)
            # the per-batch counts never change: uploaded once (a pageable host -> device
            # copy every epoch would wait for the previous epoch's work to drain)
            if getattr(self, "_dev_counts", None) is None:
                n = perm.numel()
                self._dev_counts = torch.tensor([[max(0, min(B, n - s * B))] for s in range(nb)],
                                                dtype=torch.int32).to(self.device)
            seeds.view(-1)[:perm.numel()].copy_(perm)
            return seeds, self._dev_counts
        n = perm.numel()
        seeds.view(-1)[:n].copy_(perm)
        counts.copy_(torch.tensor([[max(0, min(B, n - s * B))] for s in range(nb)], dtype=torch.int32))
        return seeds, counts

    # ------------------------------------------------------------------ host feed
    def _host_buffers(self, slot):
        """Two pinned [n_batches, B] seed / [n_batches, 1] count buffers (epochs alternate
        between them) and the pinned per-step loss ring, allocated once."""
        if getattr(self, "_pinned", None) is None:
            nb, B = self.n_batches, self.batch_size
            self._pinned = [(torch.zeros((nb, B), dtype=torch.int32).pin_memory(),
                             torch.zeros((nb, 1), dtype=torch.int32).pin_memory()) for _ in range(2)]
            self._ring = torch.zeros(nb, dtype=torch.float32).pin_memory()
            self._train_ids_host = self.train_ids.cpu()
            B_, n = self.batch_size, self._train_ids_host.numel()
            self._host_counts = torch.tensor([[max(0, min(B_, n - s * B_))] for s in range(nb)], dtype=torch.int32)
        return self._pinned[slot]

    def _fill_host_seeds(self, epoch):
        """The epoch's shuffled seeds (the same order as ``epoch_seeds``) in its pinned slot."""
        seeds, counts = self._host_buffers(epoch & 1)
        ids = self._train_ids_host
        perm = ids[torch.argsort(shuffle_keys(ids, self.seed, epoch), stable=True)].to(torch.int32)
        seeds.view(-1)[:perm.numel()].copy_(perm)
        counts.copy_(self._host_counts)
        return seeds, counts

    def _host_seeds(self, epoch):
        fut = getattr(self, "_prefetched", {}).pop(epoch, None)
        return fut.result() if fut is not None else self._fill_host_seeds(epoch)

    def _prefetch_host_seeds(self, epoch):
        """Shuffle the next epoch's seeds on a host thread while this epoch runs on the
        device (its pinned slot is not the one the current epoch's copies read)."""
        if getattr(self, "_pool", None) is None:
            from concurrent.futures import ThreadPoolExecutor

            self._pool = ThreadPoolExecutor(max_workers=1)
            self._prefetched = {}
        self._prefetched[epoch] = self._pool.submit(self._fill_host_seeds, epoch)

    def _maybe_repartition(self, epoch):
        first = self._last_repart is None
        if not first and (epoch % self.repart_every != 0 or epoch == self._last_repart):
            return
        t0 = time.perf_counter()
        if self.world > 1:
            self.nbr_idx = next_neighbor(self.nbr_idx, self.rank, self.world)
        w = self.store.repartition(self.nbr_idx)
        self.engine.bind_working(w, self.own.label, self.own.gideg)
        self._last_repart = epoch
        if not first:
            self.repart_seconds.append(time.perf_counter() - t0)

    # ------------------------------------------------------------------ epochs
    def warmup(self):
        """Run one eager step (kernel attributes, tensor maps), then capture the step graph."""
        if self._warm:
            return
        seeds, counts = self.epoch_seeds(0, on_host=False)
        self.engine.set_epoch(0)
        self.engine.step(seeds[0], counts[0])
        torch.cuda.synchronize(self.device)
        self.engine.check_errors()
        self.engine.prepare()
        self._warm = True

    def train_epoch(self, epoch, host_feed=False):
        """Run one epoch.  With ``host_feed`` the seeds come from pinned host memory and
        every step's loss is copied back; returns the mean loss then (else None).
        With a ``watchdog`` (grappa_b200.parallel.watchdog.Heartbeat) set, a peer that
        left the job raises PeerFailure here, before any collective of the epoch."""
        if getattr(self, "watchdog", None) is not None:
            self.watchdog.check()
        self._maybe_repartition(epoch)
        if self._warm:
            self.engine.prepare()
        if host_feed:
            seeds, counts = self._host_seeds(epoch)
        else:
            seeds, counts = self.epoch_seeds(epoch, on_host=False)
        self.engine.set_epoch(epoch)
        # device -> host read of every step's loss (pinned, asynchronous)
        ring = self._ring if host_feed else None
        self.engine.run_epoch(seeds, counts, ring)
        if host_feed:
            self._prefetch_host_seeds(epoch + 1)
            torch.cuda.current_stream(self.device).synchronize()
            self.last_losses = ring.clone()
            return float(self.last_losses.mean())
        return None

    def evaluate(self, mask, fanouts=None):
        """Accuracy on the own nodes selected by ``mask`` with sampled neighbourhoods
        (the training fanouts), all on the device; summed over ranks."""
        ids = torch.nonzero(mask).squeeze(1).to(torch.int32)
        B = self.batch_size
        correct, total = 0.0, 0.0
        for s in range(0, ids.numel(), B):
            part = ids[s:s + B]
            buf = torch.zeros(B, dtype=torch.int32, device=self.device)
            buf[: part.numel()] = part
            c, _ = self.engine.predict(buf, torch.tensor([part.numel()], dtype=torch.int32, device=self.device))
            correct += float(c.item())
            total += part.numel()
        if self.comm is not None and self.comm.world > 1:
            correct, total = self.comm.all_reduce_sum([correct, total])
        return correct / max(total, 1.0)

    def evaluate_exact(self, masks):
        """Exact accuracy (full neighbourhoods across partitions, layer by layer, the
        reference's run_infer_xborder_by_layer) on the own nodes selected by each mask,
        over all ranks; a collective.  ``evaluate`` samples instead."""
        return _exact_accuracy(self, masks)

    def load_state_dict(self, state_dict):
        """Load model weights into the flat master buffer and refresh the bf16 working copy."""
        self.model.load_state_dict(state_dict)
        with torch.no_grad():
            self.engine.wbf.copy_(self.engine.flat)

    def close(self):
        if getattr(self, "_pool", None) is not None:
            self._pool.shutdown(wait=True)
            self._pool = None
        if getattr(self, "_exact", None) is not None:
            self._exact.close()
            self._exact = None
        self.engine._graph = None
        if self.engine.allreduce is not None:
            self.engine.allreduce.close()
        self.store.close()


def _exact_accuracy(trainer, masks):
    from grappa_b200.infer_gpu import ExactInference

    torch.cuda.synchronize(trainer.device)
    if getattr(trainer, "_exact", None) is None:
        trainer._exact = ExactInference(trainer.model, trainer.own, trainer.comm)
    return trainer._exact.accuracy(masks)


def full_graph_blocks(working, n_layers, own, cap_nodes=0, cap_edges=0, into=None):
    """FullGraphBlocks of the working graph's own + neighbour rows: the in-edges whose
    source is one of those rows (halo sources dropped, as the reference's isolated
    full-graph partition holds only the two chunks, t10n/dataloader.py:492-502).
    Labels and the training mask exist for the own rows only.  ``into``: a FullGraphBlocks
    to refill in place when the graph fits (its pointers, and a step graph captured on
    them, stay valid); ``cap_nodes`` / ``cap_edges`` size a new one.

    The coverage weight c_r of the partition is the mini-batch path's per-seed ratio
    (csrc/graph/sampling_h.h:97-116, t10n/dataloader.py:647-663) averaged over every
    own training node, with the kept in-degree in place of the sampled node's local
    degree: r_v = min(1, (max(kept_v - 1, 0) + 1) / (global_indeg_v + 1)).  kept_v
    counts v's self-loop, global_indeg_v does not.  An own node whose in-neighbours all
    lie in the own or the neighbour partition has r_v = 1; one that lost in-edges to a
    third partition has r_v < 1.  Computed on the device, once per repartition."""
    from grappa_b200.engine import FullGraphBlocks

    n = int(working.n_own + working.n_nbr)
    dev = working.indices.device
    ip = working.indptr[: n + 1].to(torch.int64)
    E = int(ip[-1].item())
    ind = working.indices[:E].to(torch.int64)
    keep = ind < n
    deg = (ip[1:] - ip[:-1])
    row = torch.repeat_interleave(torch.arange(n, device=dev), deg)
    cnt = torch.bincount(row[keep], minlength=n)
    new_ip = torch.zeros(n + 1, dtype=torch.int64, device=dev)
    new_ip[1:] = torch.cumsum(cnt, 0)
    labels = torch.zeros(n, dtype=torch.int32, device=dev)
    labels[: working.n_own] = own.label
    train = torch.zeros(n, dtype=torch.uint8, device=dev)
    train[: working.n_own] = own.train_mask.to(torch.uint8)
    cov = coverage_of_rows(cnt[: working.n_own], own.gideg.to(dev), own.train_mask.to(dev))
    ind = ind[keep]
    if into is not None and into.refill(new_ip, ind, labels, train, cov):
        return into
    return FullGraphBlocks(new_ip, ind, n_layers, dev, labels, train, cov=cov, cap_nodes=cap_nodes,
                           cap_edges=cap_edges)


def coverage_of_rows(kept_deg, gideg, mask):
    """[sum, count] of min(1, (max(kept - 1, 0) + 1) / (gideg + 1)) over the rows selected
    by ``mask`` (float32, on the rows' device)."""
    up = (kept_deg.to(torch.float32) - 1.0).clamp(min=0.0) + 1.0
    r = (up / (gideg.to(torch.float32).clamp(min=0.0) + 1.0)).clamp(max=1.0)
    sel = mask.to(torch.bool)
    return torch.stack([r[sel].sum(), sel.sum().to(torch.float32)]).to(torch.float32)


class FullGraphTrainer:
    """Isolated full-graph training of one partition (reference:
    experiments/grappa/train/t10n_fullgraph_train.py:142-254): every epoch is one step
    over the whole working graph (own + neighbour partition), loss on the own training
    nodes, coverage-corrected gradient aggregation across ranks (c_r from the kept
    in-degrees of the own training nodes, ``full_graph_blocks``), repartitioned every
    ``repart_every`` epochs.  The reference computes the loss on every own node
    (training, validation and test); here only the training nodes contribute."""

    def __init__(self, model, own, lr=3e-3, repart_every=10, comm=None, seed=0, fused_allreduce=True,
                 use_cuda_graph=True, ar_mode=None):
        from grappa_b200.engine import make_engine

        self.model, self.own, self.comm = model, own, comm
        self.rank, self.world = own.rank, own.world
        self.repart_every = max(1, int(repart_every))
        self.device = own.indices.device
        self.store = PartitionStore(own, comm)
        self.nbr_idx = self.rank
        self._last_repart = None
        self.repart_seconds = []
        if self.world > 1:
            self.nbr_idx = next_neighbor(self.nbr_idx, self.rank, self.world)
        w = self.store.repartition(self.nbr_idx)
        # capacity of the own + neighbour rows and their edges over every repartition
        self._caps = (getattr(self.store, "cap_own_nbr", 0), getattr(self.store, "cap_edges", 0))
        blocks = full_graph_blocks(w, len(model.layers), own, *self._caps)
        self.engine = make_engine(model, self.store.cap_nodes, [], 0, self.device, lr=lr, comm=comm, seed=seed,
                                  fused_allreduce=fused_allreduce, use_cuda_graph=use_cuda_graph, blocks=blocks,
                                  ar_mode=ar_mode)
        self.engine.bind_working(w, own.label, own.gideg)
        self._last_repart = 0
        self._warm = False

    def _maybe_repartition(self, epoch):
        if self.world == 1 or epoch % self.repart_every != 0 or epoch == self._last_repart:
            return
        t0 = time.perf_counter()
        self.nbr_idx = next_neighbor(self.nbr_idx, self.rank, self.world)
        w = self.store.repartition(self.nbr_idx)
        cur = self.engine.sm
        blocks = full_graph_blocks(w, len(self.model.layers), self.own, *self._caps, into=cur)
        if blocks is not cur:
            self.engine.set_blocks(blocks)
            self._warm = False
        self.engine.bind_working(w, self.own.label, self.own.gideg)
        if self.engine._graph is None:
            self._warm = False
        self._last_repart = epoch
        self.repart_seconds.append(time.perf_counter() - t0)

    def warmup(self):
        if self._warm:
            return
        self.engine.set_epoch(0)
        self.engine.step()
        torch.cuda.synchronize(self.device)
        self.engine.check_errors()
        self.engine.prepare()
        self._warm = True

    def train_epoch(self, epoch, read_loss=True):
        self._maybe_repartition(epoch)
        if not self._warm:
            self.warmup()
        self.engine.set_epoch(epoch)
        self.engine.step()
        if read_loss:
            return float(self.engine.fstats[2].item())
        return None

    def evaluate(self, mask):
        """Accuracy (forward without dropout) on the own rows selected by ``mask``, summed over ranks."""
        sm = self.engine.sm
        keep_mask, keep_sel = sm.row_mask, sm.n_sel
        m = torch.zeros_like(keep_mask)
        m[: self.own.n_nodes] = mask.to(torch.uint8)
        sm.row_mask = m
        sm.n_sel = torch.tensor([int(m.sum())], dtype=torch.int32, device=self.device)
        c, _ = self.engine.predict(None, None)
        correct, total = float(c.item()), float(sm.n_sel.item())
        sm.row_mask, sm.n_sel = keep_mask, keep_sel
        if self.comm is not None and self.comm.world > 1:
            correct, total = self.comm.all_reduce_sum([correct, total])
        return correct / max(total, 1.0)

    def evaluate_exact(self, masks):
        """Exact full-neighbour layer-wise accuracy over all ranks (see MiniBatchTrainer)."""
        return _exact_accuracy(self, masks)

    def load_state_dict(self, state_dict):
        """Load model weights into the flat master buffer and refresh the bf16 working copy."""
        self.model.load_state_dict(state_dict)
        with torch.no_grad():
            self.engine.wbf.copy_(self.engine.flat)

    def close(self):
        if getattr(self, "_exact", None) is not None:
            self._exact.close()
            self._exact = None
        self.engine._graph = None
        if self.engine.allreduce is not None:
            self.engine.allreduce.close()
        self.store.close()
