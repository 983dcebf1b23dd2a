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
from grappa_b200.engine import SageEngine
from grappa_b200.graph_store import PartitionStore, next_neighbor


class MiniBatchTrainer:
    def __init__(self, model, own, fanouts, batch_size, lr=3e-3, repart_every=10, comm=None, seed=0,
                 fused_allreduce=True, use_cuda_graph=True):
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
        self.engine = SageEngine(model, self.store.cap_nodes, fanouts, self.batch_size, self.device, lr=lr,
                                 comm=comm, seed=seed, fused_allreduce=fused_allreduce,
                                 use_cuda_graph=use_cuda_graph)
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
            counts = torch.zeros((nb, 1), dtype=torch.int32, device=self.device)
        n = perm.numel()
        seeds.view(-1)[:n].copy_(perm)
        counts.copy_(torch.tensor([[max(0, min(B, n - s * B))] for s in range(nb)], dtype=torch.int32))
        return seeds, counts

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
        every step's loss is copied back; returns the mean loss then (else None)."""
        self._maybe_repartition(epoch)
        if self._warm:
            self.engine.prepare()
        seeds, counts = self.epoch_seeds(epoch, on_host=host_feed)
        self.engine.set_epoch(epoch)
        ring = torch.zeros(self.n_batches, dtype=torch.float32).pin_memory() if host_feed else None
        for s in range(self.n_batches):
            self.engine.step(seeds[s], counts[s])
            if host_feed:
                # device -> host read of the step's loss (pinned, asynchronous)
                ring[s:s + 1].copy_(self.engine.fstats[2:3], non_blocking=True)
        if host_feed:
            torch.cuda.current_stream(self.device).synchronize()
            self.last_losses = ring
            return float(ring.mean())
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

    def close(self):
        self.engine._graph = None
        if self.engine.allreduce is not None:
            self.engine.allreduce.close()
        self.store.close()
