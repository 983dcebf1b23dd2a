"""Host-side failure detection between training steps.

Every rank publishes a heartbeat (a monotonic counter and its wall time) in the
job's key-value store from a background thread; ``check()`` (called by the
training loop between steps, never with kernels of this rank waiting on peers)
raises ``PeerFailure`` naming the ranks whose heartbeat is older than the limit.
A rank that leaves the job therefore stops the others before their next
collective launch instead of letting them wait in a peer-memory kernel or an
NCCL call.  The reference has no failure detection (24 h process-group timeouts,
experiments/grappa/train/t10n_train.py:373,390).
"""
import threading
import time


class PeerFailure(RuntimeError):
    pass


class Heartbeat:
    def __init__(self, store, rank, world, interval_s=0.5, limit_s=5.0, prefix="grappa_hb"):
        self.store, self.rank, self.world = store, int(rank), int(world)
        self.interval_s, self.limit_s, self.prefix = float(interval_s), float(limit_s), prefix
        self._stop = threading.Event()
        self._count = 0
        self._beat()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def _key(self, r):
        return f"{self.prefix}/{r}"

    def _beat(self):
        self._count += 1
        self.store.set(self._key(self.rank), f"{self._count}:{time.time():.6f}")

    def _run(self):
        while not self._stop.wait(self.interval_s):
            try:
                self._beat()
            except Exception:  # the store is gone: the job is ending
                return

    def ages(self):
        """Seconds since every peer's last heartbeat (inf if it never beat or the read fails)."""
        now = time.time()
        out = {}
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                val = self.store.get(self._key(r)).decode()
                out[r] = now - float(val.split(":")[1])
            except Exception:
                out[r] = float("inf")
        return out

    def check(self):
        stale = {r: a for r, a in self.ages().items() if a > self.limit_s}
        if stale:
            raise PeerFailure(f"rank {self.rank}: no heartbeat from rank(s) {sorted(stale)} "
                              f"for more than {self.limit_s:.1f} s")

    def stop(self):
        self._stop.set()
        self._thread.join(timeout=5)


def default_store():
    """The store of the default process group (torchrun / init_process_group)."""
    import torch.distributed as dist

    return dist.distributed_c10d._get_default_store()
