"""Failure handling of the training entry points: peer watchdog, periodic checkpoints,
resume from the newest checkpoint, and host-side fault injection.

The reference has none of this (24 h process-group timeouts, one checkpoint after the
final inference: experiments/grappa/train/t10n_train.py:137,350,373,390).  Here

* ``--heartbeat_limit S`` starts a heartbeat per rank (grappa_b200.parallel.watchdog);
  every epoch begins with a check, and a peer silent for S seconds ends the rank with a
  ``fault_|...`` line and exit code 3 before its next collective;
* ``--checkpoint_every K`` saves rank 0's model and optimizer every K epochs (the
  reference's dict and file names), and ``--resume_path latest`` starts from the newest
  ``epoch_NNN.pt`` under ``--checkpoint_path`` (from scratch when there is none), so a
  job run under ``torchrun --max-restarts N`` continues where it stopped;
* ``--inject_fault RANK:EPOCH:KIND`` makes rank RANK leave at the start of epoch EPOCH,
  between steps with nothing in flight: ``exit`` ends the process (code 17), ``hang``
  stops its heartbeat and sleeps.  Only the first attempt of a job injects (torchrun's
  TORCHELASTIC_RESTART_COUNT is 0 or unset), so the restarted job runs through.  The
  injection is host-side only; nothing here touches a GPU.
"""
import glob
import os
import re
import sys
import time

import torch.distributed as dist

FAULT_EXIT_CODE = 3


def init_process_group(backend, timeout):
    """``dist.init_process_group`` that keeps restarted attempts apart: from torchrun's
    second attempt on (TORCHELASTIC_RESTART_COUNT > 0) the group's keys live under
    ``/attempt_N/`` of the job's store.  Without that, a restarted rank can read the
    address a rank of the failed attempt published and fail to connect (seen with gloo:
    "connectFullMesh failed ... Connection refused").  The heartbeat keys, kept in the
    same store, are per attempt too."""
    import datetime

    rc = os.environ.get("TORCHELASTIC_RESTART_COUNT", "0") or "0"
    if not isinstance(timeout, datetime.timedelta):
        timeout = datetime.timedelta(seconds=float(timeout))
    if rc == "0" or "MASTER_ADDR" not in os.environ:
        dist.init_process_group(backend=backend, timeout=timeout)
        return
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    agent_store = os.environ.get("TORCHELASTIC_USE_AGENT_STORE", "").lower() == "true"
    store = dist.TCPStore(os.environ["MASTER_ADDR"], int(os.environ["MASTER_PORT"]), world_size=world,
                          is_master=(rank == 0 and not agent_store), timeout=timeout, wait_for_workers=False)
    dist.init_process_group(backend=backend, store=dist.PrefixStore(f"/attempt_{rc}", store), rank=rank,
                            world_size=world, timeout=timeout)


def start_watchdog(args):
    """A Heartbeat over the default process group's store, or None."""
    limit = float(getattr(args, "heartbeat_limit", 0.0) or 0.0)
    if limit <= 0 or not dist.is_initialized() or dist.get_world_size() < 2:
        return None
    from grappa_b200.parallel.watchdog import Heartbeat, default_store

    return Heartbeat(default_store(), dist.get_rank(), dist.get_world_size(), interval_s=min(0.5, limit / 4),
                     limit_s=limit)


def latest_checkpoint(path):
    """The newest epoch_NNN.pt under ``path``, or None."""
    if not path or not os.path.isdir(path):
        return None
    found = []
    for f in glob.glob(os.path.join(path, "epoch_*.pt")):
        m = re.search(r"epoch_(\d+)\.pt$", f)
        if m:
            found.append((int(m.group(1)), f))
    return max(found)[1] if found else None


def resolve_resume(args):
    """``--resume_path latest`` (or a directory) becomes the newest checkpoint file or
    None; an explicit file is kept."""
    rp = getattr(args, "resume_path", None)
    if rp is None or rp.strip() == "":
        return None
    if rp == "latest":
        return latest_checkpoint(getattr(args, "checkpoint_path", None))
    if os.path.isdir(rp):
        return latest_checkpoint(rp)
    return rp


def parse_fault(spec):
    if not spec:
        return None
    rank, epoch, kind = spec.split(":")
    if kind not in ("exit", "hang"):
        raise ValueError(f"--inject_fault kind must be exit or hang, not {kind}")
    return int(rank), int(epoch), kind


def maybe_inject_fault(args, rank, epoch, watchdog, hang_s=600.0):
    """Leave the job here if ``--inject_fault`` names this rank and epoch (first attempt only)."""
    f = parse_fault(getattr(args, "inject_fault", None))
    if f is None or f[0] != rank or f[1] != epoch:
        return
    if os.environ.get("TORCHELASTIC_RESTART_COUNT", "0") not in ("", "0"):
        return
    print(f"rank{rank} inject_|rank|{rank:04d}|epoch|{epoch:04d}|kind|{f[2]}", flush=True)
    if f[2] == "exit":
        os._exit(17)
    if watchdog is not None:
        watchdog.stop()
    time.sleep(hang_s)
    os._exit(17)


def fault_exit(err, rank, epoch):
    """Report a detected peer failure and end this rank without touching the process
    group (its peers are gone, so a collective or its teardown could wait)."""
    print(f"rank{rank} fault_|rank|{rank:04d}|epoch|{epoch:04d}|reason|{err}", flush=True)
    sys.stdout.flush()
    sys.stderr.flush()
    os._exit(FAULT_EXIT_CODE)


def periodic_checkpoint(args, epoch, rank, model, optimizer_state_fn, loss):
    """Save every ``--checkpoint_every`` epochs (rank 0), the reference's dict and file
    name; ``optimizer_state_fn`` is called only when a file is written."""
    from grappa_b200.train.t10n_train import save_to_ckpt

    if not getattr(args, "checkpoint_path", None) or getattr(args, "checkpoint_every", -1) <= 0:
        return None
    if (epoch + 1) % args.checkpoint_every != 0 or rank != 0:
        return None
    return save_to_ckpt(args, epoch, rank, model, optimizer_state_fn(), loss)
