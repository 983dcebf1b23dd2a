"""Small utilities of the runtime (reference: t10n/util.py:11-194).

* ``timing``         decorator printing a function's wall time
* ``pprint``         print from one rank only
* ``shell_or``       run a shell command, return its output or a default
* ``DeviceTimer``    CUDA-event phase timer (device time, max over ranks on request)
* ``PyNVML``         read-only GPU memory / clock report through NVML
* ``set_py_affinity`` pin the process to the CPUs of a NUMA node (opt-in)
"""
import functools
import os
import subprocess
import time

import torch


def timing(f):
    @functools.wraps(f)
    def wrap(*args, **kwargs):
        t0 = time.time()
        r = f(*args, **kwargs)
        print(f"func:{f.__name__} took: {time.time() - t0:.4f} sec", flush=True)
        return r

    return wrap


def pprint(rank, *args, **kwargs):
    """Print only on rank 0 (or on the given rank when `rank` is 0)."""
    if rank == 0:
        print(*args, **kwargs, flush=True)


def shell_or(cmd, default=""):
    try:
        return subprocess.check_output(cmd, shell=True, text=True, stderr=subprocess.DEVNULL).strip()
    except (subprocess.CalledProcessError, OSError):
        return default


class DeviceTimer:
    """Accumulates device time of named phases with CUDA events (no host sync per phase)."""

    def __init__(self, device=None):
        self.device = device
        self.events = {}
        self.totals = {}

    def start(self, name):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.events[name] = ev

    def stop(self, name):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.events[name] = (self.events[name], ev)

    def collect(self):
        torch.cuda.synchronize()
        for name, pair in list(self.events.items()):
            if isinstance(pair, tuple):
                self.totals[name] = self.totals.get(name, 0.0) + pair[0].elapsed_time(pair[1]) / 1000.0
                del self.events[name]
        return dict(self.totals)

    def max_over_ranks(self):
        import torch.distributed as dist

        out = self.collect()
        if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
            return out
        names = sorted(out)
        t = torch.tensor([out[n] for n in names], dtype=torch.float64,
                         device="cuda" if dist.get_backend() == "nccl" else "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return dict(zip(names, t.cpu().tolist()))


class PyNVML:
    """Read-only NVML queries (memory in use, clocks).  Never changes GPU settings."""

    def __init__(self):
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.ok = True
        except Exception:
            self.nv = None

    def report_memory(self, rank, tag=""):
        if not self.ok:
            return None
        idx = torch.cuda.current_device() if torch.cuda.is_available() else 0
        h = self.nv.nvmlDeviceGetHandleByIndex(idx)
        info = self.nv.nvmlDeviceGetMemoryInfo(h)
        line = f"rank{rank:02d} {tag} gpu{idx} used {info.used / 2**30:.2f} GiB of {info.total / 2**30:.2f} GiB"
        pprint(0 if rank == 0 else 1, line)
        return info.used

    def clocks(self, index=0):
        if not self.ok:
            return None
        h = self.nv.nvmlDeviceGetHandleByIndex(index)
        return {"sm_mhz": self.nv.nvmlDeviceGetClockInfo(h, self.nv.NVML_CLOCK_SM),
                "sm_max_mhz": self.nv.nvmlDeviceGetMaxClockInfo(h, self.nv.NVML_CLOCK_SM)}


pyml_handle = PyNVML()


def set_py_affinity(node_id, enable=None):
    """Pin this process to the CPUs of NUMA node ``node_id``.  Off unless enabled
    (the reference returns early from its version, t10n/util.py:172-194)."""
    if enable is None:
        enable = os.environ.get("GRAPPA_SET_AFFINITY", "0") == "1"
    if not enable or node_id is None or node_id < 0:
        return False
    path = f"/sys/devices/system/node/node{node_id}/cpulist"
    try:
        with open(path) as f:
            spec = f.read().strip()
    except OSError:
        return False
    cpus = set()
    for part in spec.split(","):
        if "-" in part:
            a, b = part.split("-")
            cpus.update(range(int(a), int(b) + 1))
        elif part:
            cpus.add(int(part))
    os.sched_setaffinity(0, cpus)
    return True


def backtrace():
    import traceback

    traceback.print_stack()
