"""Small utilities of the runtime (reference: t10n/util.py:11-194).

* ``timing``         decorator printing a function's wall time
* ``pprint``         print from one rank only
* ``shell_or``       run a shell command, return its output or a default
* ``DeviceTimer``    CUDA-event phase timer (device time, max over ranks on request)
* ``PyNVML``         read-only GPU memory / clock report through NVML
* ``set_py_affinity`` pin the process to the CPUs of a NUMA node (opt-in)
* ``mp_run`` / ``cluster_run`` run one shell command per local process / per host (ssh),
  each logged to ``{log_dir}/{tag}_{idx}.txt``; ``parse_hosts_file``, ``is_in_slurm``,
  ``green_str`` / ``printg``
"""
import functools
import os
import shlex
import signal
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


def green_str(s):
    return f"\033[0;32m{s}\033[0m"


def printg(s):
    print(green_str(s), flush=True)


def is_in_slurm():
    """True inside a SLURM allocation."""
    return any(k in os.environ for k in ("SLURM_JOB_ID", "SLURM_NODELIST", "SLURM_JOB_NODELIST"))


def parse_hosts_file(hosts_file):
    """(hosts, n_gpu) from a hosts file of ``host [n_gpu=K]`` lines (reference format,
    t10n/util.py:50-59); n_gpu is -1 where a line gives none.  Blank lines and lines
    starting with '#' are skipped."""
    hosts, n_gpu = [], []
    with open(hosts_file) as f:
        for line in f:
            fields = line.split()
            if not fields or fields[0].startswith("#"):
                continue
            k = -1
            for tok in fields[1:]:
                if tok.startswith("n_gpu="):
                    k = int(tok.split("=", 1)[1])
            hosts.append(fields[0])
            n_gpu.append(k)
    return hosts, n_gpu


def _run_group(tag_id, argvs, log_dir, timeout):
    """Start every argv in its own session (process group), output to
    {log_dir}/{tag_id}_{idx}.txt; wait for all.  On timeout the groups still running are
    ended (SIGTERM, then SIGKILL after 10 s) by their own ids.  Returns the exit codes
    (-1 for a group ended by the timeout)."""
    os.makedirs(log_dir, exist_ok=True)
    procs, logs = [], []
    try:
        for idx, argv in enumerate(argvs):
            log = open(os.path.join(log_dir, f"{tag_id}_{idx}.txt"), "w")
            logs.append(log)
            procs.append(subprocess.Popen(argv, stdout=log, stderr=subprocess.STDOUT, start_new_session=True))
        deadline = None if timeout is None else time.monotonic() + timeout
        codes = []
        for p in procs:
            try:
                left = None if deadline is None else max(0.0, deadline - time.monotonic())
                codes.append(p.wait(timeout=left))
            except subprocess.TimeoutExpired:
                codes.append(None)
        for i, p in enumerate(procs):
            if codes[i] is None:
                _end_group(p)
                codes[i] = -1
        return codes
    finally:
        for p in procs:
            if p.poll() is None:
                _end_group(p)
        for log in logs:
            log.close()


def _end_group(p):
    for sig, wait in ((signal.SIGTERM, 10), (signal.SIGKILL, 10)):
        try:
            os.killpg(p.pid, sig)  # the group this function started, by its id
        except ProcessLookupError:
            return
        try:
            p.wait(timeout=wait)
            return
        except subprocess.TimeoutExpired:
            continue


def mp_run(num_process, tag_id, cmd_func, work_dir=".", log_dir="log", timeout=None):
    """Run ``cmd_func(idx)`` (a shell command) for idx in [0, num_process) as concurrent
    local processes in ``work_dir`` (reference: t10n/util.py:91-109).  Returns the exit
    codes."""
    printg(f"{tag_id} starting {num_process} processes")
    argvs = [["bash", "-c", f"cd {shlex.quote(work_dir)} && {cmd_func(i)}"] for i in range(num_process)]
    codes = _run_group(tag_id, argvs, log_dir, timeout)
    printg(f"{tag_id} end: {codes}")
    return codes


def cluster_ssh_argv(host, cmd, work_dir=".", keepalive=True):
    """ssh argv that runs ``cmd`` in ``work_dir`` on ``host``."""
    opts = ["-o", "StrictHostKeyChecking=no", "-o", "BatchMode=yes"]
    if keepalive:
        opts += ["-o", "ServerAliveInterval=60", "-o", "ServerAliveCountMax=3"]
    return ["ssh"] + opts + [host, f"cd {shlex.quote(work_dir)} && {cmd}"]


def cluster_run(host_file, tag_id, cmd_func, work_dir=".", timeout=True, log_dir="log", time_limit=None,
                dry_run=False):
    """Run ``cmd_func(hosts, idx)`` on every host of ``host_file`` over ssh, concurrently
    (reference: t10n/util.py:62-88; ``timeout`` keeps the reference's meaning, ssh
    keep-alives that end a command whose host stops answering).  Each host's output goes
    to {log_dir}/{tag_id}_{idx}.txt.  Returns the exit codes, or with ``dry_run`` the ssh
    argvs without running them."""
    hosts, _ = parse_hosts_file(host_file)
    argvs = [cluster_ssh_argv(h, cmd_func(hosts, i).replace("\n", " "), work_dir, timeout)
             for i, h in enumerate(hosts)]
    if dry_run:
        return argvs
    printg(f"{tag_id} starting on {len(hosts)} hosts")
    codes = _run_group(tag_id, argvs, log_dir, time_limit)
    printg(f"{tag_id} end: {codes}")
    return codes
