"""Device placement (reference: t10n/device_allocator.py:4-138).

``DeviceAllocCPUServing``: topology and features on the host, communication device
the GPU for NCCL (the reference's CPU-serving mode, used by the CPU path here).
``DeviceAllocGPUServing``: everything on the GPU (the product path).
``T10nDeviceAllocator``: local GPU of a rank and its NUMA node (read-only queries).
"""
import os

import torch

from grappa_b200.util import shell_or


class DeviceAllocCPUServing:
    def __init__(self, device, backend):
        self.device = torch.device(device)
        self.backend = backend

    def part_topo_dev(self):
        return torch.device("cpu")

    def part_feat_dev(self):
        return torch.device("cpu")

    def comm_dev(self):
        return self.device if self.backend == "nccl" else torch.device("cpu")


class DeviceAllocGPUServing:
    def __init__(self, device, backend="nccl"):
        self.device = torch.device(device)
        self.backend = backend

    def part_topo_dev(self):
        return self.device

    def part_feat_dev(self):
        return self.device

    def comm_dev(self):
        return self.device if self.backend == "nccl" else torch.device("cpu")


class T10nDeviceAllocator:
    def __init__(self, num_gpus):
        self.num_gpus = num_gpus

    def get_local_gpu_id(self, world, rank):
        if self.num_gpus is None or self.num_gpus <= 0:
            return -1
        return int(os.environ.get("LOCAL_RANK", rank % self.num_gpus))

    def get_numa_affinity(self, local_gid):
        """NUMA node of the GPU from `nvidia-smi topo -C` (read-only), else from the PCI
        device's sysfs ``numa_node``; -1 if unknown."""
        if local_gid is None or local_gid < 0:
            return -1
        out = shell_or(f"nvidia-smi topo -C -i {local_gid}", "")
        for tok in out.replace(":", " ").split():
            if tok.isdigit():
                return int(tok)
        return pci_numa_node(local_gid)

    def get_local_cpu_num(self):
        """Logical CPUs of this machine."""
        return os.cpu_count() or 1

    def get_local_cpu_ids(self, world_size, rank):
        """CPUs close to this rank's GPU, among those the process may use: NVML's CPU
        affinity of the GPU (read-only), else the CPUs of its NUMA node, else every
        allowed CPU."""
        allowed = sorted(os.sched_getaffinity(0))
        gid = self.get_local_gpu_id(world_size, rank)
        ids = nvml_cpu_affinity(gid, self.get_local_cpu_num()) if gid >= 0 else []
        if not ids and gid >= 0:
            node = self.get_numa_affinity(gid)
            if node >= 0:
                from grappa_b200 import host

                ids = host().numa.node_cpus(node)
        ids = [c for c in ids if c in set(allowed)]
        return ids or allowed

    def set_omp_dev_assignments(self, world_size, rank, cg_idx=0, dup_per_gpu=1):
        """OpenMP placement for this rank (reference: t10n/device_allocator.py:120-138):
        the rank's CPUs (split into ``dup_per_gpu`` groups when several processes share
        a GPU, group ``cg_idx`` taken) as OMP_PLACES, spread binding, one thread per
        CPU.  The variables reach OpenMP runtimes started after the call (this
        process's, if it has not run a parallel region yet, and its children's).
        Returns the CPUs."""
        cpus = self.get_local_cpu_ids(world_size, rank)
        if dup_per_gpu > 1:
            stride = max(1, len(cpus) // dup_per_gpu)
            cpus = cpus[cg_idx * stride:(cg_idx + 1) * stride] or cpus[:stride]
        os.environ["OMP_PROC_BIND"] = "spread"
        os.environ["OMP_PLACES"] = ",".join(f"{{{c}}}" for c in cpus)
        os.environ["OMP_NUM_THREADS"] = str(len(cpus))
        return cpus


def nvml_cpu_affinity(local_gid, n_cpus):
    """CPU ids in NVML's affinity mask of GPU ``local_gid`` (read-only query); [] when
    NVML is unavailable."""
    try:
        import pynvml

        pynvml.nvmlInit()
    except Exception:
        return []
    try:
        h = pynvml.nvmlDeviceGetHandleByIndex(local_gid)
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (n_cpus + 63) // 64)
        out = []
        for w, word in enumerate(words):
            for b in range(64):
                if (int(word) >> b) & 1 and w * 64 + b < n_cpus:
                    out.append(w * 64 + b)
        return out
    except Exception:
        return []
    finally:
        try:
            pynvml.nvmlShutdown()
        except Exception:
            pass


def pci_numa_node(local_gid, sysfs="/sys/bus/pci/devices"):
    """NUMA node of CUDA device ``local_gid`` from its PCI address's sysfs entry; -1 when
    unknown (no CUDA, no such device, or a firmware that gives none)."""
    try:
        if not torch.cuda.is_available() or local_gid >= torch.cuda.device_count():
            return -1
        p = torch.cuda.get_device_properties(local_gid)
        addr = f"{getattr(p, 'pci_domain_id', 0):04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(f"{sysfs}/{addr}/numa_node") as f:
            node = int(f.read().strip())
        return node if node >= 0 else -1
    except (AttributeError, OSError, ValueError, RuntimeError):
        return -1
