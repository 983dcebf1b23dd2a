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
