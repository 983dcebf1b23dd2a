"""NUMA placement and bandwidth probes of the host engine (grappa_b200._C.numa): node and
CPU lists, the preferred-node policy scope, the NUMA-placed host graph, the bandwidth
matrix and its command line, the host-path benchmark's lines; one GPU test of the pinned
copy probe."""
import json

import numpy as np
import pytest
import torch

from grappa_b200 import host
from grappa_b200.device_allocator import T10nDeviceAllocator, pci_numa_node
from grappa_b200.utils import numa_bench

N = host().numa


def test_nodes_and_cpus():
    nodes = N.nodes()
    assert nodes and all(n >= 0 for n in nodes)
    assert N.node_cpus(nodes[0])
    assert N.node_cpus(-1) == []
    assert N.parse_cpulist("0-3,8,10-11") == [0, 1, 2, 3, 8, 10, 11]
    assert N.parse_cpulist("") == []


def test_policy_scope_places_pages_and_ends():
    node = N.nodes()[0]
    with N.MemPolicy(node) as active:
        a = np.ones(1 << 22)  # 32 MB faulted in under the policy
    assert isinstance(active, bool)
    assert N.node_of(a) in (-1, node)
    with N.MemPolicy(100000) as active:  # not a node: nothing changes
        assert active is False
    b = np.ones(1 << 20)
    assert N.node_of(b) in (-1, *N.nodes())


def test_numa_placed_host_graph_is_the_same_graph():
    rng = np.random.default_rng(0)
    u = rng.integers(0, 3000, 40000)
    v = rng.integers(0, 3000, 40000)
    G = host().graph
    plain = G.HostGraph(u, v, 3000)
    placed = G.HostGraph(u, v, 3000, N.nodes()[0])
    assert not plain.numa_placed
    assert np.array_equal(plain.indptr(), placed.indptr()) and np.array_equal(plain.indices(), placed.indices())
    assert placed.numa_node_of_indices() in (-1, *N.nodes())


def test_bandwidth_matrix_and_cli(capsys):
    node = N.nodes()[0]
    r = N.bandwidth(node, node, 16, 2, 1)
    assert r["write_gbs"] > 0.1 and r["read_gbs"] > 0.1 and r["mem_node_seen"] in (-1, node)
    with pytest.raises(ValueError):
        N.bandwidth(node, 100000, 16, 2, 1)
    with pytest.raises(ValueError):
        N.bandwidth(-1, node, 16, 2, 1)
    assert numa_bench.main(["--no_gpu", "--mbytes", "16", "--reps", "1", "--threads", "2", "--json"]) == 0
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert len(out["host"]) >= 1 and out["gpu"] == []


def test_gpu_numa_node_unknown_without_gpu():
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    assert pci_numa_node(0) == -1
    assert T10nDeviceAllocator(-1).get_numa_affinity(-1) == -1


def test_pci_numa_node_reads_sysfs(tmp_path, monkeypatch):
    class Props:
        pci_domain_id, pci_bus_id, pci_device_id = 0, 0x1B, 0

    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "device_count", lambda: 1)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda i: Props())
    d = tmp_path / "0000:1b:00.0"
    d.mkdir()
    (d / "numa_node").write_text("1\n")
    assert pci_numa_node(0, sysfs=str(tmp_path)) == 1
    (d / "numa_node").write_text("-1\n")
    assert pci_numa_node(0, sysfs=str(tmp_path)) == -1
    assert pci_numa_node(3, sysfs=str(tmp_path)) == -1


@pytest.mark.gpu
def test_pinned_copy_probe():
    buf, seen = numa_bench.pinned_on(N.nodes()[0], 32 << 20)
    assert buf.is_pinned() and seen in (-1, *N.nodes())
    r = numa_bench.copy_bandwidth(torch.device("cuda", 0), buf, reps=2)
    assert r["h2d_gbs"] > 1.0 and r["d2h_gbs"] > 1.0


def test_host_bench_lines(capsys):
    from grappa_b200.utils import bench_host

    assert bench_host.main(["--graph", "tiny", "--parts", "2", "--only", "csc,sample,metis"]) == 0
    recs = [json.loads(l) for l in capsys.readouterr().out.strip().splitlines()]
    assert [r["bench"] for r in recs] == ["HostGraph", "sample_batch", "multilevel_partition"]
    assert recs[0]["median_s"] > 0 and recs[1]["mean_ms"] > 0
    assert 0 < recs[2]["edge_cut"] < recs[2]["undirected_edges"] and recs[2]["node_imbalance"] <= 1.05
