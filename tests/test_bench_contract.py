"""bench.py's command-line contract that needs no GPU: the reference arm prints one
JSON line with its reason and exits 0, and every workload names its metric."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_reports_unavailable():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference"], cwd=ROOT,
                         capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference" and rec["unavailable"]
    # the reason quotes the exception that the import attempt observed
    assert "Error" in rec["unavailable"] and "t10n" in rec["unavailable"]


def test_every_workload_has_a_metric():
    sys.path.insert(0, ROOT)
    import bench

    assert set(bench.METRICS) == set(bench.WORKLOADS)
    assert bench.METRICS["sage"].startswith("s/epoch")


def test_one_shot_crossover():
    from grappa_b200.parallel.allreduce import FusedAllReduceAdam

    lim = FusedAllReduceAdam.one_shot_max_bytes
    assert lim(2) >= lim(4) >= lim(8) > 0
