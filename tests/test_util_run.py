"""Process fan-out helpers of grappa_b200.util (the reference's t10n/util.py:50-109):
local processes, ssh fan-out through a stand-in ``ssh`` that runs the command locally,
the hosts-file parser, and the time limit that ends the groups it started."""
import os
import stat
import time

from grappa_b200 import util


def test_mp_run_logs_each_process(tmp_path):
    log = tmp_path / "log"
    codes = util.mp_run(3, "mp", lambda i: f"echo rank {i}; exit {i % 2}", work_dir=str(tmp_path),
                        log_dir=str(log))
    assert codes == [0, 1, 0]
    for i in range(3):
        assert (log / f"mp_{i}.txt").read_text().strip() == f"rank {i}"


def test_mp_run_time_limit_ends_its_groups(tmp_path):
    log = tmp_path / "log"
    marker = tmp_path / "child_done"
    t0 = time.monotonic()
    # the child of the shell sleeps too: ending the whole group must end it as well
    codes = util.mp_run(2, "slow", lambda i: f"(sleep 30; touch {marker}) & sleep 30", log_dir=str(log),
                        timeout=1.0)
    assert codes == [-1, -1]
    assert time.monotonic() - t0 < 25
    time.sleep(0.5)
    assert not marker.exists()


def test_parse_hosts_file(tmp_path):
    f = tmp_path / "hosts"
    f.write_text("volta09 n_gpu=2\n\n# spare\nvolta10\nh100a n_gpu=8 extra\n")
    assert util.parse_hosts_file(str(f)) == (["volta09", "volta10", "h100a"], [2, -1, 8])


def test_cluster_run_through_ssh(tmp_path, monkeypatch):
    hosts = tmp_path / "hosts"
    hosts.write_text("nodeA n_gpu=8\nnodeB n_gpu=8\n")
    bindir = tmp_path / "bin"
    bindir.mkdir()
    fake = bindir / "ssh"
    # stand-in for ssh: skip the -o options, record the host, run the command here
    fake.write_text("#!/bin/bash\nwhile [ \"$1\" = -o ]; do shift 2; done\nhost=$1; shift\n"
                    "echo \"host=$host\"; exec bash -c \"$1\"\n")
    fake.chmod(fake.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{bindir}:{os.environ['PATH']}")
    argvs = util.cluster_run(str(hosts), "cl", lambda hs, i: f"echo {hs[i]} is {i} of {len(hs)}", dry_run=True)
    assert argvs[0][0] == "ssh" and "nodeA" in argvs[0] and "ServerAliveInterval=60" in argvs[0]
    log = tmp_path / "log"
    codes = util.cluster_run(str(hosts), "cl", lambda hs, i: f"echo {hs[i]} is {i} of {len(hs)}\n",
                             work_dir=str(tmp_path), log_dir=str(log))
    assert codes == [0, 0]
    assert (log / "cl_0.txt").read_text().split("\n")[:2] == ["host=nodeA", "nodeA is 0 of 2"]
    assert (log / "cl_1.txt").read_text().split("\n")[:2] == ["host=nodeB", "nodeB is 1 of 2"]


def test_is_in_slurm(monkeypatch):
    for k in ("SLURM_JOB_ID", "SLURM_NODELIST", "SLURM_JOB_NODELIST"):
        monkeypatch.delenv(k, raising=False)
    assert not util.is_in_slurm()
    monkeypatch.setenv("SLURM_JOB_ID", "42")
    assert util.is_in_slurm()
    assert util.green_str("ok").startswith("\033[0;32m")
