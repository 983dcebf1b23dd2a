"""Cluster deployment helpers (CPU): hosts files, the SLURM job-array script of a sweep,
the container commands and the per-host inline command (through a stand-in ssh that
runs it locally); nothing is submitted."""
import os

import pytest

from grappa_b200 import cluster, launch


def test_parse_hosts_file(tmp_path):
    p = tmp_path / "hosts"
    p.write_text("# machines\nnode01 n_gpu=8\n\nnode02 n_gpu=4\nnode03\n")
    assert cluster.parse_hosts_file(str(p)) == [("node01", 8), ("node02", 4), ("node03", -1)]


def test_slurm_job_array_runs_the_sweep(tmp_path):
    out, logs = tmp_path / "jobs", tmp_path / "log"
    cluster.main(["slurm", "--out", str(out), "--log_dir", str(logs), "--graphs", "rmat16k,reddit",
                  "--models", "sage,gat", "--nproc", "8", "--partition", "gpu", "--job_name", "sw"])
    script = (out / "sw.sbatch").read_text()
    sweep = (out / "sweep.txt").read_text().splitlines()
    assert len(sweep) == 4  # 2 graphs x 2 models
    for line in ("#SBATCH --nodes=1", "#SBATCH --exclusive", "#SBATCH --gres=gpu:8", "#SBATCH --array=0-3",
                 "#SBATCH --partition=gpu", "MASTER_ADDR=127.0.0.1"):
        assert line in script
    assert str(out / "sweep.txt") in script and "SLURM_ARRAY_TASK_ID + 1" in script
    # each line is a launch.py sweep command with its log redirection, one rank per GPU
    assert all("--nproc-per-node 8" in c and "--num_gpus 8" in c and str(logs) in c for c in sweep)
    assert os.access(out / "sw.sbatch", os.X_OK)


def test_slurm_rejects_multi_node():
    with pytest.raises(ValueError, match="one node"):
        cluster.slurm_script(3, "sweep.txt", job_name="x", gpus=8, cpus=8, mem="0", time_limit="1:00:00",
                             log_dir="log", nodes=2)


def test_docker_command_shares_ipc_and_all_gpus(capsys):
    argv = cluster.docker_command("img:1", "python -m x", data_path="/data", workspace="/ws", name="n1")
    assert argv[:3] == ["docker", "run", "--rm"]
    assert "--gpus=all" in argv and "--ipc=host" in argv
    assert argv[-4:] == ["img:1", "bash", "-lc", "python -m x"]
    assert cluster.main(["docker", "--image", "img:1", "--data_path", "/data", "--models", "sage,gcn"]) == 0
    lines = capsys.readouterr().out.strip().splitlines()
    assert len(lines) == 2 and all(line.startswith("docker run") for line in lines)


def test_inline_command_on_every_host(tmp_path, monkeypatch, capsys):
    import stat

    hosts = tmp_path / "hosts"
    hosts.write_text("h1 n_gpu=8\nh2 n_gpu=8\n")
    assert cluster.main(["inline", "--host_file", str(hosts), "--dry_run", "--", "nvidia-smi", "-L"]) == 0
    lines = capsys.readouterr().out.strip().splitlines()
    assert len(lines) == 2 and lines[0].startswith("ssh ") and " h1 " in lines[0] and "nvidia-smi -L" in lines[0]
    bindir = tmp_path / "bin"
    bindir.mkdir()
    fake = bindir / "ssh"  # runs the command here, as if on the host
    fake.write_text("#!/bin/bash\nwhile [ \"$1\" = -o ]; do shift 2; done\nshift\nexec bash -c \"$1\"\n")
    fake.chmod(fake.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{bindir}:{os.environ['PATH']}")
    log = tmp_path / "log"
    assert cluster.main(["inline", "--host_file", str(hosts), "--tag_id", "t", "--log_dir", str(log), "--",
                         "echo hello"]) == 0
    assert (log / "t_0.txt").read_text().strip() == "hello" and (log / "t_1.txt").read_text().strip() == "hello"
    assert cluster.main(["inline", "--host_file", str(hosts), "--log_dir", str(log), "--", "exit 3"]) == 1


def test_slurm_partition_job_runs_first(tmp_path):
    data = tmp_path / "data"
    out = tmp_path / "jobs"
    import argparse

    path = cluster.write_slurm_job(argparse.Namespace(
        out=str(out), job_name="sw", partition="gpu", nodes=1, cpus=16, mem="0", time="1:00:00",
        log_dir=str(tmp_path / "log"), partition_step=True, script="t10n_train", data_path=str(data),
        parts="hash,metis", graphs="tiny", models="sage", layers_fanouts="2:10,5", runs=1, nproc=2, num_gpus=2,
        hidden=16, epochs=2, bs=256, eval_bs=1000, eval_every=1, repart=1, log_every=20, tag_prefix="t",
        port=29600))
    assert path.endswith("submit.sh") and os.access(path, os.X_OK)
    submit = open(path).read()
    assert "jid=$(sbatch --parsable" in submit and "--dependency=afterok:$jid" in submit
    part = open(out / "partition.sbatch").read()
    assert part.count("grappa_b200.dataset.partition generate") == 1  # one graph
    assert part.count("grappa_b200.dataset.partition seq") == 2 and "--part_method metis" in part
    assert "#SBATCH --partition=gpu" in part and "#SBATCH --gres" not in part
    assert len(open(out / "sweep.txt").read().strip().splitlines()) == 2


def test_docker_partition_steps_come_first(tmp_path, capsys):
    rc = cluster.main(["docker", "--image", "img:1", "--data_path", str(tmp_path / "d"), "--graphs", "tiny",
                       "--nproc", "2", "--partition_step"])
    assert rc == 0
    lines = capsys.readouterr().out.strip().splitlines()
    assert "dataset.partition generate" in lines[0] and "dataset.partition seq" in lines[1]
    assert "grappa_b200.train.t10n_train" in lines[2] and all(l.startswith("docker run") for l in lines)
