"""Elastic recovery on CPU ranks: a rank leaves mid-job (host-side injection, no GPU),
the job stops with a clear status, and torchrun's restart resumes from the newest
periodic checkpoint and finishes.

* ``hang``: the rank stops its heartbeat and sleeps; the other rank's next collective
  times out, its watchdog names the silent rank (``fault_`` line, exit code 3), and the
  agent restarts the group;
* ``exit``: the rank's process ends; the agent sees the failure and restarts the group.
"""
import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def chunks(tmp_path_factory):
    from grappa_b200.dataset import partition

    d = tmp_path_factory.mktemp("el")
    assert partition.main(["generate", "--graph_name", "tiny", "--out", str(d / "t10n" / "tiny")]) == 0
    assert partition.main(["seq", "--src_path", str(d / "t10n" / "tiny"), "--dest_path", str(d), "--graph_name",
                           "tiny", "--n_part", "2"]) == 0
    return d


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("kind", ["hang", "exit"])
def test_restart_resumes_from_the_newest_checkpoint(chunks, tmp_path, kind):
    ck = tmp_path / "ck"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--max-restarts", "1",
           "--monitor-interval", "0.5", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           "-m", "grappa_b200.train.t10n_train", "--data_path", str(chunks), "--graph_name", "tiny",
           "--part_method", "hash", "--n_part", "2", "--model", "sage", "--num_hidden", "16", "--num_layers", "2",
           "--fan_out", "5,5", "--num_epochs", "5", "--batch_size", "256", "--batch_size_eval", "1000",
           "--eval_every", "5", "--repart_every", "2", "--num_gpus", "-1", "--backend", "gloo", "--tag_id", "el",
           "--close_dd", "--checkpoint_path", str(ck), "--checkpoint_every", "1", "--resume_path", "latest",
           "--heartbeat_limit", "2", "--pg_timeout", "8", "--inject_fault", f"1:2:{kind}",
           "--metrics_jsonl", str(tmp_path / "m_{rank}.jsonl")]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert "inject_|rank|0001|epoch|0002" in out
    if kind == "hang":
        assert "fault_|rank|0000|epoch|0002" in out and "rank(s) [1]" in out
    assert "resumed from epoch 1" in out
    assert sorted(os.listdir(ck))[-1] == "epoch_004.pt"
    recs = [json.loads(l) for l in open(tmp_path / "m_0.jsonl")]
    epochs = [x["epoch"] for x in recs if x["event"] == "epoch"]
    # epochs 0 and 1 before the fault (2 may have started on rank 0 only), 2-4 after the restart
    assert epochs[:2] == [0, 1] and epochs[-3:] == [2, 3, 4]
    assert any(x["event"] == "infer" for x in recs)
