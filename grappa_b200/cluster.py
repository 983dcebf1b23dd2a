"""Cluster deployment of the training sweeps: SLURM batch scripts and container launches
(reference: experiments/grappa/slurm_per_node_h100.sh and slurm_per_node_a100*.sh for
SLURM, experiments/grappa/create_swarm_cluster.py for the Docker swarm, t10n/util.py:50-59
for the hosts-file format).

A training job here is one node: the ranks of a job map each other's device memory
(gradient buckets, partitions and feature tables through CUDA IPC), which needs every
rank's GPU on the same host and in the same IPC namespace.  So

  * ``slurm`` writes one batch script that runs the sweep of ``grappa_b200.launch`` as a
    SLURM job array, one exclusive node per array task (the reference runs one job of
    several nodes with ``srun torch.distributed.run`` across them);
  * ``docker`` runs (or prints) the sweep's commands in one container per host that
    holds all the host's GPUs with the host's IPC namespace (the reference builds a swarm
    of one container per GPU over many hosts; per-GPU containers would hide the peers'
    devices from each rank).

Nothing here runs unless asked: ``slurm`` writes files, ``docker`` prints its commands
unless given ``--execute``.

    python -m grappa_b200.cluster slurm --out jobs --data_path /data --graphs rmat16k \\
        --models sage,gcn --nproc 8 --partition gpu
    python -m grappa_b200.cluster docker --image grappa_b200:latest --data_path /data \\
        --graphs rmat16k --nproc 8 [--execute]
    python -m grappa_b200.cluster hosts hosts.txt     # parse a hosts file ("host n_gpu=K")
    python -m grappa_b200.cluster inline --host_file hosts.txt --tag_id probe -- nvidia-smi -L

``inline`` runs one shell command on every host of a hosts file over ssh (the
reference's ``t10nrun.py --task inline`` / ``--task test``), each host's output in
``{log_dir}/{tag_id}_{idx}.txt``; ``--time_limit`` ends the ssh sessions it started
when they run over (the reference's ``--task kill`` matches processes by name on every
host instead).
"""
import argparse
import os
import shlex
import subprocess
import sys

from grappa_b200 import launch, util


def parse_hosts_file(path):
    """[(host, n_gpu)] from a hosts file with one ``host [n_gpu=K]`` line per machine (the
    reference's format; n_gpu is -1 when the line gives none).  Blank lines and lines
    starting with '#' are skipped."""
    hosts, n_gpu = util.parse_hosts_file(path)
    return list(zip(hosts, n_gpu))


def sweep_commands(args):
    """The sweep of ``grappa_b200.launch`` as [(tag, command)] for the given arguments."""
    return list(launch.sweep(args))


def slurm_script(n_tasks, sweep_file, *, job_name, gpus, cpus, mem, time_limit, log_dir, partition=None,
                 nodes=1):
    """A SLURM batch script that runs line SLURM_ARRAY_TASK_ID + 1 of ``sweep_file`` (one
    command per line) on one exclusive node with ``gpus`` GPUs."""
    if nodes != 1:
        raise ValueError("a job is one node: its ranks share device memory through CUDA IPC, which does not "
                         "reach across hosts; run the sweep's configurations as separate single-node jobs")
    if n_tasks < 1:
        raise ValueError("the sweep is empty")
    lines = ["#!/bin/bash",
             f"#SBATCH --job-name={job_name}",
             "#SBATCH --nodes=1",
             "#SBATCH --ntasks-per-node=1",
             "#SBATCH --exclusive",
             f"#SBATCH --gres=gpu:{gpus}",
             f"#SBATCH --cpus-per-task={cpus}",
             f"#SBATCH --mem={mem}",
             f"#SBATCH --time={time_limit}",
             f"#SBATCH --array=0-{n_tasks - 1}",
             f"#SBATCH --output={log_dir}/%x_%A_%a.out",
             f"#SBATCH --error={log_dir}/%x_%A_%a.err"]
    if partition:
        lines.append(f"#SBATCH --partition={partition}")
    lines += ["",
              "set -euo pipefail",
              "# the job's ranks talk over NCCL and CUDA IPC on this node only",
              "export MASTER_ADDR=127.0.0.1",
              f"CMD=$(sed -n \"$((SLURM_ARRAY_TASK_ID + 1))p\" {shlex.quote(sweep_file)})",
              "echo \"task $SLURM_ARRAY_TASK_ID on $(hostname): $CMD\"",
              "eval \"$CMD\"",
              ""]
    return "\n".join(lines)


def write_slurm_job(args):
    """Write ``{out}/sweep.txt`` (the commands) and ``{out}/{job_name}.sbatch``; with
    ``--partition`` also ``{out}/partition.sbatch`` (the missing chunk sets, built once on
    one node before the array runs) and ``{out}/submit.sh``, which submits both with the
    array waiting for the partition job.  Returns the path to submit."""
    cmds = sweep_commands(args)
    os.makedirs(args.out, exist_ok=True)
    log_dir = os.path.abspath(args.log_dir)
    sweep_file = os.path.abspath(os.path.join(args.out, "sweep.txt"))
    with open(sweep_file, "w") as f:
        for tag, cmd in cmds:
            f.write(f"{cmd} > {shlex.quote(os.path.join(log_dir, tag + '_0.txt'))} 2>&1\n")
    script = slurm_script(len(cmds), sweep_file, job_name=args.job_name, gpus=args.nproc, cpus=args.cpus,
                          mem=args.mem, time_limit=args.time, log_dir=log_dir, partition=args.partition, nodes=args.nodes)
    path = os.path.join(args.out, f"{args.job_name}.sbatch")
    with open(path, "w") as f:
        f.write(script)
    os.chmod(path, 0o755)
    if not getattr(args, "partition_step", False):
        return path
    steps = list(launch.partition_commands(args))
    lines = ["#!/bin/bash", f"#SBATCH --job-name={args.job_name}_partition", "#SBATCH --nodes=1",
             "#SBATCH --ntasks-per-node=1", f"#SBATCH --cpus-per-task={args.cpus}", f"#SBATCH --mem={args.mem}",
             f"#SBATCH --time={args.time}", f"#SBATCH --output={log_dir}/%x_%j.out",
             f"#SBATCH --error={log_dir}/%x_%j.err"]
    if args.partition:
        lines.append(f"#SBATCH --partition={args.partition}")
    lines += ["", "set -euo pipefail"]
    lines += [f"{cmd} > {shlex.quote(os.path.join(log_dir, tag + '_0.txt'))} 2>&1" for tag, cmd in steps]
    part = os.path.join(args.out, "partition.sbatch")
    with open(part, "w") as f:
        f.write("\n".join(lines + [""]))
    os.chmod(part, 0o755)
    submit = os.path.join(args.out, "submit.sh")
    with open(submit, "w") as f:
        f.write("\n".join(["#!/bin/bash", "set -euo pipefail",
                           f"mkdir -p {shlex.quote(log_dir)}",
                           f"jid=$(sbatch --parsable {shlex.quote(os.path.abspath(part))})",
                           f"sbatch --dependency=afterok:$jid {shlex.quote(os.path.abspath(path))}", ""]))
    os.chmod(submit, 0o755)
    return submit


def docker_command(image, cmd, *, data_path, workspace=None, name=None, shm="64g", gpus="all"):
    """``docker run`` argv for one training command: every GPU of the host, the host's IPC
    namespace (the ranks map each other's device memory), the dataset mounted at the
    same path so that the command's ``--data_path`` stays valid."""
    argv = ["docker", "run", "--rm", f"--gpus={gpus}", "--ipc=host", "--cap-add=SYS_NICE", f"--shm-size={shm}",
            "-v", f"{data_path}:{data_path}"]
    if workspace:
        argv += ["-v", f"{workspace}:/workspace", "-w", "/workspace"]
    if name:
        argv += ["--name", name]
    argv += [image, "bash", "-lc", cmd]
    return argv


def run_docker(args):
    """Print (or with --execute run, one after another) one container per configuration;
    with ``--partition_step`` the missing chunk sets are built first, one container per
    step."""
    failed = 0
    steps = list(launch.partition_commands(args)) if getattr(args, "partition_step", False) else []
    for tag, cmd in steps + sweep_commands(args):
        argv = docker_command(args.image, cmd, data_path=os.path.abspath(args.data_path), workspace=args.workspace,
                              name=f"{args.tag_prefix}_{tag}"[:63], shm=args.shm)
        print(" ".join(shlex.quote(a) for a in argv), flush=True)
        if args.execute:
            rc = subprocess.run(argv).returncode
            failed += rc != 0
    return failed


def _sweep_args(ap):
    # the sweep options of grappa_b200.launch, same names and defaults
    ap.add_argument("--script", default="t10n_train", choices=["t10n_train", "t10n_fullgraph_train"])
    ap.add_argument("--data_path", default="data")
    ap.add_argument("--parts", default="hash")
    ap.add_argument("--graphs", default="rmat16k")
    ap.add_argument("--models", default="sage")
    ap.add_argument("--layers_fanouts", default="3:15,10,5")
    ap.add_argument("--runs", type=int, default=1)
    ap.add_argument("--nproc", type=int, default=8)
    ap.add_argument("--num_gpus", type=int, default=None, help="GPUs per node (default: --nproc; -1: CPU/gloo)")
    ap.add_argument("--hidden", type=int, default=128)
    ap.add_argument("--epochs", type=int, default=20)
    ap.add_argument("--bs", type=int, default=1000)
    ap.add_argument("--eval_bs", type=int, default=100000)
    ap.add_argument("--eval_every", type=int, default=5)
    ap.add_argument("--repart", type=int, default=10)
    ap.add_argument("--log_every", type=int, default=20)
    ap.add_argument("--tag_prefix", default="t10n")
    ap.add_argument("--log_dir", default="log")
    ap.add_argument("--port", type=int, default=29611)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    sl = sub.add_parser("slurm", help="write a SLURM job-array script for the sweep")
    _sweep_args(sl)
    sl.add_argument("--out", default="jobs")
    sl.add_argument("--job_name", default="t10n_sweep")
    sl.add_argument("--partition", default=None)
    sl.add_argument("--nodes", type=int, default=1)
    sl.add_argument("--cpus", type=int, default=32)
    sl.add_argument("--mem", default="0")
    sl.add_argument("--time", default="1-00:00:00")
    sl.add_argument("--partition_step", action="store_true",
                    help="also write a job that builds the missing chunk sets first, and submit.sh chaining both")
    dk = sub.add_parser("docker", help="print (or run) one container per sweep configuration")
    _sweep_args(dk)
    dk.add_argument("--image", required=True)
    dk.add_argument("--workspace", default=None)
    dk.add_argument("--shm", default="64g")
    dk.add_argument("--execute", action="store_true")
    dk.add_argument("--partition_step", action="store_true", help="build the missing chunk sets first")
    hs = sub.add_parser("hosts", help="print the (host, n_gpu) pairs of a hosts file")
    hs.add_argument("path")
    il = sub.add_parser("inline", help="run one shell command on every host of a hosts file over ssh")
    il.add_argument("--host_file", required=True)
    il.add_argument("--tag_id", default="inline")
    il.add_argument("--work_dir", default=".")
    il.add_argument("--log_dir", default="log")
    il.add_argument("--time_limit", type=float, default=None, help="seconds")
    il.add_argument("--dry_run", action="store_true")
    il.add_argument("command", nargs=argparse.REMAINDER, help="-- then the command")
    args = ap.parse_args(argv)
    if getattr(args, "num_gpus", 0) is None:
        args.num_gpus = args.nproc  # one rank per GPU of the node
    if args.cmd == "slurm":
        print(write_slurm_job(args))
        return 0
    if args.cmd == "docker":
        return 1 if run_docker(args) else 0
    if args.cmd == "inline":
        cmd = args.command[1:] if args.command[:1] == ["--"] else args.command
        if not cmd:
            ap.error("inline needs a command after --")
        line = " ".join(shlex.quote(c) for c in cmd) if len(cmd) > 1 else cmd[0]
        out = util.cluster_run(args.host_file, args.tag_id, lambda hosts, i: line, work_dir=args.work_dir,
                               log_dir=args.log_dir, time_limit=args.time_limit, dry_run=args.dry_run)
        if args.dry_run:
            for argv_ in out:
                print(" ".join(shlex.quote(a) for a in argv_))
            return 0
        return 1 if any(c != 0 for c in out) else 0
    for host, n in parse_hosts_file(args.path):
        print(host, n)
    return 0


if __name__ == "__main__":
    sys.exit(main())
