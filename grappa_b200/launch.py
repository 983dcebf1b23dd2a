"""Sweep launcher and result table (reference: experiments/grappa/t10nrun.py:138-233,
experiments/grappa/help.py:9-56, templates experiments/grappa/train.sh.template).

One node, one process per GPU: every configuration of the sweep (partition
method x graph x run x model x (layers, fanout)) expands a command template and
runs it with ``torch.distributed.run`` on 127.0.0.1, its output in
``{log_dir}/{tag}_0.txt``.  The reference fans out over ssh to many hosts; the
product here is one 8-GPU box.

    python -m grappa_b200.launch --data_path D --graphs rmat16k --models sage,gcn \\
        --layers_fanouts "2:10,5" --nproc 2 --num_gpus -1 --runs 1 [--dry_run]
    python -m grappa_b200.launch --table log      # markdown table of the infer_ lines

With ``--partition`` the sweep first builds the chunk sets it needs that are not on
disk (``grappa_b200.dataset.partition seq`` from ``{data_path}/t10n/{graph}``, after
generating that directory for a synthetic graph name when it is missing), the role of
the reference's ``t10nrun.py --task partition`` (experiments/grappa/t10nrun.py,
partition.sh.template).
"""
import argparse
import itertools
import os
import re
import shlex
import subprocess
import sys
from collections import defaultdict

TEMPLATE = ("{python} -m torch.distributed.run --nnodes=1 --nproc-per-node {nproc} --master-addr 127.0.0.1 "
            "--master-port {port} -m grappa_b200.train.{script} --data_path {data_path} --graph_name {graph} "
            "--part_method {part} --n_part {nproc} --model {model} --num_layers {layers} --fan_out {fanout} "
            "--num_hidden {hidden} --num_epochs {epochs} --batch_size {bs} --batch_size_eval {eval_bs} "
            "--eval_every {eval_every} --repart_every {repart} --num_gpus {num_gpus} --backend {backend} "
            "--log_every {log_every} --tag_id {tag} --close_dd")


def sweep(args):
    """Yield (tag, command) for every configuration of the sweep."""
    lf = []
    for item in args.layers_fanouts.split(";"):
        layers, fanout = item.split(":")
        lf.append((int(layers), fanout))
    combos = itertools.product(args.parts.split(","), args.graphs.split(","), range(1, args.runs + 1),
                               args.models.split(","), lf)
    for i, (part, graph, run, model, (layers, fanout)) in enumerate(combos):
        tag = f"{args.tag_prefix}_{part}_{graph}_{model}_{layers}_{args.nproc}_R{run}"
        cmd = TEMPLATE.format(python=sys.executable, nproc=args.nproc, port=args.port + i,
                              script=args.script, data_path=args.data_path, graph=graph, part=part, model=model,
                              layers=layers, fanout=fanout, hidden=args.hidden, epochs=args.epochs, bs=args.bs,
                              eval_bs=args.eval_bs, eval_every=args.eval_every, repart=args.repart,
                              num_gpus=args.num_gpus, backend="gloo" if args.num_gpus == -1 else "nccl",
                              log_every=args.log_every, tag=tag)
        yield tag, cmd


def partition_commands(args):
    """Yield (tag, command) for every chunk set of the sweep missing under data_path
    (n_part = nproc), preceded once per graph by its generation when the graph's
    pre-partition directory has no t10n.json."""
    from grappa_b200.dataset.meta import t10n_chunk_path

    generated = set()
    for part, graph in dict.fromkeys(itertools.product(args.parts.split(","), args.graphs.split(","))):
        if os.path.isdir(os.path.join(args.data_path, t10n_chunk_path(graph, part, args.nproc))):
            continue
        src = os.path.join(args.data_path, "t10n", graph)
        if graph not in generated and not os.path.exists(os.path.join(src, "t10n.json")):
            generated.add(graph)
            yield f"generate_{graph}", (f"{sys.executable} -m grappa_b200.dataset.partition generate "
                                        f"--graph_name {graph} --out {shlex.quote(src)}")
        yield f"partition_{part}_{graph}_{args.nproc}", (
            f"{sys.executable} -m grappa_b200.dataset.partition seq --src_path {shlex.quote(src)} "
            f"--dest_path {shlex.quote(args.data_path)} --graph_name {graph} --part_method {part} "
            f"--n_part {args.nproc}")


def run_sweep(args):
    os.makedirs(args.log_dir, exist_ok=True)
    failed = 0
    steps = list(partition_commands(args)) if getattr(args, "partition", False) else []
    for tag, cmd in steps + list(sweep(args)):
        print(cmd, flush=True)
        if args.dry_run:
            continue
        with open(os.path.join(args.log_dir, f"{tag}_0.txt"), "w") as log:
            try:
                rc = subprocess.run(shlex.split(cmd), stdout=log, stderr=subprocess.STDOUT,
                                    timeout=args.timeout).returncode
            except subprocess.TimeoutExpired:
                rc = -1
        print(f"{tag}: exit {rc}", flush=True)
        failed += rc != 0
    return failed


_FILE = re.compile(r"_(\w+?)_(\w+?)_(gcn|sage|gat|gin|pinsage)_(\d+)_\d+_R\d+_0\.txt$")
_INFER = re.compile(r"infer_.*\|test_acc\|([\d.]+)")


def result_table(log_dir):
    """Markdown table (rows model_layers, columns graph) of the last infer_ line's test
    accuracy, as the reference's help.py prints it.  When the logs hold several partition
    methods the rows are split by method (``sage_3 [metis]``), and several runs of one
    configuration are averaged (``0.6146 (3 runs)``)."""
    data = defaultdict(lambda: defaultdict(list))
    parts = set()
    for root, _, files in os.walk(log_dir):
        for fname in files:
            m = _FILE.search(fname)
            if not m:
                continue
            part, graph, model, layers = m.groups()
            with open(os.path.join(root, fname)) as f:
                lines = [l for l in f if "infer_" in l and "test_acc" in l]
            if not lines:
                continue
            a = _INFER.search(lines[-1])
            if a:
                parts.add(part)
                data[(model, int(layers), part)][graph].append(float(a.group(1)))
    split = len(parts) > 1
    graphs = sorted({g for d in data.values() for g in d})
    out = ["| " + " | ".join(["Model_Layer"] + graphs) + " |", "|" + "|".join(["---"] * (len(graphs) + 1)) + "|"]

    def cell(v):
        if not v:
            return ""
        mean = round(sum(v) / len(v), 4)
        return str(mean) if len(v) == 1 else f"{mean} ({len(v)} runs)"

    for model, layers, part in sorted(data):
        name = f"{model}_{layers}" + (f" [{part}]" if split else "")
        out.append("| " + " | ".join([name] + [cell(data[(model, layers, part)].get(g, [])) for g in graphs]) + " |")
    return "\n".join(out)


def main(argv=None):
    ap = argparse.ArgumentParser(description="sweep launcher")
    ap.add_argument("--table", default=None, help="print the result table of a log directory and exit")
    ap.add_argument("--script", default="t10n_train", choices=["t10n_train", "t10n_fullgraph_train"])
    ap.add_argument("--data_path", default="data")
    ap.add_argument("--parts", default="hash")
    ap.add_argument("--graphs", default="rmat16k")
    ap.add_argument("--models", default="sage")
    ap.add_argument("--layers_fanouts", default="3:15,10,5")
    ap.add_argument("--runs", type=int, default=1)
    ap.add_argument("--nproc", type=int, default=1)
    ap.add_argument("--num_gpus", type=int, default=1)
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
    ap.add_argument("--timeout", type=int, default=3600)
    ap.add_argument("--partition", action="store_true",
                    help="first build the missing chunk sets (and synthetic source graphs) of the sweep")
    ap.add_argument("--dry_run", action="store_true")
    args = ap.parse_args(argv)
    if args.table:
        print(result_table(args.table))
        return 0
    return run_sweep(args)


if __name__ == "__main__":
    sys.exit(main())
