"""Mini-batch training CLI with the reference's flags, log lines and checkpoints
(reference: experiments/grappa/train/t10n_train.py:148-510).

  python -m grappa_b200.train.t10n_train --data_path D --graph_name G --part_method hash \\
      --n_part P --model sage --num_hidden 128 --num_layers 3 --fan_out 15,10,5 \\
      --num_epochs 20 --batch_size 1000 --lr 0.003 --repart_every 50 --num_gpus -1 \\
      --tag_id job --close_dd

One process per partition (``torchrun --nproc-per-node P``).  ``--num_gpus -1``
trains on CPU ranks over gloo with the PyTorch layers, the C++ host sampler and
the coverage-weighted gradient all-reduce.  ``--num_gpus N`` trains on GPUs: the
partition is loaded from the same chunk files into HBM and every step runs on the
sm_100a engine (sampling, compaction, GEMMs, aggregation and the fused
all-reduce + Adam over NVLink peer memory), captured in a CUDA graph.

Log lines (``step_|...``, ``epoch_|...``, ``infer_|...``) keep the reference's
field order; checkpoints are ``{checkpoint_path}/epoch_{epoch:03d}.pt`` with keys
epoch / state_dict / optimizer_state_dict / loss.
"""
import argparse
import datetime
import json
import os
import socket
import time
from copy import deepcopy

import numpy as np
import torch
import torch.distributed as dist
import torch.nn.functional as F

from grappa_b200.dataset.meta import name_to_meta
from grappa_b200.grad import coverage_all_reduce
from grappa_b200.models import get_model
from grappa_b200.parallel.watchdog import PeerFailure
from grappa_b200.train import resilience


_METRICS = None  # JSONL sink of the metric lines (--metrics_jsonl)


def parse_metrics_line(line):
    """A ``kind_|key|value|key|value|...`` log line (step_, epoch_, infer_, or the
    full-graph trainer's per-step ``epoch|...`` line) as a dict with ``event`` and typed
    values; trailing ``name:value`` fields are kept too.  None for other text."""
    fields = line.strip().split("|")
    head = fields[0]
    if head in ("step_", "epoch_", "infer_"):
        rec, rest = {"event": head[:-1]}, fields[1:]
    elif head == "epoch" and len(fields) > 2:
        rec, rest = {"event": "step"}, fields
    else:
        return None

    def value(x):
        for cast in (int, float):
            try:
                return cast(x)
            except ValueError:
                pass
        return x

    i = 0
    while i < len(rest):
        tok = rest[i]
        if ":" in tok:  # a trailing name:value field
            k, _, v = tok.partition(":")
            rec[k] = value(v)
            i += 1
        elif i + 1 < len(rest):
            rec[tok] = value(rest[i + 1])
            i += 2
        else:
            i += 1
    return rec


def set_metrics_sink(path):
    """Append every metric line as one JSON object to ``path`` ({rank} in the path: one
    file per rank; otherwise rank 0 only).  Each record also holds the rank and the
    wall-clock time."""
    global _METRICS
    rank = dist.get_rank() if dist.is_initialized() else 0
    if not path or ("{rank}" not in path and rank != 0):
        _METRICS = None
        return
    path = path.format(rank=rank)
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    _METRICS = open(path, "a")


def rank_print(*args, **kwargs):
    rank = dist.get_rank() if dist.is_initialized() else 0
    if _METRICS is not None and args and isinstance(args[0], str):
        rec = parse_metrics_line(args[0])
        if rec is not None:
            rec.update(rank=rank, time=time.time())
            _METRICS.write(json.dumps(rec) + "\n")
            _METRICS.flush()
    if rank % 2 == 0:
        print(f"rank{rank}", *args, **kwargs, flush=True)


def compute_acc(pred, labels, device):
    n_correct = (torch.argmax(pred, dim=1) == labels.long()).float().sum()
    t = torch.tensor([float(n_correct), float(len(pred))], device=device)
    if dist.is_initialized():
        dist.all_reduce(t)
    return t


def resume_from_ckpt(model, optimizer, resume_path):
    if resume_path is None or resume_path.strip() == "":
        return -1
    ckpt = torch.load(resume_path, weights_only=False)
    model.load_state_dict(ckpt["state_dict"])
    if optimizer is not None:
        optimizer.load_state_dict(ckpt["optimizer_state_dict"])
    return int(ckpt["epoch"])


def save_to_ckpt(args, epoch, rank, model, optimizer_state, loss):
    if not args.checkpoint_path or args.checkpoint_path.strip() == "" or args.checkpoint_every <= 0:
        return None
    if (epoch + 1) % args.checkpoint_every != 0 or rank != 0:
        return None
    os.makedirs(args.checkpoint_path, exist_ok=True)
    name = f"{args.checkpoint_path}/epoch_{epoch:03d}.pt"
    state = model.state_dict_contiguous() if hasattr(model, "state_dict_contiguous") else model.state_dict()
    # written under a temporary name and renamed: a rank stopped mid-save (a restart ends
    # the attempt's processes) leaves no truncated epoch_NNN.pt for a resume to pick up
    torch.save({"epoch": epoch, "state_dict": state, "optimizer_state_dict": optimizer_state,
                "loss": float(loss.detach() if torch.is_tensor(loss) else loss)}, name + ".tmp")
    os.replace(name + ".tmp", name)
    return name


def run_cpu(args):
    """CPU ranks: the reference's training loop on the host engine."""
    from grappa_b200.dataloader import IsolatedDataloader
    from grappa_b200.infer import run_infer_xborder_by_layer as run_infer

    device = torch.device("cpu")
    meta = name_to_meta(args.graph_name)
    torch.manual_seed(args.seed)
    model = get_model(args.model, meta.n_dim, meta.n_label, num_hidden=args.num_hidden, num_layers=args.num_layers,
                      dropout=args.dropout)
    optimizer = torch.optim.Adam(model.parameters(), lr=args.lr)
    ckpt_epoch = resume_from_ckpt(model, optimizer, resilience.resolve_resume(args))
    loader = IsolatedDataloader(device, args)
    rank = loader.get_rank()
    world = loader.world
    watchdog = resilience.start_watchdog(args)
    best = {"val_acc": 0.0, "state_dict": None}
    iter_tput, epoch_loss = [], []
    loss = torch.zeros(())
    epoch = ckpt_epoch
    if ckpt_epoch >= 0:
        rank_print(f"resumed from epoch {ckpt_epoch}")
    for epoch in range(ckpt_epoch + 1, args.num_epochs):
        resilience.maybe_inject_fault(args, rank, epoch, watchdog)
        if watchdog is not None:
            try:
                watchdog.check()
            except PeerFailure as e:
                resilience.fault_exit(e, rank, epoch)
        tic = time.time()
        t = dict(sample=0.0, fetch=0.0, pcie=0.0, fwd=0.0, bwd=0.0, upd=0.0, acct=0.0)
        n_seed = n_input = 0
        losses = []
        step_time = []
        try:
            dataloader = loader.get_cur_dataloader(args, epoch)
            start = time.time()
            for step, (input_nodes, seeds, blocks) in enumerate(dataloader):
                t0 = time.time()
                t["sample"] += t0 - start
                x = torch.zeros([input_nodes.shape[0], loader.in_feats], dtype=torch.float32)
                loader.get_batch_input(x, input_nodes)
                coverage = loader.get_coarse_count() if world > 1 else 1.0
                labels = loader.get_batch_labels(seeds).long()
                t1 = time.time()
                t["fetch"] += t1 - t0
                n_seed += len(seeds)
                n_input += len(input_nodes)
                t2 = time.time()
                pred = model(blocks, x)
                loss = F.cross_entropy(pred, labels)
                t3 = time.time()
                optimizer.zero_grad(set_to_none=True)
                loss.backward()
                coverage_all_reduce(list(model.parameters()), coverage, world)
                t4 = time.time()
                optimizer.step()
                t5 = time.time()
                t["fwd"] += t3 - t2
                t["bwd"] += t4 - t3
                t["upd"] += t5 - t4
                step_time.append(t5 - t0)
                iter_tput.append(len(seeds) / max(t5 - t0, 1e-9))
                losses.append(float(loss.detach()))
                if step % args.log_every == 0:
                    acc = compute_acc(pred.detach(), labels, loader.get_comm_dev())
                    rank_print("step_|epoch|{:04d}|step|{:04d}|part|{:04d}|loss|{:.4f}|train_acc|{:.4f}|sample_p_s|{:.2f}|"
                               "gpu_mb|{:.1f}|step_time|{:.2f}|train:{:.1f},{:.1f}".format(
                                   epoch, step, rank, float(loss), float(acc[0] / max(acc[1], 1)),
                                   float(np.mean(iter_tput[3:])) if len(iter_tput) > 3 else 0.0, 0.0,
                                   float(np.sum(step_time[-args.log_every:])), float(acc[0]), float(acc[1])))
                start = time.time()
                t["acct"] += start - t5
        except Exception as e:  # a collective that timed out: name the silent peers if the watchdog can
            if watchdog is not None:
                try:
                    watchdog.check()
                except PeerFailure as pf:
                    resilience.fault_exit(f"{pf} ({type(e).__name__} in epoch {epoch})", rank, epoch)
            raise
        toc = time.time()
        epoch_loss.append(float(np.mean(losses)) if losses else 0.0)
        rank_print("epoch_|epoch|{:04d}|part|{:04d}|epoch_seconds|{:.4f}|sampling|{:.4f}|f_fetch|{:.4f}|pcie|{:.4f}|"
                   "forward|{:.4f}|backward|{:.4f}|update|{:.4f}|account|{:.4f}|n_seed|{:012d}|n_input|{:012d}".format(
                       epoch, rank, toc - tic, t["sample"], t["fetch"], t["pcie"], t["fwd"], t["bwd"], t["upd"],
                       t["acct"], n_seed, n_input))
        resilience.periodic_checkpoint(args, epoch, rank, model, optimizer.state_dict, loss)
        if epoch != 0 and (epoch + 1) % args.eval_every == 0:
            c = run_infer(model, loader, device, args, subset_tag="valid")
            val_acc = float(c[1]) / max(float(c[4]), 1.0)
            rank_print(f"epoch={epoch}, val_acc={val_acc}")
            if val_acc >= best["val_acc"]:
                best["val_acc"] = val_acc
                best["state_dict"] = deepcopy(model.state_dict_contiguous())
    summary = {"epochs": epoch + 1, "loss": epoch_loss, "val_acc": 0.0, "test_acc": 0.0, "train_acc": 0.0}
    if watchdog is not None:
        watchdog.stop()
    if best["state_dict"] is not None:
        t0 = time.time()
        model.load_state_dict(best["state_dict"])
        c = run_infer(model, loader, device, args, subset_tag="all")
        tr, va, te = (float(c[i]) / max(float(c[i + 3]), 1.0) for i in range(3))
        rank_print("infer_|epoch|{:04d}|part|{:04d}|val_acc|{:.4f}|test_acc|{:.4f}|train_acc|{:.4f}|time_sec|{:.4f}|"
                   "val:{:.1f}|test:{:.1f}|train:{:.1f}".format(epoch, rank, va, te, tr, time.time() - t0,
                                                                 float(c[4]), float(c[5]), float(c[3])))
        summary.update(val_acc=va, test_acc=te, train_acc=tr)
    save_to_ckpt(args, epoch, rank, model, optimizer.state_dict(), loss)
    return summary


def run_gpu(args):
    """GPU ranks: chunk files -> HBM partition -> sm_100a engine."""
    from grappa_b200.graph_store import partition_from_chunks
    from grappa_b200.parallel.comm import Comm
    from grappa_b200.trainer import MiniBatchTrainer

    rank = dist.get_rank() if dist.is_initialized() else 0
    world = dist.get_world_size() if dist.is_initialized() else 1
    device = torch.device("cuda", rank % max(args.num_gpus, 1))
    torch.cuda.set_device(device)
    meta = name_to_meta(args.graph_name)
    torch.manual_seed(args.seed)
    model = get_model(args.model, meta.n_dim, meta.n_label, num_hidden=args.num_hidden, num_layers=args.num_layers,
                      dropout=args.dropout)
    ckpt = None
    resume = resilience.resolve_resume(args)
    if resume:
        ckpt = torch.load(resume, weights_only=False)
        model.load_state_dict(ckpt["state_dict"])
    own = partition_from_chunks(args.data_path, args.graph_name, args.part_method, args.n_part, rank, meta.n_dim,
                                device)
    comm = Comm() if world > 1 else None
    fanouts = [int(f) for f in args.fan_out.split(",")]
    trainer = MiniBatchTrainer(model, own, fanouts, args.batch_size, lr=args.lr, repart_every=args.repart_every,
                               comm=comm, seed=args.seed)
    if ckpt is not None:
        trainer.engine.load_optimizer_state_dict(ckpt["optimizer_state_dict"])
    first = int(ckpt["epoch"]) + 1 if ckpt is not None else 0
    trainer.warmup()
    watchdog = resilience.start_watchdog(args)
    trainer.watchdog = watchdog  # checked by train_epoch before the epoch's first collective
    best = {"val_acc": 0.0, "state_dict": None}
    epoch_loss = []
    epoch = first - 1
    for epoch in range(first, args.num_epochs):
        resilience.maybe_inject_fault(args, rank, epoch, watchdog)
        tic = time.time()
        try:
            loss = trainer.train_epoch(epoch, host_feed=True)
        except PeerFailure as e:
            resilience.fault_exit(e, rank, epoch)
        toc = time.time()
        epoch_loss.append(float(loss))
        rank_print("epoch_|epoch|{:04d}|part|{:04d}|epoch_seconds|{:.4f}|loss|{:.4f}|n_seed|{:012d}".format(
            epoch, rank, toc - tic, float(loss), int(trainer.train_ids.numel())))
        resilience.periodic_checkpoint(args, epoch, rank, model, trainer.engine.optimizer_state_dict, float(loss))
        if epoch != 0 and (epoch + 1) % args.eval_every == 0:
            val_acc = trainer.evaluate_exact([own.val_mask])[0]
            rank_print(f"epoch={epoch}, val_acc={val_acc}")
            if val_acc >= best["val_acc"]:
                best["val_acc"] = val_acc
                best["state_dict"] = model.state_dict_contiguous()
    summary = {"epochs": epoch + 1, "loss": epoch_loss, "val_acc": 0.0, "test_acc": 0.0, "train_acc": 0.0}
    if watchdog is not None:
        watchdog.stop()
        trainer.watchdog = None
    if best["state_dict"] is not None:
        t0 = time.time()
        trainer.load_state_dict(best["state_dict"])
        # exact layer-wise inference across partitions (reference: run_infer_xborder_by_layer)
        va, te, trn = trainer.evaluate_exact([own.val_mask, own.test_mask, own.train_mask])
        acc = {"val": va, "test": te, "train": trn}
        rank_print("infer_|epoch|{:04d}|part|{:04d}|val_acc|{:.4f}|test_acc|{:.4f}|train_acc|{:.4f}|time_sec|{:.4f}"
                   .format(epoch, rank, acc["val"], acc["test"], acc["train"], time.time() - t0))
        summary.update(val_acc=acc["val"], test_acc=acc["test"], train_acc=acc["train"])
    save_to_ckpt(args, epoch, rank, model, trainer.engine.optimizer_state_dict(),
                 epoch_loss[-1] if epoch_loss else 0.0)
    trainer.close()
    return summary


def main(args, init_pg=True):
    print(socket.gethostname(), "Initializing", flush=True)
    if init_pg and not args.standalone:
        backend = args.backend if args.num_gpus != -1 else "gloo"
        resilience.init_process_group(backend, datetime.timedelta(seconds=args.pg_timeout))
    set_metrics_sink(getattr(args, "metrics_jsonl", None))
    if args.num_gpus == -1:
        return run_cpu(args)
    return run_gpu(args)


def build_parser():
    p = argparse.ArgumentParser(description="t10n_train")
    p.add_argument("--data_path", type=str, help="path where you put dataset for t10n")
    p.add_argument("--graph_name", type=str, help="graph name")
    p.add_argument("--part_method", type=str, help="name of the partition method")
    p.add_argument("--n_part", type=int, help="number of partitions")
    p.add_argument("--model", type=str, default="sage", required=True, help="gnn model in(sage, gcn, gat, gin, pinsage)")
    p.add_argument("--num_hidden", type=int, default=128)
    p.add_argument("--num_layers", type=int, default=3)
    p.add_argument("--fan_out", type=str, default="15,10,5")
    p.add_argument("--num_epochs", type=int, default=20)
    p.add_argument("--batch_size", type=int, default=1000)
    p.add_argument("--batch_size_eval", type=int, default=100000)
    p.add_argument("--lr", type=float, default=0.003)
    p.add_argument("--dropout", type=float, default=0.5)
    p.add_argument("--stop_at_border", action="store_true", default=False, help="sampler will stop at border")
    p.add_argument("--disable_backup_server", action="store_true", default=False)
    p.add_argument("--repart_every", type=int, default=50)
    p.add_argument("--num_gpus", type=int, default=-1, help="#GPU per machine. Use -1 for CPU training")
    p.add_argument("--standalone", action="store_true", help="run in the standalone mode")
    p.add_argument("--backend", type=str, default="gloo", help="pytorch distributed backend")
    p.add_argument("--socket_ifname", type=str, default="eth0")
    p.add_argument("--log_every", type=int, default=20)
    p.add_argument("--eval_every", type=int, default=5)
    p.add_argument("--resume_path", type=str, default=None, help="resume from a path of a checkpoint")
    p.add_argument("--checkpoint_path", type=str, default=None, help="a path to store all checkpoints")
    p.add_argument("--checkpoint_every", type=int, default=-1, help="save a checkpoint every N epochs")
    p.add_argument("--tag_id", type=str, required=True, help="name for this job")
    p.add_argument("--close_dd", action="store_true", help="native sampler (the only sampler of this framework)")
    p.add_argument("--seed", type=int, default=0, help="seed of sampling, shuffling and initialisation")
    p.add_argument("--pg_timeout", type=int, default=600, help="process group timeout in seconds")
    p.add_argument("--heartbeat_limit", type=float, default=0.0,
                   help="seconds without a peer's heartbeat before this rank stops with exit code 3 (0: off)")
    p.add_argument("--inject_fault", type=str, default=None,
                   help="RANK:EPOCH:{exit,hang} - that rank leaves at the start of that epoch (first attempt only)")
    p.add_argument("--metrics_jsonl", type=str, default=None,
                   help="also append the step_/epoch_/infer_ lines as JSON objects to this file ({rank}: one per rank)")
    return p


def parse_args(argv=None):
    return build_parser().parse_args(argv)


if __name__ == "__main__":
    a = parse_args()
    print(a, flush=True)
    out = main(a)
    if dist.is_initialized():
        dist.destroy_process_group()
