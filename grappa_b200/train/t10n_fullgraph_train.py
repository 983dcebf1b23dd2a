"""Full-graph training CLI (reference: experiments/grappa/train/t10n_fullgraph_train.py:142-412).

Every rank trains its partition full-graph in isolation: the working graph is the
own partition plus the current neighbour partition (in-edges among their nodes),
one step per epoch over all of it, loss on the own training nodes, gradients
aggregated across ranks with the coverage-corrected all-reduce (coverage 1: the
working graph holds every in-edge among its rows), repartitioned every
``--repart_every`` epochs.  Same flags as grappa_b200.train.t10n_train.

Deviations (the reference's behaviour, decided differently here):
  * the reference multiplies every gradient by a coverage count that is never set
    (0.0, t10n_fullgraph_train.py:153) when n_part > 1; here the weight is 1;
  * the reference's loss covers every own node, training, validation and test
    (t10n_fullgraph_train.py:199-201); here only the training nodes.

  python -m grappa_b200.train.t10n_fullgraph_train --data_path D --graph_name G \\
      --part_method hash --n_part P --model gcn --num_gpus 1 --tag_id job
"""
import time

import numpy as np
import torch
import torch.distributed as dist
import torch.nn.functional as F

from grappa_b200.dataset.meta import name_to_meta
from grappa_b200.grad import coverage_all_reduce
from grappa_b200.models import get_model
from grappa_b200.train import resilience
from grappa_b200.train.t10n_train import build_parser, rank_print, save_to_ckpt, set_metrics_sink


def _cpu_full_block(loader):
    """Block over the own + neighbour nodes of the CPU loader's working graph."""
    from grappa_b200.block import Block

    ps = loader.prefix_sum
    r, q = loader.rank, loader.nbr_idx
    ids = [torch.arange(ps[r], ps[r + 1])]
    if q != r:
        ids.append(torch.arange(ps[q], ps[q + 1]))
    nodes = torch.cat(ids)
    ip = torch.from_numpy(loader.cur_g.indptr())
    ix = torch.from_numpy(loader.cur_g.indices())
    lid = torch.full((ps[-1],), -1, dtype=torch.int64)
    lid[nodes] = torch.arange(nodes.numel())
    beg, end = ip[nodes], ip[nodes + 1]
    deg = end - beg
    owner = torch.repeat_interleave(torch.arange(nodes.numel()), deg)
    e = torch.arange(int(deg.sum()))
    off = torch.zeros(nodes.numel() + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(deg, 0)
    src = lid[ix[beg[owner] + e - off[owner]]]
    keep = src >= 0
    cnt = torch.bincount(owner[keep], minlength=nodes.numel())
    indptr = torch.zeros(nodes.numel() + 1, dtype=torch.int64)
    indptr[1:] = torch.cumsum(cnt, 0)
    return Block(indptr, src[keep], nodes, nodes.numel(), nodes.numel()), nodes


def run_cpu(args):
    from grappa_b200.dataloader import IsolatedDataloader

    meta = name_to_meta(args.graph_name)
    torch.manual_seed(args.seed)
    model = get_model(args.model, meta.n_dim, meta.n_label, num_hidden=args.num_hidden, num_layers=args.num_layers,
                      dropout=args.dropout)
    opt = torch.optim.Adam(model.parameters(), lr=args.lr)
    loader = IsolatedDataloader(torch.device("cpu"), args)
    rank, world = loader.get_rank(), loader.world
    losses = []
    blk = nodes = x = None
    loss = torch.zeros(())
    for epoch in range(args.num_epochs):
        tic = time.time()
        if blk is None or epoch % args.repart_every == 0:
            loader.get_cur_dataloader(args, epoch)
            blk, nodes = _cpu_full_block(loader)
            x = torch.zeros((nodes.numel(), loader.in_feats))
            loader.get_batch_input(x, nodes)
        n_own = loader.get_num_node()
        tr = torch.nonzero(loader.train_mask).squeeze(1)
        labels = loader.node_label.long()
        t0 = time.time()
        out = model([blk] * len(model.layers), x)
        loss = F.cross_entropy(out[tr], labels[tr])
        t1 = time.time()
        opt.zero_grad(set_to_none=True)
        loss.backward()
        coverage_all_reduce(list(model.parameters()), 1.0, world)
        t2 = time.time()
        opt.step()
        t3 = time.time()
        losses.append(float(loss.detach()))
        if epoch % args.log_every == 0:
            ok = float((out[:n_own][tr].argmax(1) == labels[tr]).float().sum())
            rank_print("epoch|{:04d}|part|{:04d}|loss|{:.4f}|train_acc|{:.4f}|gpu_mb|{:.1f}|step_time|{:.2f}|"
                       "train:{:.1f},{:.1f}".format(epoch, rank, float(loss), ok / max(tr.numel(), 1), 0.0, t3 - t0,
                                                    ok, float(tr.numel())))
        rank_print("epoch_|epoch|{:04d}|part|{:04d}|epoch_seconds|{:.4f}|pcie|{:.4f}|forward|{:.4f}|backward|{:.4f}|"
                   "update|{:.4f}|account|{:.4f}".format(epoch, rank, time.time() - tic, 0.0, t1 - t0, t2 - t1,
                                                         t3 - t2, time.time() - t3))
    save_to_ckpt(args, args.num_epochs - 1, rank, model, opt.state_dict(), loss)
    return {"epochs": args.num_epochs, "loss": losses}


def run_gpu(args):
    from grappa_b200.graph_store import partition_from_chunks
    from grappa_b200.parallel.comm import Comm
    from grappa_b200.trainer import FullGraphTrainer

    rank = dist.get_rank() if dist.is_initialized() else 0
    world = dist.get_world_size() if dist.is_initialized() else 1
    device = torch.device("cuda", rank % max(args.num_gpus, 1))
    torch.cuda.set_device(device)
    meta = name_to_meta(args.graph_name)
    torch.manual_seed(args.seed)
    model = get_model(args.model, meta.n_dim, meta.n_label, num_hidden=args.num_hidden, num_layers=args.num_layers,
                      dropout=args.dropout)
    own = partition_from_chunks(args.data_path, args.graph_name, args.part_method, args.n_part, rank, meta.n_dim,
                                device)
    tr = FullGraphTrainer(model, own, lr=args.lr, repart_every=args.repart_every, comm=Comm() if world > 1 else None,
                          seed=args.seed)
    losses = []
    for epoch in range(args.num_epochs):
        tic = time.time()
        loss = tr.train_epoch(epoch)
        losses.append(loss)
        rank_print("epoch_|epoch|{:04d}|part|{:04d}|epoch_seconds|{:.4f}|loss|{:.4f}".format(
            epoch, rank, time.time() - tic, loss))
    # exact layer-wise inference across partitions (full neighbourhoods, not the isolated partition)
    va, te, trn = tr.evaluate_exact([own.val_mask, own.test_mask, own.train_mask])
    acc = {"val": va, "test": te, "train": trn}
    rank_print("infer_|epoch|{:04d}|part|{:04d}|val_acc|{:.4f}|test_acc|{:.4f}|train_acc|{:.4f}".format(
        args.num_epochs - 1, rank, acc["val"], acc["test"], acc["train"]))
    save_to_ckpt(args, args.num_epochs - 1, rank, model, tr.engine.optimizer_state_dict(), losses[-1] if losses else 0)
    tr.close()
    return {"epochs": args.num_epochs, "loss": losses, **{f"{k}_acc": v for k, v in acc.items()}}


def main(args, init_pg=True):
    if init_pg and not args.standalone and not dist.is_initialized():
        import datetime

        backend = args.backend if args.num_gpus != -1 else "gloo"
        resilience.init_process_group(backend, datetime.timedelta(seconds=args.pg_timeout))
    set_metrics_sink(getattr(args, "metrics_jsonl", None))
    return run_cpu(args) if args.num_gpus == -1 else run_gpu(args)


if __name__ == "__main__":
    a = build_parser().parse_args()
    print(a, flush=True)
    main(a)
    if dist.is_initialized():
        dist.destroy_process_group()
