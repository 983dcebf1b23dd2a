"""Multi-GPU tests (2 ranks, one process per GPU, NCCL for bootstrap only):
the fused coverage-weighted all-reduce + Adam over peer memory, the peer-memory
repartition, and a short partition-parallel training run."""
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(fn, port, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_entry, args=(r, port, fn, q) + args) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(WORLD):
        r, ok, payload = q.get(timeout=600)
        results[r] = (ok, payload)
    for p in procs:
        p.join(timeout=120)
    for r, (ok, payload) in sorted(results.items()):
        assert ok, f"rank {r} failed:\n{payload}"
    return {r: payload for r, (ok, payload) in results.items()}


def _entry(rank, port, fn, q, *args):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(WORLD),
                          LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        out = fn(rank, *args)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, True, out))
    except Exception:
        q.put((rank, False, traceback.format_exc()))


def _ar_body(rank, mode, dtype_name):
    """Two ranks, two buckets, three steps of the fused all-reduce + Adam against torch's
    Adam on the coverage-weighted mean of both ranks' gradients (rebuilt on the CPU)."""
    from grappa_b200.parallel.allreduce import FusedAllReduceAdam
    from grappa_b200.parallel.comm import Comm
    from grappa_b200.sampler_gpu import new_counters

    dtype = getattr(torch, dtype_name)
    dev = torch.device("cuda", rank)
    n = 300001
    comm = Comm()
    buckets = [(0, 120000), (120000, n)]
    ar = FusedAllReduceAdam(comm, n, buckets, grad_dtype=dtype, modes=[mode, mode])
    p0 = torch.randn(n, generator=torch.Generator(device="cpu").manual_seed(5))
    ar.param.copy_(p0)
    m, v = torch.zeros(n, device=dev), torch.zeros(n, device=dev)
    wbf = torch.zeros(n, dtype=torch.bfloat16, device=dev)
    counters = new_counters(0, dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    cov = torch.zeros(2, device=dev)
    ar.bind(counters, m, v, wbf, 1e-2, err=err, cov=cov)
    p_ref = torch.nn.Parameter(p0.clone())
    opt = torch.optim.Adam([p_ref], lr=1e-2)
    cleared = True
    for step in range(3):
        grads = [torch.randn(n, generator=torch.Generator(device="cpu").manual_seed(100 * step + r)).to(dtype)
                 for r in range(WORLD)]
        c = [0.5 + 0.25 * r for r in range(WORLD)]  # coverage weight of each rank
        cov.copy_(torch.tensor([c[rank] * 8.0, 8.0]))
        ar.grad.copy_(grads[rank])
        ar.launch(1)  # buckets in backward order
        ar.launch(0)
        torch.cuda.synchronize()
        assert err.item() == 0, err.item()
        cleared = cleared and bool((ar.grad == 0).all())
        counters[3] += 1  # next step (flag tags and slot parity)
        counters[5] += 1  # Adam step
        want = torch.zeros(n, dtype=torch.float64)
        for r in range(WORLD):
            want += c[r] / WORLD * grads[r].double()
        p_ref.grad = want.float()
        opt.step()
    ar.sync_moments(m, v)
    # numpy arrays travel through the result queue by value (tensors would be shared by
    # file descriptor, which dies with the child process)
    out = {"param": ar.param.cpu().numpy().copy(), "ref": p_ref.detach().numpy().copy(), "cleared": cleared,
           "wbf_ok": bool(torch.equal(wbf, ar.param.to(torch.bfloat16))),
           "m_err": float((m.cpu() - opt.state[p_ref]["exp_avg"]).abs().max())}
    ar.close()
    return out


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("dtype_name", ["float32", "bfloat16"])
def test_fused_allreduce_two_ranks(mode, dtype_name):
    res = _run(_ar_body, _free_port(), mode, dtype_name)
    for r in range(WORLD):
        o = res[r]
        assert o["cleared"] and o["wbf_ok"]
        np.testing.assert_allclose(o["param"], o["ref"], rtol=1e-5, atol=1e-5)
        assert o["m_err"] < 1e-5
    # every rank holds bit-identical parameters
    assert np.array_equal(res[0]["param"], res[1]["param"])


def _repart_body(rank):
    from grappa_b200.dataset import synthetic as S
    from grappa_b200.graph_store import PartitionStore, partition_from_global
    from grappa_b200.parallel.comm import Comm

    dev = torch.device("cuda", rank)
    g = S.build(S.SPECS["tiny"], dev)
    own = partition_from_global(g, WORLD, rank, dev, part_seed=7)
    store = PartitionStore(own, Comm())
    nbr = (rank + 1) % WORLD
    w = store.repartition(nbr)
    torch.cuda.synchronize()
    store.check_errors()
    # CPU reconstruction of the working graph from the global graph
    n = g.n_nodes
    pid = torch.from_numpy(__import__("grappa_b200").host().c_dist.random_assign_pid(n, WORLD, 7))
    order = torch.argsort(pid * n + torch.arange(n))
    new_id = torch.empty(n, dtype=torch.int64)
    new_id[order] = torch.arange(n)
    u = new_id[g.u.cpu()]
    v = new_id[g.v.cpu()]
    prefix = own.prefix
    lo_r, hi_r, lo_q, hi_q = prefix[rank], prefix[rank + 1], prefix[nbr], prefix[nbr + 1]
    n_r, n_q = hi_r - lo_r, hi_q - lo_q
    halo = int(w.n_halo_dev.item())
    ids = torch.empty(n_r + n_q + halo, dtype=torch.int64)
    ids[:n_r] = torch.arange(lo_r, hi_r)
    ids[n_r:n_r + n_q] = torch.arange(lo_q, hi_q)
    ids[n_r + n_q:] = store._halo_ids[:halo].cpu()
    # every in-edge of own and neighbour nodes (plus their self-loops) must be in the working CSR
    ip = w.indptr.cpu()
    ix = w.indices.cpu().long()
    checked = 0
    for wv in list(range(0, n_r, max(1, n_r // 50))) + list(range(n_r, n_r + n_q, max(1, n_q // 50))):
        gv = int(ids[wv])
        want = set(u[v == gv].tolist()) | {gv}
        got = set(ids[ix[ip[wv]:ip[wv + 1]]].tolist())
        assert got == want, (wv, gv)
        checked += 1
    # halo rows: sources outside both partitions, sorted, features pulled from their owners
    hal = ids[n_r + n_q:]
    assert bool((hal[1:] > hal[:-1]).all())
    assert bool((((hal < lo_r) | (hal >= hi_r)) & ((hal < lo_q) | (hal >= hi_q))).all())
    feat_all = torch.zeros((n, w.feat.shape[1]))
    feat_all[new_id, : g.spec.feat_dim] = g.feat.cpu()
    wf = w.feat[: n_r + n_q + halo].float().cpu()
    torch.testing.assert_close(wf, feat_all[ids].to(torch.bfloat16).float())
    store.close()
    return checked


def test_repartition_two_ranks():
    res = _run(_repart_body, _free_port())
    assert all(v > 10 for v in res.values())


def _train_body(rank, ar_mode=None):
    import torch.nn.functional as F

    from grappa_b200.dataset import synthetic as S
    from grappa_b200.graph_store import partition_from_global
    from grappa_b200.models import SAGE
    from grappa_b200.parallel.comm import Comm
    from grappa_b200.trainer import MiniBatchTrainer

    dev = torch.device("cuda", rank)
    g = S.build(S.SPECS["tiny"], dev)
    own = partition_from_global(g, WORLD, rank, dev, part_seed=3)
    torch.manual_seed(0)
    model = SAGE(g.spec.feat_dim, 64, g.spec.n_classes, 3, F.relu, 0.5)
    tr = MiniBatchTrainer(model, own, [10, 10, 5], 128, comm=Comm(), seed=2, repart_every=2, ar_mode=ar_mode)
    tr.warmup()
    losses = []
    for e in range(5):  # crosses two repartitions
        losses.append(tr.train_epoch(e, host_feed=True))
    torch.cuda.synchronize()
    tr.engine.check_errors()
    flat = tr.engine.flat.cpu().clone()
    acc = tr.evaluate(own.val_mask)
    tr.close()
    return {"losses": losses, "flat_sum": float(flat.double().sum()), "flat_head": flat[:64].tolist(), "acc": acc}


@pytest.mark.parametrize("ar_mode", [None, "shard"])
def test_partition_parallel_training_two_ranks(ar_mode):
    res = _run(_train_body, _free_port(), ar_mode)
    a, b = res[0], res[1]
    # the fused all-reduce + Adam keeps the replicas bit-identical
    assert a["flat_head"] == b["flat_head"] and a["flat_sum"] == b["flat_sum"]
    assert a["losses"][-1] < a["losses"][0]
    assert a["acc"] == b["acc"]


def _train_model_body(rank, name, full):
    from grappa_b200.dataset import synthetic as S
    from grappa_b200.graph_store import partition_from_global
    from grappa_b200.models import get_model
    from grappa_b200.parallel.comm import Comm
    from grappa_b200.trainer import FullGraphTrainer, MiniBatchTrainer

    dev = torch.device("cuda", rank)
    g = S.build(S.SPECS["tiny"], dev)
    own = partition_from_global(g, WORLD, rank, dev, part_seed=3)
    torch.manual_seed(0)
    model = get_model(name, g.spec.feat_dim, g.spec.n_classes, num_hidden=32, num_layers=2, dropout=0.2, n_heads=2)
    if full:
        tr = FullGraphTrainer(model, own, comm=Comm(), seed=2, repart_every=2, lr=1e-2)
    else:
        tr = MiniBatchTrainer(model, own, [5, 5], 128, comm=Comm(), seed=2, repart_every=2, lr=1e-2)
        tr.warmup()
    losses = []
    for e in range(5):
        losses.append(tr.train_epoch(e) if full else tr.train_epoch(e, host_feed=True))
    torch.cuda.synchronize()
    tr.engine.check_errors()
    flat = tr.engine.flat.cpu().clone()
    tr.close()
    return {"losses": losses, "flat_sum": float(flat.double().sum()), "flat_head": flat[:64].tolist()}


@pytest.mark.parametrize("name,full", [("gcn", True), ("gat", False), ("gin", False), ("pinsage", False)])
def test_model_families_two_ranks(name, full):
    res = _run(_train_model_body, _free_port(), name, full)
    a, b = res[0], res[1]
    assert a["flat_head"] == b["flat_head"] and a["flat_sum"] == b["flat_sum"]
    assert all(np.isfinite(a["losses"]))


def _exact_infer_body(rank):
    """Exact inference is partition-invariant: the accuracy over two partitions equals
    the single-partition accuracy of the same weights; the peer all-to-all and the
    peer-memory xb_gather return the owners' rows."""
    from grappa_b200.cl import PeerAllToAll
    from grappa_b200.dataset import synthetic as S
    from grappa_b200.graph_store import partition_from_global
    from grappa_b200.infer_gpu import ExactInference
    from grappa_b200.models import get_model
    from grappa_b200.parallel.comm import Comm
    from grappa_b200.xborder import xb_gather_peer

    dev = torch.device("cuda", rank)
    g = S.build(S.SPECS["tiny"], dev)
    comm = Comm()
    torch.manual_seed(6)
    model = get_model("sage", g.spec.feat_dim, g.spec.n_classes, num_hidden=48, num_layers=3, dropout=0.0)
    model.place(dev)
    own = partition_from_global(g, WORLD, rank, dev, part_seed=3)
    ex = ExactInference(model, own, comm)
    acc2 = ex.accuracy([own.val_mask, own.test_mask])
    ex.close()
    solo = partition_from_global(g, 1, 0, dev)
    ex1 = ExactInference(model, solo, _SoloComm())
    acc1 = ex1.accuracy([solo.val_mask, solo.test_mask])
    ex1.close()
    # peer-memory gather of feature rows by global id
    a2a = PeerAllToAll(comm, dev)
    n_global = own.prefix[-1]
    ids = torch.randint(0, n_global, (777,), generator=torch.Generator().manual_seed(rank)).to(dev)
    out = torch.zeros((777, own.feat.shape[1]), dtype=torch.float32, device=dev)
    xb_gather_peer(a2a, out, ids, own.feat, rank, WORLD, own.prefix)
    parts = [partition_from_global(g, WORLD, p, dev, part_seed=3) for p in range(WORLD)]
    table = torch.cat([p.feat for p in parts]).float()
    gather_ok = bool(torch.equal(out, table[ids]))
    a2a.close()
    return {"acc2": acc2, "acc1": acc1, "gather_ok": gather_ok}


class _SoloComm:
    rank, world = 0, 1

    def barrier(self):
        pass

    def all_reduce_sum(self, v):
        return v

    def all_gather_object(self, obj):
        return [obj]


def test_exact_inference_partition_invariant():
    res = _run(_exact_infer_body, _free_port())
    for r in range(WORLD):
        o = res[r]
        assert o["gather_ok"]
        for a2, a1 in zip(o["acc2"], o["acc1"]):
            assert abs(a2 - a1) < 5e-3, (o["acc2"], o["acc1"])
