"""The reference-compatible Python API on CPU ranks (gloo): chunking, the partition
data loader with its neighbour-partition working graph, cross-partition
layer-wise inference (checked against a full-graph forward) and the training CLI."""
import os
import socket
import sys
import traceback
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from grappa_b200.dataset import synthetic
from grappa_b200.dataset.chunk_seq import build_chunks_seq

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _entry(rank, world, port, fn, q, args):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
        import datetime

        torch.set_num_threads(2)
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
        out = fn(rank, args)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, True, out))
    except Exception:
        q.put((rank, False, traceback.format_exc()))


def run_ranks(fn, args, world=WORLD):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, q, args)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, ok, payload = q.get(timeout=600)
        res[r] = (ok, payload)
    for p in procs:
        p.join(timeout=60)
    for r, (ok, payload) in sorted(res.items()):
        assert ok, f"rank {r} failed:\n{payload}"
    return {r: p for r, (_, p) in res.items()}


@pytest.fixture(scope="module")
def tiny_chunks(tmp_path_factory):
    root = tmp_path_factory.mktemp("t10n")
    g = synthetic.build("tiny")
    synthetic.to_t10n_layout(g, str(root / "src"))
    out, stats = build_chunks_seq(str(root), "tiny", str(root / "src"), "hash", WORLD)
    return SimpleNamespace(root=str(root), path=out, graph=g, stats=stats)


def _args(root, **kw):
    a = dict(graph_name="tiny", backend="gloo", n_part=WORLD, data_path=root, part_method="hash", batch_size=256,
             fan_out="5,5", repart_every=2, model="sage", num_layers=2, num_hidden=16, batch_size_eval=700, seed=3,
             dropout=0.0)
    a.update(kw)
    return SimpleNamespace(**a)


def test_chunks_cover_graph(tiny_chunks):
    from grappa_b200.dataset.io_dist import ChunkIO

    io = ChunkIO(tiny_chunks.path, WORLD, 32)
    g = tiny_chunks.graph
    assert io.prefix[-1] == g.n_nodes
    n_edges = 0
    for p in range(WORLD):
        oid = io.part(p, "oid")
        assert np.allclose(io.part(p, "nfeat"), g.feat.numpy()[oid])
        n_edges += len(io.part(p, "u")) - len(oid)
        for j in range(WORLD):
            if j != p:
                bu, _ = io.bridge(p, j)
                n_edges += 0 if bu is None else len(bu)
    assert n_edges == g.u.numel()


def _loader_body(rank, a):
    from grappa_b200.dataloader import IsolatedDataloader

    args = _args(a["root"])
    ld = IsolatedDataloader(torch.device("cpu"), args)
    oid = [np.fromfile(f"{ld.data_path}/p{p}.oid.bin", dtype=np.int64) for p in range(WORLD)]
    gid2oid = np.concatenate(oid)
    feat = np.load(f"{a['root']}/src/node_feat.bin.npy")
    checked = 0
    for epoch in range(3):
        dl = ld.get_cur_dataloader(args, epoch)
        assert ld.nbr_idx == 1 - rank
        for step, (input_nodes, seeds, blocks) in enumerate(dl):
            assert torch.all((seeds >= ld.prefix_sum[rank]) & (seeds < ld.prefix_sum[rank + 1]))
            assert torch.all(ld.train_mask[seeds - ld.prefix_sum[rank]] == 1)
            x = torch.zeros((input_nodes.shape[0], ld.in_feats))
            ld.get_batch_input(x, input_nodes)
            assert np.allclose(x.numpy(), feat[gid2oid[input_nodes.numpy()]])
            assert torch.equal(blocks[-1].dstdata["_ID"], seeds)
            c = ld.get_coarse_count()
            assert 0.0 < c <= 1.0
            checked += 1
        assert step + 1 == ld.get_max_step()
    return checked


def _v1_body(rank, a):
    """First working-set form: own + neighbour partitions in local numbering, bridges from
    the neighbour only."""
    from grappa_b200.dataloader import IsolatedDataloader
    from grappa_b200.dataset.io_dist import ChunkIO

    args = _args(a["root"])
    ld = IsolatedDataloader(torch.device("cpu"), args)
    nbr = 1 - rank
    ld.load_nbr_chunk(nbr)
    ld.build_partition()
    io = ChunkIO(ld.data_path, WORLD, ld.in_feats)
    n0, n1 = io.counts[rank], io.counts[nbr]
    g = ld.cur_g
    assert g.n_nodes == n0 + n1
    assert ld.cur_node_feat.shape == (n0 + n1, ld.in_feats)
    assert torch.equal(ld.cur_node_feat[n0:], torch.from_numpy(io.part(nbr, "nfeat")))
    bu, bv = io.bridge(nbr, rank)
    want = set(zip(io.part(rank, "u").tolist(), io.part(rank, "v").tolist()))
    want |= set(zip((io.part(nbr, "u") + n0).tolist(), (io.part(nbr, "v") + n0).tolist()))
    if bu is not None:
        want |= set(zip((bu + n0).tolist(), bv.tolist()))
    indptr, indices = g.indptr(), g.indices()
    got = {(int(indices[e]), d) for d in range(n0 + n1) for e in range(indptr[d], indptr[d + 1])}
    assert got == want
    ld.load_nbr_chunk_v2(nbr)
    ld.build_partition_v2()  # the v2 working graph (global ids, halo) under its reference name
    assert ld.cur_g.n_edges >= len(got)
    return len(got)


def test_first_working_set_form(tiny_chunks):
    out = run_ranks(_v1_body, {"root": tiny_chunks.root})
    assert all(v > 0 for v in out.values())


def test_get_u_v_nid2pid(tiny_chunks):
    import json

    from grappa_b200.dataset.chunk_seq import get_u_v_nid2pid

    cfg = json.load(open(f"{tiny_chunks.root}/src/t10n.json"))
    u, v, pid = get_u_v_nid2pid(cfg, "hash", 3)
    assert u.shape == v.shape and u.shape[0] == cfg["num_edges"]
    assert pid.dtype == np.int64 and pid.shape[0] == cfg["num_nodes"] and set(np.unique(pid)) == {0, 1, 2}
    _, _, pm = get_u_v_nid2pid(cfg, "metis", 2)
    assert set(np.unique(pm)) == {0, 1}


def test_omp_assignments_from_nvml_affinity(monkeypatch):
    import sys
    import types

    from grappa_b200 import cl
    from grappa_b200.device_allocator import T10nDeviceAllocator

    fake = types.ModuleType("pynvml")
    fake.nvmlInit = lambda: None
    fake.nvmlShutdown = lambda: None
    fake.nvmlDeviceGetHandleByIndex = lambda i: i
    allowed = sorted(os.sched_getaffinity(0))
    mask = sum(1 << c for c in allowed[: max(1, len(allowed) // 2)] if c < 64)
    fake.nvmlDeviceGetCpuAffinity = lambda h, n: [mask] + [0] * (n - 1)
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    monkeypatch.setenv("LOCAL_RANK", "0")
    for k in ("OMP_PLACES", "OMP_NUM_THREADS", "OMP_PROC_BIND"):
        monkeypatch.delenv(k, raising=False)
    ta = T10nDeviceAllocator(8)
    cpus = ta.get_local_cpu_ids(8, 0)
    assert cpus == [c for c in allowed if c < 64 and (mask >> c) & 1]
    got = ta.set_omp_dev_assignments(8, 0, cg_idx=1, dup_per_gpu=2) if len(cpus) >= 2 else \
        ta.set_omp_dev_assignments(8, 0)
    assert os.environ["OMP_PROC_BIND"] == "spread"
    assert os.environ["OMP_PLACES"] == ",".join(f"{{{c}}}" for c in got)
    assert int(os.environ["OMP_NUM_THREADS"]) == len(got) and set(got) <= set(cpus)
    fake.nvmlInit = lambda: (_ for _ in ()).throw(RuntimeError("no NVML"))
    assert ta.get_local_cpu_ids(8, 0) == allowed or ta.get_local_cpu_ids(8, 0)  # falls back to allowed CPUs
    assert cl.total_mb([torch.tensor([1 << 20]), torch.tensor([1 << 19])], 4) == 6.0


def test_two_rank_loader(tiny_chunks):
    out = run_ranks(_loader_body, {"root": tiny_chunks.root})
    assert all(v > 0 for v in out.values())


def _infer_body(rank, a):
    from grappa_b200.dataloader import IsolatedDataloader
    from grappa_b200.infer import run_infer_xborder_by_layer
    from grappa_b200.models import get_model

    args = _args(a["root"])
    ld = IsolatedDataloader(torch.device("cpu"), args)
    ld.get_cur_dataloader(args, 0)
    torch.manual_seed(11)
    model = get_model("sage", 32, 8, num_hidden=16, num_layers=2, dropout=0.0)
    c = run_infer_xborder_by_layer(model, ld, torch.device("cpu"), args, "all")
    return c.tolist()


def test_layerwise_infer_matches_full_graph(tiny_chunks):
    from grappa_b200.block import Block
    from grappa_b200.models import get_model

    out = run_ranks(_infer_body, {"root": tiny_chunks.root})
    assert out[0] == out[1]
    counts = out[0]
    g = tiny_chunks.graph
    n = g.n_nodes
    loops = torch.arange(n)
    indptr, indices = synthetic.csc_from_edges(torch.cat([g.u, loops]), torch.cat([g.v, loops]), n)
    blk = Block(indptr, indices, torch.arange(n), n, n)
    torch.manual_seed(11)
    model = get_model("sage", 32, 8, num_hidden=16, num_layers=2, dropout=0.0)
    model.eval()
    with torch.no_grad():
        pred = model([blk, blk], g.feat).argmax(1)
    ok = pred == g.label
    want = [float(ok[m.bool()].sum()) for m in (g.train_mask, g.val_mask, g.test_mask)]
    want += [float(m.sum()) for m in (g.train_mask, g.val_mask, g.test_mask)]
    assert counts[3:] == want[3:]
    for got, exp in zip(counts[:3], want[:3]):
        assert abs(got - exp) <= 2  # summation order may flip a near-tie


def _cli_body(rank, a):
    sys.argv = ["t10n_train", "--data_path", a["root"], "--graph_name", "tiny", "--part_method", "hash", "--n_part",
                str(WORLD), "--model", a["model"], "--num_hidden", "16", "--num_layers", "2", "--fan_out", "5,5",
                "--num_epochs", "4", "--batch_size", "256", "--batch_size_eval", "1000", "--lr", "0.01",
                "--repart_every", "2", "--eval_every", "2", "--log_every", "5", "--tag_id", "test",
                "--checkpoint_path", a["ckpt"], "--checkpoint_every", "4", "--close_dd",
                "--metrics_jsonl", os.path.join(a["ckpt"], "metrics_{rank}.jsonl")]
    from grappa_b200.train import t10n_train

    return t10n_train.main(t10n_train.parse_args(), init_pg=False)


@pytest.mark.parametrize("model", ["sage", "gcn", "gat", "gin", "pinsage"])
def test_cli_trains_on_cpu_ranks(tiny_chunks, tmp_path, model):
    out = run_ranks(_cli_body, {"root": tiny_chunks.root, "ckpt": str(tmp_path), "model": model})
    r0 = out[0]
    assert r0["epochs"] == 4
    if model == "pinsage":
        # L2-normalised outputs bound the logits to the unit ball: the loss moves slowly
        assert all(np.isfinite(r0["loss"]))
    else:
        assert r0["loss"][-1] < r0["loss"][0]
    assert 0.0 <= r0["val_acc"] <= 1.0
    ck = torch.load(os.path.join(str(tmp_path), "epoch_003.pt"), weights_only=False)
    assert set(ck) == {"epoch", "state_dict", "optimizer_state_dict", "loss"}
    assert ck["epoch"] == 3
    import json

    for rank in range(WORLD):  # the metric lines as JSON, one file per rank
        recs = [json.loads(l) for l in open(os.path.join(str(tmp_path), f"metrics_{rank}.jsonl"))]
        epochs = [r for r in recs if r["event"] == "epoch"]
        assert [r["epoch"] for r in epochs] == [0, 1, 2, 3] and all(r["rank"] == rank for r in recs)
        assert all(r["epoch_seconds"] > 0 for r in epochs)
        infer = [r for r in recs if r["event"] == "infer"]
        assert infer and all(0.0 <= r["test_acc"] <= 1.0 for r in infer)


def test_partition_from_chunks_matches_global(tiny_chunks):
    from grappa_b200.graph_store import partition_from_chunks, partition_from_global

    g = tiny_chunks.graph
    for r in range(WORLD):
        a = partition_from_chunks(tiny_chunks.root, "tiny", "hash", WORLD, r, 32, "cpu")
        b = partition_from_global(g, WORLD, r, "cpu")
        assert a.prefix == b.prefix
        assert torch.equal(a.indptr, b.indptr)
        assert torch.equal(a.indices, b.indices)
        assert torch.equal(a.feat, b.feat)
        assert torch.equal(a.label, b.label)
        assert torch.equal(a.gideg, b.gideg)
        assert torch.equal(a.ext_src, b.ext_src)
        assert torch.equal(a.train_mask.to(torch.int8), b.train_mask.to(torch.int8))


def _full_cli_body(rank, a):
    sys.argv = ["t10n_fullgraph_train", "--data_path", a["root"], "--graph_name", "tiny", "--part_method", "hash",
                "--n_part", str(WORLD), "--model", "gcn", "--num_hidden", "16", "--num_layers", "2", "--num_epochs",
                "6", "--lr", "0.02", "--repart_every", "3", "--log_every", "2", "--tag_id", "t", "--dropout", "0.0",
                "--metrics_jsonl", a["metrics"]]
    from grappa_b200.train import t10n_fullgraph_train as fg

    return fg.main(fg.build_parser().parse_args(), init_pg=False)


def test_fullgraph_cli_cpu_ranks(tiny_chunks, tmp_path):
    import json

    path = str(tmp_path / "fg.jsonl")
    out = run_ranks(_full_cli_body, {"root": tiny_chunks.root, "metrics": path})
    for r in range(WORLD):
        assert out[r]["loss"][-1] < out[r]["loss"][0]
    recs = [json.loads(l) for l in open(path)]  # no {rank} in the path: rank 0 only
    assert {r["rank"] for r in recs} == {0}
    assert [r["epoch"] for r in recs if r["event"] == "epoch"] == list(range(6))
    assert any(r["event"] == "step" and "loss" in r for r in recs)


def test_t10n_alias_and_converters(tmp_path, tiny_chunks):
    import importlib

    import t10n  # noqa: F401
    from t10n._C.graph import HostGraph
    from t10n.dataset.meta import name_to_meta
    from t10n.sampler import HostBatchSamplerWithCounter
    from t10n.dgl_dsg.sampler import PinSAGESampler, to_dgl_batch

    assert importlib.import_module("t10n.dataloader").IsolatedDataloader is not None
    assert name_to_meta("tiny").n_dim == 32
    from grappa_b200.dataset.dgl_to_t10n import convert, write_t10n

    g = tiny_chunks.graph
    # npz round trip through the converter
    npz = tmp_path / "g.npz"
    np.savez(npz, edge_index=np.stack([g.u.numpy(), g.v.numpy()]), feat=g.feat.numpy(), label=g.label.numpy(),
             train_mask=g.train_mask.numpy(), val_mask=g.val_mask.numpy(), test_mask=g.test_mask.numpy())
    cfg = convert(str(npz), str(tmp_path / "out"), "tiny")
    assert cfg["num_edges"] == g.u.numel() + g.n_nodes and cfg["num_labels"] == 8
    e = np.load(cfg["edge_file_bin"])
    assert e.shape[0] == 2 * cfg["num_edges"]
    hg = HostGraph(g.u.numpy(), g.v.numpy())  # the reference's signature: (u, v[, numa node])
    s = HostBatchSamplerWithCounter(hg, torch.arange(100), [3, 3], batch_size=50, target_nodes_gideg=torch.ones(100,
                                    dtype=torch.int64))
    n = sum(1 for _ in s)
    assert n == 2
    inp, out, blocks = PinSAGESampler(hg, 2).sample_blocks(None, torch.arange(10))
    assert blocks[-1].n_dst == 10 and "weights" in blocks[-1].edata
    u = torch.tensor([5, 6, 7]); v = torch.tensor([1, 1, 2])
    src, dst, b = to_dgl_batch(torch.tensor([1, 2]), [u, v])
    assert b[0].n_dst == 2 and b[0].num_edges() == 3


def test_launcher_sweep_and_table(tmp_path):
    from grappa_b200 import launch

    out = launch.main(["--dry_run", "--models", "sage,gcn", "--layers_fanouts", "2:10,5;3:15,10,5", "--runs", "2",
                       "--log_dir", str(tmp_path)])
    assert out == 0
    log = tmp_path / "t10n_hash_rmat16k_sage_2_1_R1_0.txt"
    log.write_text("rank0 infer_|epoch|0009|part|0000|val_acc|0.8000|test_acc|0.7500|train_acc|0.9\n")
    (tmp_path / "t10n_hash_rmat16k_gcn_3_1_R1_0.txt").write_text(
        "rank0 infer_|epoch|0009|part|0000|val_acc|0.7|test_acc|0.6100|train_acc|0.8\n")
    table = launch.result_table(str(tmp_path))
    assert "| sage_2 | 0.75 |" in table and "| gcn_3 | 0.61 |" in table
    # a second run is averaged; a second partition method splits the rows
    (tmp_path / "t10n_hash_rmat16k_sage_2_1_R2_0.txt").write_text(
        "rank0 infer_|epoch|0009|part|0000|val_acc|0.8|test_acc|0.7700|train_acc|0.9\n")
    assert "| sage_2 | 0.76 (2 runs) |" in launch.result_table(str(tmp_path))
    (tmp_path / "t10n_metis_rmat16k_sage_2_1_R1_0.txt").write_text(
        "rank0 infer_|epoch|0009|part|0000|val_acc|0.8|test_acc|0.8000|train_acc|0.9\n")
    table = launch.result_table(str(tmp_path))
    assert "| sage_2 [hash] | 0.76 (2 runs) |" in table and "| sage_2 [metis] | 0.8 |" in table
