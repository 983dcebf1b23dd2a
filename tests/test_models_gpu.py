"""GPU engines of every model family (GCN, GIN, GAT, PinSAGE; SAGE is covered in
test_engine_gpu.py) against the PyTorch fp32 models: one training step on the
sm_100a kernels versus the same model run on CPU over the identical blocks
(materialised from the GPU sampler), then a short training run per model, the
full-graph trainer and the GPU random-walk sampler's exact replay on the CPU."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from grappa_b200 import _native
from grappa_b200.block import Block
from grappa_b200.dataset import synthetic as S
from grappa_b200.graph_store import partition_from_global
from grappa_b200.models import get_model
from grappa_b200.trainer import FullGraphTrainer, MiniBatchTrainer

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def tiny():
    g = S.build(S.SPECS["tiny"], DEV)
    own = partition_from_global(g, 1, 0, DEV)
    return g, own


def _one_step_grads(trainer):
    eng = trainer.engine
    seeds, counts = trainer.epoch_seeds(0, on_host=False)
    eng.set_epoch(0)
    eng.load_seeds(seeds[0], counts[0])
    eng.cu.zero_(eng.fstats)
    eng.cu.zero_(eng.istats)
    eng._sample()
    eng._forward(True)
    eng._backward()
    torch.cuda.synchronize()
    eng.check_errors()
    n = int(counts[0, 0])
    return float(eng.fstats[2]), eng.grad.clone().cpu(), seeds[0, :n].long().cpu()


CASES = [
    ("gcn", dict(num_hidden=64, num_layers=3), [10, 10, 5]),   # agg-first hidden layers, projection-first last
    ("gcn", dict(num_hidden=16, num_layers=2), [10, 5]),       # projection-first on gathered inputs
    ("gin", dict(num_hidden=64, num_layers=3), [10, 10, 5]),
    ("gat", dict(num_hidden=16, num_layers=3, n_heads=4), [10, 10, 5]),
    ("gat", dict(num_hidden=24, num_layers=2, n_heads=3), [10, 5]),  # heads straddling 8-column chunks
    ("pinsage", dict(num_hidden=64, num_layers=3), None),
]


@pytest.mark.parametrize("name,kw,fanouts", CASES)
def test_engine_step_matches_cpu_model(tiny, name, kw, fanouts):
    g, own = tiny
    torch.manual_seed(0)
    model = get_model(name, g.spec.feat_dim, g.spec.n_classes, dropout=0.0, **kw)
    cpu_model = get_model(name, g.spec.feat_dim, g.spec.n_classes, dropout=0.0, **kw)
    cpu_model.load_state_dict(model.state_dict())
    L = kw["num_layers"]
    trainer = MiniBatchTrainer(model, own, fanouts or [5] * L, 128, comm=None, seed=5, use_cuda_graph=False)
    loss_gpu, grad_gpu, seeds = _one_step_grads(trainer)
    blocks = trainer.engine.sm.blocks()
    blocks = [b.to("cpu") for b in blocks]
    for b in blocks:
        b.indices = b.indices.long()
        b.indptr = b.indptr.long()
        b.srcdata["_ID"] = b.srcdata["_ID"].long()
    x = own.feat[:, : g.spec.feat_dim].float().cpu()[blocks[0].srcdata["_ID"]]
    cpu_model.train()
    flat_grad = cpu_model.flat_grad()
    out = cpu_model(blocks, x)
    loss = F.cross_entropy(out, own.label.long().cpu()[seeds])
    loss.backward()
    assert abs(loss_gpu - float(loss)) < 2e-2 * max(1.0, float(loss)), (loss_gpu, float(loss))
    rel = (grad_gpu - flat_grad).norm() / flat_grad.norm()
    # GIN: every layer runs two BatchNorm backward passes whose mean/projection removal
    # amplifies the bf16 rounding of the stored pre-activations; the error grows by a few
    # percent per layer towards the input (BatchNorm kernels alone: test_nn_kernels_gpu.py)
    tol = 0.15 if name == "gin" else 6e-2
    assert rel < tol, f"{name}: gradient relative error {rel:.3e}"
    if name == "gat":
        # the input layer's weight and attention gradients take their own kernel path
        for seg_name in ("layers.0.W", "layers.0.A", "layers.0.b"):
            seg = model.segment(seg_name)
            a, b = seg.view(grad_gpu), seg.view(flat_grad.detach())
            r = (a - b).norm() / b.norm().clamp(min=1e-12)
            assert r < 6e-2, f"gat {seg_name}: gradient relative error {r:.3e}"
    if name == "gin":
        # BatchNorm running statistics follow the batch statistics
        for a, b in zip(model.batch_norms, cpu_model.batch_norms):
            torch.testing.assert_close(a.running_mean.cpu(), b.running_mean, rtol=5e-2, atol=5e-2)
    trainer.close()


@pytest.mark.parametrize("name,kw,fanouts", CASES)
def test_training_reduces_loss(tiny, name, kw, fanouts):
    g, own = tiny
    torch.manual_seed(2)
    model = get_model(name, g.spec.feat_dim, g.spec.n_classes, dropout=0.2, **kw)
    L = kw["num_layers"]
    trainer = MiniBatchTrainer(model, own, fanouts or [5] * L, 256, comm=None, seed=1, lr=1e-2)
    trainer.warmup()
    first = trainer.train_epoch(0, host_feed=True)
    for e in range(1, 6):
        last = trainer.train_epoch(e, host_feed=True)
    trainer.engine.check_errors()
    acc = trainer.evaluate(own.val_mask)
    trainer.close()
    assert np.isfinite(last)
    if name != "pinsage":  # L2-normalised logits: the loss moves slowly
        assert last < first, (first, last)
        assert acc > 1.2 / g.spec.n_classes


def test_walk_sampler_replays_on_cpu(tiny):
    g, own = tiny
    from grappa_b200.engine import GpuWalkSampler
    from grappa_b200.sampler_gpu import new_counters

    sm = GpuWalkSampler(2, 64, own.n_nodes, DEV, length=3, num_walks=4, num_neighbors=5)
    seeds = torch.nonzero(own.train_mask).squeeze(1)[:64].to(torch.int32)
    sm.load_seeds(seeds)
    counters = new_counters(7, DEV)
    counters[1], counters[2] = 2, 3
    sm.sample(own.indptr, own.indices, counters)
    torch.cuda.synchronize()
    assert int(sm.err.item()) == 0
    blocks = sm.blocks()
    n = own.n_nodes
    v = torch.repeat_interleave(torch.arange(n), (own.indptr[1:] - own.indptr[:-1]).cpu())
    hg = _native.host().graph.HostGraph(own.indices.long().cpu().numpy(), v.numpy(), n)
    dst = seeds.long().cpu()
    for hop in range(2):
        key = int(_native.host().graph.hop_key(7, 2, 3, hop))
        d = _native.host().graph.random_walk_topk(hg, dst.numpy(), 3, 0.5, 4, 5, key)
        b = blocks[1 - hop]
        assert np.array_equal(d["indptr"], b.indptr.cpu().numpy())
        assert np.array_equal(d["src_nid"], b.srcdata["_ID"].cpu().numpy())
        assert np.array_equal(d["indices"], b.indices.cpu().numpy())
        assert np.allclose(d["weights"], b.edata["weights"].cpu().numpy())
        dst = torch.from_numpy(d["src_nid"])


def test_full_graph_gcn_matches_cpu(tiny):
    g, own = tiny
    torch.manual_seed(3)
    model = get_model("gcn", g.spec.feat_dim, g.spec.n_classes, num_hidden=64, num_layers=3, dropout=0.0)
    cpu_model = get_model("gcn", g.spec.feat_dim, g.spec.n_classes, num_hidden=64, num_layers=3, dropout=0.0)
    cpu_model.load_state_dict(model.state_dict())
    tr = FullGraphTrainer(model, own, comm=None, use_cuda_graph=False)
    eng = tr.engine
    eng.set_epoch(0)
    eng.cu.zero_(eng.fstats)
    eng.cu.zero_(eng.istats)
    eng._forward(True)
    eng._backward()
    torch.cuda.synchronize()
    eng.check_errors()
    loss_gpu = float(eng.fstats[2])
    grad_gpu = eng.grad.clone().cpu()
    n = own.n_nodes
    blk = Block(own.indptr.cpu(), own.indices.long().cpu(), torch.arange(n), n, n)
    x = own.feat[:, : g.spec.feat_dim].float().cpu()
    flat_grad = cpu_model.flat_grad()
    out = cpu_model([blk] * 3, x)
    tr_mask = own.train_mask.cpu().bool()
    loss = F.cross_entropy(out[tr_mask], own.label.long().cpu()[tr_mask])
    loss.backward()
    assert abs(loss_gpu - float(loss)) < 2e-2 * max(1.0, float(loss))
    rel = (grad_gpu - flat_grad).norm() / flat_grad.norm()
    assert rel < 6e-2, f"gradient relative error {rel:.3e}"
    # a few graph-replayed epochs reduce the loss
    tr2 = FullGraphTrainer(get_model("gcn", g.spec.feat_dim, g.spec.n_classes, num_hidden=64, num_layers=3,
                                     dropout=0.5), own, comm=None, lr=1e-2)
    first = tr2.train_epoch(0)
    for e in range(1, 10):
        last = tr2.train_epoch(e)
    assert last < first
    assert tr2.evaluate(own.val_mask) > 1.2 / g.spec.n_classes
    tr.close()
    tr2.close()
