"""GPU-serving data loader on one GPU: chunk files -> HBM partition -> device
sampling; blocks carry global ids and the gathered features match the chunk files."""
import numpy as np
import pytest
import torch
from types import SimpleNamespace

from grappa_b200.dataset import synthetic as S
from grappa_b200.dataset.chunk_seq import build_chunks_seq

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_gpu_loader_epoch(tmp_path):
    from grappa_b200.dataloader_gpu import IsolatedDataloaderGPU

    g = S.build("tiny")
    S.to_t10n_layout(g, str(tmp_path / "src"))
    out, _ = build_chunks_seq(str(tmp_path), "tiny", str(tmp_path / "src"), "hash", 1)
    args = SimpleNamespace(graph_name="tiny", backend="nccl", n_part=1, data_path=str(tmp_path), part_method="hash",
                           batch_size=256, fan_out="5,5", repart_every=2, seed=1)
    ld = IsolatedDataloaderGPU(DEV, args)
    oid = np.fromfile(f"{out}/p0.oid.bin", dtype=np.int64)
    feat = torch.from_numpy(np.load(str(tmp_path / "src" / "node_feat.bin.npy"))).to(DEV)
    n_steps = 0
    for input_nodes, seeds, blocks in ld.get_cur_dataloader(args, 0):
        assert torch.all(ld.train_mask[seeds] == 1)
        assert torch.equal(blocks[-1].dstdata["_ID"].long(), seeds.to(DEV))
        x = torch.zeros((input_nodes.numel(), 32), device=DEV)
        ld.get_batch_input(x, input_nodes)
        ref = feat[torch.from_numpy(oid).to(DEV)[input_nodes.long()]]
        torch.testing.assert_close(x, ref.to(torch.bfloat16).float())
        assert 0.0 < ld.get_coarse_count() <= 1.0
        n_steps += 1
    assert n_steps == ld.get_max_step()
    blk = ld.full_neighbor_block(seeds)
    assert blk.n_dst == seeds.numel()
    deg = (ld.own.indptr[1:] - ld.own.indptr[:-1])[seeds.to(DEV)]
    assert torch.equal(blk.in_degrees().cpu(), deg.cpu())
    ld.close()
