"""Cross-partition helpers (reference: t10n/xborder.py:9-167).

``XBorder`` is the C++ helper (grappa_b200/csrc/host/xborder.cc).  ``xb_gather``
fetches rows (features or embeddings) of arbitrary global ids owner-computes
style: ids are grouped by owner and exchanged, every owner gathers the requested
rows from its shard and sends them back (two ragged all-to-alls).  With NCCL/gloo
that is the CPU path; when ``comm_dev`` is a ``grappa_b200.cl.PeerAllToAll`` both
exchanges run through NVLink peer memory (``xb_gather_peer``).  Exact layer-wise
inference on GPUs skips the id exchange altogether: the global id names the owner
and the row, so it pulls the rows straight from the owners' tables
(grappa_b200/csrc/cuda/peer.cu, pull_rows; grappa_b200.infer_gpu.ExactInference).
"""
import torch

from grappa_b200 import _native
from grappa_b200.cl import t10n_all_to_all_1d_int64_nccl as t10n_all_to_all_1d_int64
from grappa_b200.cl import t10n_all_to_all_2d_float32_nccl as t10n_all_to_all_2d_float32

XBorder = _native.host().xborder.XBorder


def xb_mask_by_partition(xb, ids_th, n_part):
    mask = torch.empty([n_part, ids_th.shape[0]], dtype=torch.int8)  # every entry written
    xb.mask_by_partition(ids_th.cpu().numpy(), mask.numpy())
    return mask


def xb_group_by_partition_v1(xb, ids_th, n_part):
    mask = xb_mask_by_partition(xb, ids_th, n_part)
    return [ids_th[torch.nonzero(mask[i]).flatten()] for i in range(n_part)], mask


def xb_group_by_partition(xb, ids_th, n_part):
    mask = torch.empty([n_part, ids_th.shape[0]], dtype=torch.int8)  # every entry written
    groups = xb.group_by_partition(ids_th.cpu().numpy(), mask.numpy())
    return [torch.from_numpy(g) for g in groups], mask


def xb_ad_hoc_fill_batch_feat(xb, device, input_nodes, local_feat_n, rank, nbr_idx, n_part, prefix_sum):
    """Rows of ``input_nodes`` from the own partition, the neighbour partition and the halo
    cache (tables indexed by partition id; halo tables are in the order given to
    ``ad_hoc_build_id_mapping``)."""
    dim = next(t.shape[1] for t in local_feat_n if t is not None)
    out = torch.zeros((input_nodes.shape[0], dim), dtype=torch.float32)
    tables = [None if t is None else t.contiguous().numpy() for t in local_feat_n]
    xb.ad_hoc_fill_batch_feat(out.numpy(), tables, input_nodes.cpu().numpy())
    return out.to(device)


def _group_by_owner(ids, prefix_sum, world_size):
    """(ids sorted by owner, the sort order, per-owner counts) on the ids' device."""
    bounds = torch.tensor(prefix_sum[1:], dtype=torch.int64, device=ids.device)
    owner = torch.bucketize(ids, bounds, right=True)
    order = torch.argsort(owner, stable=True)
    counts = torch.bincount(owner, minlength=world_size).cpu().tolist()
    return ids[order], order, counts


def xb_gather_peer(a2a, batch_input, target_nodes, emb_self, rank, world_size, prefix_sum):
    """GPU form of ``xb_gather``: the ids grouped by owner go to the owners and the owners'
    rows come back, both through the peer-memory all-to-all ``a2a``."""
    dev = emb_self.device
    ids = target_nodes.to(dev).long()
    sorted_ids, order, counts = _group_by_owner(ids, prefix_sum, world_size)
    requests = a2a.exchange(list(torch.split(sorted_ids, counts)))
    lo = prefix_sum[rank]
    replies = [emb_self[(q.long() - lo)].contiguous() for q in requests]
    rows = a2a.exchange(replies)
    got = torch.cat(rows) if rows else emb_self[:0]
    out = torch.empty((ids.numel(),) + tuple(emb_self.shape[1:]), dtype=emb_self.dtype, device=dev)
    out[order] = got
    cols = batch_input.shape[1] if batch_input.dim() > 1 else None
    batch_input.copy_((out[:, :cols] if cols is not None else out).to(batch_input.device, batch_input.dtype))
    return batch_input


def xb_gather(xb, comm_dev, batch_input, target_nodes, emb_self, rank, world_size, prefix_sum):
    """batch_input[i] = row of global id target_nodes[i], fetched from its owner."""
    from grappa_b200.cl import PeerAllToAll

    if isinstance(comm_dev, PeerAllToAll):
        return xb_gather_peer(comm_dev, batch_input, target_nodes, emb_self, rank, world_size, prefix_sum)
    groups, mask = xb_group_by_partition(xb, target_nodes, world_size)
    own_idx = torch.nonzero(mask[rank]).flatten()
    if own_idx.numel():
        batch_input[own_idx] = emb_self[(groups[rank] - prefix_sum[rank]).to(emb_self.device)].to(batch_input.device)
    requests = t10n_all_to_all_1d_int64(groups, rank, world_size, device=comm_dev)
    replies = []
    for p, gids in enumerate(requests):
        if p == rank or gids.shape[0] == 0:
            replies.append(torch.zeros((0, emb_self.shape[1]), dtype=torch.float32))
        else:
            replies.append(emb_self[(gids - prefix_sum[rank]).to(emb_self.device)].float())
    rows = t10n_all_to_all_2d_float32(replies, rank, world_size, device=comm_dev, dim_2nd=emb_self.shape[1])
    for p in range(world_size):
        if p == rank:
            continue
        idx = torch.nonzero(mask[p]).flatten()
        if idx.numel():
            batch_input[idx] = rows[p].to(batch_input.device, batch_input.dtype)
    return batch_input


def xb_scatter(xb, comm_dev, target_nodes_emb, target_nodes, emb_self, rank, world_size, prefix_sum):
    """emb_self[id] = row for the ids this rank owns; rows of other owners are sent to them."""
    groups, mask = xb_group_by_partition(xb, target_nodes, world_size)
    payload = [target_nodes_emb[torch.nonzero(mask[p]).flatten()].float() for p in range(world_size)]
    ids = t10n_all_to_all_1d_int64(groups, rank, world_size, device=comm_dev)
    rows = t10n_all_to_all_2d_float32(payload, rank, world_size, device=comm_dev, dim_2nd=emb_self.shape[1])
    for p in range(world_size):
        if ids[p].numel():
            emb_self[(ids[p] - prefix_sum[rank]).to(emb_self.device)] = rows[p].to(emb_self.device, emb_self.dtype)
    return emb_self


def __getattr__(name):
    # the reference declares MiniBatchXborderSampler as an empty class (t10n/xborder.py:165-167);
    # here the name gives the cross-partition mini-batch sampler (imported late: it imports this module)
    if name == "MiniBatchXborderSampler":
        from grappa_b200.xbsampler import HostXBBatchSampler

        return HostXBBatchSampler
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
