"""Cross-partition inference (reference: t10n/infer.py:14-198).

``run_infer_xborder``: mini-batch inference where the sampled neighbourhood may
cross partitions (xbsampler), input rows fetched from their owners.

``run_infer_xborder_by_layer``: exact layer-wise inference.  For every layer, each
rank computes the embeddings of its own nodes from the full in-neighbourhood
(layer 0 reads features from the working partition's tables, later layers fetch
the previous layer's embeddings of remote sources from their owners), so that
the last layer's logits of every node are those of the full graph.  Hidden
layers are computed for every node, not only for ``subset_tag`` (the reference
restricts every layer to the subset, so neighbours outside it read zeros,
t10n/infer.py:106-108).  Accuracy
counts are all-reduced: [train_ok, valid_ok, test_ok, train_n, valid_n, test_n].

Layers run on the tensors' device: the PyTorch path on CPU tensors, the sm_100a
layer kernels (grappa_b200.infer_gpu.infer_layer) on CUDA tensors.
"""
import gc

import torch
import torch.nn.functional as F

from grappa_b200.util import pprint


def infer_sync_count(device, train_yes_n, valid_yes_n, test_yes_n, train_n, valid_n, test_n):
    c = torch.tensor([float(train_yes_n), float(valid_yes_n), float(test_yes_n), float(train_n), float(valid_n),
                      float(test_n)], device=device)
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(c)
    return c


def get_inc_count(batch_pred, batch_labels, mask):
    idx = torch.nonzero(mask.to(batch_pred.device)).flatten()
    pred = batch_pred[idx]
    lab = batch_labels.to(batch_pred.device)[idx].long()
    return idx.shape[0], float((torch.argmax(pred, dim=1) == lab).float().sum())


def apply_layer(model, layer_i, block, h):
    """One layer of ``model`` plus its inter-layer activation (eval mode: no dropout)."""
    last = layer_i == len(model.layers) - 1
    if h.is_cuda:
        from grappa_b200.infer_gpu import infer_layer

        return infer_layer(model, layer_i, block, h)
    layer = model.layers[layer_i]
    h_dst = h[: block.num_dst_nodes()]
    if model.name == "gat":
        h = layer(block, (h, h_dst))
        return h.mean(1) if last else model.activation(h.flatten(1))
    if model.name in ("sage", "gcn"):
        h = layer(block, (h, h_dst)) if model.name == "sage" else layer(block, h)
        return h if last else model.activation(h)
    if model.name == "gin":
        h = layer(block, (h, h_dst))
        return F.relu(model.batch_norms[layer_i](h))
    if model.name == "pinsage":
        w = block.edata.get("weights")
        if w is None:
            w = torch.ones(block.num_edges(), dtype=torch.float32)
        return layer(block, (h, h_dst), w)
    raise ValueError(f"{model.name} is not supported")


def _out_dim(model, layer_i):
    layer = model.layers[layer_i]
    if model.name == "gat":
        return layer.out_feats * (layer.num_heads if layer_i != len(model.layers) - 1 else 1)
    if model.name == "gin":
        return model.batch_norms[layer_i].num_features
    if model.name == "pinsage":
        return layer.output_dims
    return layer.out_feats


def run_infer_xborder(model, isloader, device, args, subset_tag):
    model.eval()
    loader = isloader.xb_dataloader(args, force_even=True, full_neighbor=False, subset_tag=subset_tag)
    counts = [0, 0, 0, 0, 0, 0]
    with torch.no_grad():
        for input_nodes, seeds, blocks in loader:
            labels = isloader.get_batch_labels(seeds)
            x = torch.zeros([input_nodes.shape[0], isloader.in_feats], dtype=torch.float32,
                            device=isloader.da.comm_dev())
            isloader.xb_get_batch_input(x, input_nodes)
            blocks = [b.to(device) for b in blocks]
            h = x.to(device)
            for i, block in enumerate(blocks):
                h = apply_layer(model, i, block, h)
            for k, (tag, fn) in enumerate((("train", isloader.infer_train_mask_of),
                                          ("valid", isloader.infer_valid_mask_of),
                                          ("test", isloader.infer_test_mask_of))):
                if subset_tag in ("all", tag):
                    n, ok = get_inc_count(h, labels, fn(seeds))
                    counts[k] += ok
                    counts[k + 3] += n
    model.train()
    return infer_sync_count(isloader.get_comm_dev(), *counts)


def run_infer_xborder_by_layer(model, isloader, device, args, subset_tag):
    model.eval()
    n_local = isloader.get_num_node()
    off = isloader.get_nid_offset()
    with torch.no_grad():
        y = None
        for layer_i in range(len(model.layers)):
            gc.collect()
            pprint(isloader.rank, f"infer:layer_{layer_i}")
            y_next = torch.zeros([n_local, _out_dim(model, layer_i)], dtype=torch.float32, device=device)
            # hidden layers need every node's embedding (the next layer reads all in-neighbours)
            tag = subset_tag if layer_i == len(model.layers) - 1 else "all"
            for input_nodes, output_nodes, blocks in isloader.xb_dataloader_per_layer(args, subset_tag=tag):
                block = blocks[0].to(device)
                if layer_i == 0:
                    x = torch.zeros([input_nodes.shape[0], isloader.in_feats], dtype=torch.float32,
                                    device=isloader.da.part_feat_dev())
                    isloader.get_batch_input(x, input_nodes)
                else:
                    x = torch.zeros([input_nodes.shape[0], y.shape[1]], dtype=torch.float32, device=y.device)
                    isloader.xb_get_batch_emb(x, input_nodes, y)
                if output_nodes.numel() == 0:
                    continue
                h = apply_layer(model, layer_i, block, x.to(device))
                y_next[(output_nodes - off).to(device)] = h.float()
            y = y_next
    model.train()
    truth = isloader.node_label.to(device)
    counts = [0, 0, 0, 0, 0, 0]
    for k, (tag, mask) in enumerate((("train", isloader.train_mask), ("valid", isloader.valid_mask),
                                     ("test", isloader.test_mask))):
        if subset_tag in ("all", tag):
            n, ok = get_inc_count(y, truth, mask)
            counts[k] += ok
            counts[k + 3] += n
    return infer_sync_count(isloader.get_comm_dev(), *counts)
