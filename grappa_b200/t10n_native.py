"""The reference's native module API (``t10n._C``; csrc/python/pybind11.cc:59-130) with
its class names and call signatures, over this package's host engine (grappa_b200._C).
The ``t10n`` package serves ``t10n._C.graph``, ``.xborder``, ``.c_seq`` and ``.c_dist``
from here; every name of the engine's own submodules is there as well.

Where the signatures differ from the engine's:

* ``HostGraph(u, v[, node_id])``: the third argument is the NUMA node of the CSC (the
  engine's third argument is the node count);
* ``HostSampler.c_next_batch()`` returns a ``Batch`` (``get_layers()``: per hop the
  sampled sources and their destinations, seed hop first; ``get_input_nodes()``: per hop
  the distinct sampled sources, ascending);
* ``HostNeighborSampler(g, repeated).c_next_batch_py(seeds, fanout)``: one hop as
  ``([u, v], [])``;
* ``GpuGraph(host_graph)``: the CSC in device memory (``indptr``, ``indices`` tensors);
* ``XBorder.ad_hoc_fill_batch_feat_v2(out, feat_n, ids, batch_idx)``: row i of ``ids``
  goes to ``out[batch_idx[i]]``;
* ``c_dist.random_assign_pid(rank, local_slice, num_part)`` fills an int32 slice in
  place with the partition of global ids ``rank * len + i`` (the engine's seeded hash:
  the reference draws them from an unseeded generator); the engine's
  ``random_assign_pid(n, n_part, seed)`` form is accepted too;
* ``py_test_batch()``: the reference's fixture filled as it meant to (its fill takes the
  vectors by value, so it returns zeros): layers [0..2], [0..4], [0..2], [0..4] and input
  nodes [0], [0, 1].

The reference's ``GpuSampler`` is an empty stub (csrc/python/py_graph.h:117-122) and has
no counterpart here; the device sampler is grappa_b200.sampler_gpu.GpuNeighborSampler.
"""
import types

import numpy as np
import torch

from grappa_b200 import _native


def _C():
    return _native.host()


class Batch:
    """One sampled batch: ``layers`` = [u_hop0, v_hop0, u_hop1, v_hop1, ...] (graph ids,
    seed hop first), ``input_nodes`` = the distinct sources of every hop, ``resampling``
    = [coverage sum, seeds counted] when the sampler counts coverage."""

    def __init__(self, layers=(), input_nodes=(), resampling=()):
        self.layers = [np.asarray(x, dtype=np.int64) for x in layers]
        self.input_nodes = [np.asarray(x, dtype=np.int64) for x in input_nodes]
        self.resampling = np.asarray(resampling, dtype=np.float32)

    def get_layers(self):
        return [x.tolist() for x in self.layers]

    def get_input_nodes(self):
        return [x.tolist() for x in self.input_nodes]


def py_test_batch():
    a = lambda n: np.arange(n, dtype=np.int64)  # noqa: E731
    return Batch([a(3), a(5), a(3), a(5)], [a(1), a(2)])


class HostGraph:
    """``HostGraph(u, v)`` or ``HostGraph(u, v, node_id)`` -> the engine's HostGraph (node
    count = max id + 1; with node_id its arrays are placed on that NUMA node)."""

    def __new__(cls, u, v, node_id=-1):
        return _C().graph.HostGraph(np.ascontiguousarray(u, dtype=np.int64), np.ascontiguousarray(v, dtype=np.int64),
                                    -1, int(node_id))


def _host_sampler_class():
    native = _C().graph.HostSampler

    class HostSampler(native):
        """The engine's pipelined sampler with the reference's ``c_next_batch``."""

        def c_next_batch(self):
            layers, correct = self.c_next_batch_py()
            inputs = [np.unique(np.asarray(layers[2 * h])) for h in range(len(layers) // 2)]
            return Batch(layers, inputs, correct)

    return HostSampler


class HostNeighborSampler:
    """One-hop sampling of given seeds (reference: csrc/python/py_graph.h:124-134)."""

    def __init__(self, g, repeated=False):
        self.g, self.repeated = g, bool(repeated)
        self._step = 0

    def c_next_batch_py(self, seeds, fanouts):
        seeds = np.ascontiguousarray(seeds, dtype=np.int64)
        if self.repeated:
            blocks, _, _ = _C().graph.sample_batch(self.g, [int(fanouts)], seeds, None, 0, 0, self._step, True)
            b = blocks[0]
            src, ip, ix = b["src_nid"], b["indptr"], b["indices"]
            u = src[ix]
            v = np.repeat(seeds, np.diff(ip))
        else:
            u, v = _C().graph.sample_neighbors(self.g, seeds, int(fanouts), self._step)
        self._step += 1
        return [np.asarray(u, dtype=np.int64), np.asarray(v, dtype=np.int64)], np.zeros(0, dtype=np.float32)


class GpuGraph:
    """The CSC of a HostGraph in device memory (reference: csrc/python/py_graph.h:41-50).
    ``device`` defaults to the current CUDA device."""

    def __init__(self, host_graph, device=None):
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.n_nodes = int(host_graph.n_nodes)
        self.indptr = torch.from_numpy(np.asarray(host_graph.indptr())).to(dev)
        self.indices = torch.from_numpy(np.asarray(host_graph.indices())).to(dev)


def _xborder_class():
    native = _C().xborder.XBorder

    class XBorder(native):
        def ad_hoc_fill_batch_feat_v2(self, batch_feat, feat_n, ids, batch_idx):
            return self.ad_hoc_fill_batch_feat(batch_feat, feat_n, ids, batch_idx)

    return XBorder


def random_assign_pid(*args, **kwargs):
    """``(rank, local_slice, num_part)`` (the reference's in-place form) or
    ``(n, n_part, seed=0)`` (the engine's)."""
    if len(args) == 3 and isinstance(args[1], np.ndarray) and not kwargs:
        rank, local, num_part = int(args[0]), args[1], int(args[2])
        gids = rank * local.shape[0] + np.arange(local.shape[0], dtype=np.int64)
        local[...] = _C().graph.hash_part(gids, 0, num_part).astype(local.dtype)
        return None
    return _C().c_dist.random_assign_pid(*args, **kwargs)


def _wrap(native_mod, name, overrides):
    mod = types.ModuleType(name, native_mod.__doc__)
    for k in dir(native_mod):
        if not k.startswith("__"):
            setattr(mod, k, getattr(native_mod, k))
    for k, v in overrides.items():
        setattr(mod, k, v)
    return mod


def build_modules(prefix="t10n._C"):
    """{submodule name: module} with the reference's API over the engine's."""
    C = _C()
    return {
        "graph": _wrap(C.graph, f"{prefix}.graph", {
            "Batch": Batch, "py_test_batch": py_test_batch, "HostGraph": HostGraph,
            "HostSampler": _host_sampler_class(), "HostNeighborSampler": HostNeighborSampler, "GpuGraph": GpuGraph}),
        "xborder": _wrap(C.xborder, f"{prefix}.xborder", {"XBorder": _xborder_class()}),
        "c_seq": _wrap(C.c_seq, f"{prefix}.c_seq", {}),
        "c_dist": _wrap(C.c_dist, f"{prefix}.c_dist", {"random_assign_pid": random_assign_pid}),
    }
