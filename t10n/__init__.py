"""The reference's package name (``t10n``) over this framework.

Code written against mpi-dsg/grappa imports ``t10n.dataloader``, ``t10n.sampler``,
``t10n._C.graph`` and so on (t10n/__init__.py, t10n/*.py of the reference); those
names resolve to the grappa_b200 modules of the same role, imported on first use:

  t10n.{dataloader, dataloader_gpu, sampler, xbsampler, xborder, grad, cl, infer,
        device_allocator, util}                      -> grappa_b200.<same name>
  t10n.dataset.{meta, io_dist, chunk_seq, chunk_dist, dgl_to_t10n}
                                                     -> grappa_b200.dataset.<same name>
  t10n.dgl_dsg.{sampler, compliant}                  -> grappa_b200.dgl_dsg
  t10n._C.{graph, xborder, c_seq, c_dist}            -> grappa_b200._C (C++ host engine) with the
                                                        reference's native signatures
                                                        (grappa_b200.t10n_native)
"""
import importlib
import importlib.abc
import importlib.util
import sys

_ALIASES = {
    "t10n.dataloader": "grappa_b200.dataloader",
    "t10n.dataloader_gpu": "grappa_b200.dataloader_gpu",
    "t10n.sampler": "grappa_b200.sampler",
    "t10n.xbsampler": "grappa_b200.xbsampler",
    "t10n.xborder": "grappa_b200.xborder",
    "t10n.grad": "grappa_b200.grad",
    "t10n.cl": "grappa_b200.cl",
    "t10n.infer": "grappa_b200.infer",
    "t10n.device_allocator": "grappa_b200.device_allocator",
    "t10n.util": "grappa_b200.util",
    "t10n.dataset": "grappa_b200.dataset",
    "t10n.dataset.meta": "grappa_b200.dataset.meta",
    "t10n.dataset.io_dist": "grappa_b200.dataset.io_dist",
    "t10n.dataset.chunk_seq": "grappa_b200.dataset.chunk_seq",
    "t10n.dataset.chunk_dist": "grappa_b200.dataset.chunk_dist",
    "t10n.dataset.dgl_to_t10n": "grappa_b200.dataset.dgl_to_t10n",
    "t10n.dgl_dsg": "grappa_b200.dgl_dsg",
    "t10n.dgl_dsg.sampler": "grappa_b200.dgl_dsg",
    "t10n.dgl_dsg.compliant": "grappa_b200.dgl_dsg",
    "t10n._C": "grappa_b200._C",
}


class _AliasFinder(importlib.abc.MetaPathFinder, importlib.abc.Loader):
    def find_spec(self, name, path=None, target=None):
        if name in _ALIASES:
            return importlib.util.spec_from_loader(name, self, is_package=name.count(".") == 1)
        return None

    def create_module(self, spec):
        if spec.name == "t10n._C":
            # the submodules (graph, xborder, c_seq, c_dist) with the reference's native
            # signatures over the engine's (grappa_b200.t10n_native), importable by name
            import types

            from grappa_b200.t10n_native import build_modules

            native = importlib.import_module("grappa_b200._C")
            mod = types.ModuleType("t10n._C", native.__doc__)
            mod.__path__ = []
            for sub, m in build_modules("t10n._C").items():
                setattr(mod, sub, m)
                sys.modules[f"t10n._C.{sub}"] = m
            sys.modules[spec.name] = mod
            return mod
        mod = importlib.import_module(_ALIASES[spec.name])
        sys.modules[spec.name] = mod
        return mod

    def exec_module(self, module):
        return None


sys.meta_path.insert(0, _AliasFinder())
