"""Loader of the native extensions.

``host()`` returns grappa_b200._C (the C++ host engine, always required).
``cuda()`` returns grappa_b200._cuda (the sm_100a kernels).  On a machine with a
GPU a missing or unloadable CUDA extension is an error, never a silent fallback:
the CUDA code path is the product.
"""
import importlib

import torch

_host = None
_cuda = None


def host():
    global _host
    if _host is None:
        _host = importlib.import_module("grappa_b200._C")
    return _host


def cuda():
    global _cuda
    if _cuda is None:
        try:
            _cuda = importlib.import_module("grappa_b200._cuda")
        except ImportError as e:
            raise RuntimeError(
                "grappa_b200._cuda is not built; run `python setup.py build_ext --inplace`"
            ) from e
    return _cuda


def cuda_available():
    try:
        cuda()
    except RuntimeError:
        return False
    return torch.cuda.is_available()
