"""GPU test of the allocation-free sampling entry point.

``grappa_sample_hop_noalloc`` serves callers that must not allocate device memory
themselves (an application that owns every device allocation up front, or a
latency-critical loop that cannot afford cudaMalloc's implicit synchronisation):
its scan scratch is a fixed device array inside the library.  The test calls the
exported C symbol through ctypes, exactly as such a caller would, and checks two
calls in a row against the regular (allocating) entry point, whose scratch is a
caller-provided buffer.  The file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

from grappa_b200 import _native
from grappa_b200.sampler_gpu import new_counters

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _lib():
    lib = ctypes.CDLL(_native.cuda().__file__)
    f = lib.grappa_sample_hop_noalloc
    P = ctypes.c_void_p
    f.argtypes = [P, P, ctypes.c_int64, P, ctypes.c_int32, P, ctypes.c_int32, ctypes.c_int32, P, ctypes.c_int32,
                  P, P, P, P, ctypes.c_int32, P, P, P]
    f.restype = ctypes.c_int
    lib.grappa_sample_hop_noalloc_max_dst.restype = ctypes.c_int
    return lib


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _graph(n=3000, m=40000, seed=12):
    rng = np.random.default_rng(seed)
    u = rng.integers(0, n, m)
    v = rng.integers(0, n, m)
    v[: m // 5] = rng.integers(0, 10, m // 5)
    u2 = np.concatenate([u, v, np.arange(n)])
    v2 = np.concatenate([v, u, np.arange(n)])
    g = _native.host().graph.HostGraph(u2, v2, n)
    return torch.from_numpy(g.indptr()).to(DEV), torch.from_numpy(g.indices()).to(torch.int32).to(DEV), n


def _regular(indptr, indices, dst, fanout, counters, hop, gideg, cap_e, frontier=None, replace=False):
    n_dst = dst.numel()
    out_indptr = torch.full((n_dst + 1,), -7, dtype=torch.int32, device=DEV)
    out_nbr = torch.full((cap_e,), -7, dtype=torch.int32, device=DEV)
    n_e = torch.zeros(1, dtype=torch.int32, device=DEV)
    cov = torch.zeros(2, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    scratch = torch.zeros(_native.cuda().sample_scratch_words(n_dst), dtype=torch.int64, device=DEV)
    _native.cuda().sample_hop(indptr, indices, dst, None, n_dst, frontier, fanout, replace, counters, hop, gideg, cov,
                              out_indptr, out_nbr, n_e, scratch, err, n_dst)
    return out_indptr, out_nbr, n_e, cov, err


def _noalloc(lib, indptr, indices, n, dst, fanout, counters, hop, gideg, cap_e, frontier=None, replace=False,
             with_err=True):
    n_dst = dst.numel()
    out_indptr = torch.full((n_dst + 1,), -7, dtype=torch.int32, device=DEV)
    out_nbr = torch.full((cap_e,), -7, dtype=torch.int32, device=DEV)
    n_e = torch.zeros(1, dtype=torch.int32, device=DEV)
    cov = torch.zeros(2, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV) if with_err else None
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.grappa_sample_hop_noalloc(_ptr(indptr), _ptr(indices), n, _ptr(dst), n_dst, _ptr(frontier), fanout,
                                       1 if replace else 0, _ptr(counters), hop, _ptr(gideg), _ptr(cov),
                                       _ptr(out_indptr), _ptr(out_nbr), cap_e, _ptr(n_e), _ptr(err), stream)
    assert rc == 0, f"entry point returned {rc}"
    return out_indptr, out_nbr, n_e, cov, err


def test_noalloc_entry_matches_regular_entry_on_two_calls():
    lib = _lib()
    indptr, indices, n = _graph()
    counters = new_counters(17, DEV)
    # call 1: 2,000 seeds with coverage; call 2: a different, larger batch and step, so
    # that the scratch left behind by call 1 would corrupt call 2 if it were not cleared
    cases = [
        (torch.randperm(n, device=DEV)[:2000].to(torch.int32), 10, 0, True, (3, 4)),
        (torch.randint(0, n, (2900,), device=DEV, dtype=torch.int32).unique().to(torch.int32), 15, 1, False, (3, 5)),
    ]
    for dst, fanout, hop, with_cov, (epoch, step) in cases:
        counters[1], counters[2] = epoch, step
        gideg = torch.randint(0, 60, (dst.numel(),), dtype=torch.int64, device=DEV) if with_cov else None
        cap_e = dst.numel() * fanout
        want = _regular(indptr, indices, dst, fanout, counters, hop, gideg, cap_e)
        got = _noalloc(lib, indptr, indices, n, dst, fanout, counters, hop, gideg, cap_e)
        torch.cuda.synchronize()
        w_ip, w_nbr, w_ne, w_cov, w_err = want
        g_ip, g_nbr, g_ne, g_cov, g_err = got
        assert int(g_err.item()) == 0 and int(w_err.item()) == 0
        assert int(g_ne.item()) == int(w_ne.item()) > 0
        ne = int(w_ne.item())
        assert torch.equal(g_ip, w_ip)
        assert torch.equal(g_nbr[:ne], w_nbr[:ne])
        torch.testing.assert_close(g_cov, w_cov, rtol=1e-3, atol=1e-3)


def test_noalloc_entry_rejects_oversize_batch():
    lib = _lib()
    limit = lib.grappa_sample_hop_noalloc_max_dst()
    assert limit == 1 << 20
    indptr, indices, n = _graph(n=100, m=500)
    dummy = torch.zeros(1, dtype=torch.int32, device=DEV)
    counters = new_counters(1, DEV)
    rc = lib.grappa_sample_hop_noalloc(_ptr(indptr), _ptr(indices), n, _ptr(dummy), limit + 1, None, 5, 0,
                                       _ptr(counters), 0, None, None, _ptr(dummy), _ptr(dummy), 1, _ptr(dummy),
                                       _ptr(dummy), None)
    assert rc == 1  # GRAPPA_NOALLOC_TOO_MANY_DST, nothing launched


def test_noalloc_entry_replace_frontier_empty_and_no_error_word():
    """The other paths of the entry point against the regular launcher: sampling with
    replacement, a partial frontier mask, an empty batch (out_indptr[0] == 0, no edges)
    and a null error word, each twice in a row."""
    lib = _lib()
    indptr, indices, n = _graph(seed=5)
    counters = new_counters(23, DEV)
    gen = torch.Generator(device="cpu").manual_seed(3)
    for rep in range(2):
        counters[1], counters[2] = 2, 7 + rep
        dst = torch.randperm(n, generator=gen)[:1500].to(torch.int32).to(DEV)
        frontier = (torch.rand(dst.numel(), generator=gen) < 0.6).to(torch.uint8).to(DEV)
        for replace, fr, with_err in ((True, None, True), (False, frontier, True), (True, frontier, False)):
            cap_e = dst.numel() * 10
            want = _regular(indptr, indices, dst, 10, counters, 1, None, cap_e, frontier=fr, replace=replace)
            got = _noalloc(lib, indptr, indices, n, dst, 10, counters, 1, None, cap_e, frontier=fr, replace=replace,
                           with_err=with_err)
            torch.cuda.synchronize()
            assert int(want[4].item()) == 0
            if with_err:
                assert int(got[4].item()) == 0
            ne = int(want[2].item())
            assert ne > 0 and int(got[2].item()) == ne
            assert torch.equal(got[0], want[0])
            assert torch.equal(got[1][:ne], want[1][:ne])
        empty = torch.zeros(0, dtype=torch.int32, device=DEV)
        got = _noalloc(lib, indptr, indices, n, empty, 10, counters, 0, None, 16)
        torch.cuda.synchronize()
        assert int(got[0][0].item()) == 0
        assert int(got[2].item()) == 0
        assert int(got[4].item()) == 0
