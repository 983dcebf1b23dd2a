"""Failure detection without a GPU fault.

Host side (CPU gloo ranks): a rank that leaves the job is detected by the
others' heartbeat check between steps, and a collective with a dead peer ends
with an error within the process-group timeout instead of hanging.
Device side (one GPU): the bounded waits of the peer-memory kernels give up on a
flag that nothing sets and report kErrPeerTimeout in the error word, leaving the
context usable."""
import os
import socket
import time
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, port, q):
    try:
        import datetime

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=10))
        from grappa_b200.parallel.watchdog import Heartbeat, PeerFailure, default_store

        hb = Heartbeat(default_store(), rank, 2, interval_s=0.2, limit_s=1.5)
        t = torch.ones(4)
        dist.all_reduce(t)  # one healthy step
        dist.barrier()
        if rank == 1:
            hb.stop()
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # flush before leaving
            os._exit(0)  # leaves between steps, nothing in flight
        hb.check()
        detected = None
        t0 = time.time()
        while time.time() - t0 < 20:
            try:
                hb.check()
            except PeerFailure as e:
                detected = str(e)
                break
            time.sleep(0.2)
        # a collective with the dead peer errors out instead of waiting forever
        collective_error = None
        t1 = time.time()
        try:
            dist.all_reduce(torch.ones(4))
        except Exception as e:
            collective_error = type(e).__name__
        q.put((rank, {"detected": detected, "collective_error": collective_error,
                      "collective_s": time.time() - t1}))
        hb.stop()
        q.close()
        q.join_thread()
        os._exit(0)
    except Exception:
        q.put((rank, traceback.format_exc()))
        q.close()
        q.join_thread()
        os._exit(1)


def test_rank_leaving_is_detected():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, payload = q.get(timeout=120)
        res[r] = payload
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    out = res[0]
    assert isinstance(out, dict), out
    assert out["detected"] is not None and "rank(s) [1]" in out["detected"]
    assert out["collective_error"] is not None
    assert out["collective_s"] < 60


@pytest.mark.gpu
def test_peer_waits_give_up_with_error_status():
    from grappa_b200 import _native
    from grappa_b200.sampler_gpu import new_counters

    cu = _native.cuda()
    dev = torch.device("cuda", 0)
    n = 4096
    # a two-rank all-reduce whose "peer" never publishes: this rank's own buffers stand
    # in for the peer's, and nothing ever raises the peer's flags
    pages = [torch.zeros(2 * 8 * 160, dtype=torch.int32, device=dev) for _ in range(2)]
    scales = [torch.zeros(2, device=dev) for _ in range(2)]
    grads = [torch.randn(n, device=dev) for _ in range(2)]
    params = [torch.zeros(n, device=dev) for _ in range(2)]
    slots = [torch.zeros(n, device=dev) for _ in range(4)]
    m, v = torch.zeros(n, device=dev), torch.zeros(n, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    counters = new_counters(0, dev)
    for mode in (0, 1):  # one-shot, shard
        err.zero_()
        plan = cu.ArPlan()
        plan.add(rank=0, world=2, mode=mode, grad_bf16=False, lo=0, hi=n, grad=grads[0].data_ptr(),
                 grad_peer=[g.data_ptr() for g in grads] if mode else [],
                 slot_local=[] if mode else [slots[0].data_ptr(), slots[1].data_ptr()],
                 slot_peer=[] if mode else [t.data_ptr() for t in slots], param=params[0].data_ptr(),
                 param_peer=[t.data_ptr() for t in params] if mode else [], m=m, v=v, wbf=None,
                 scale_local=scales[0].data_ptr(), scale_peer=[t.data_ptr() for t in scales] if mode else [],
                 flags_local=pages[0].data_ptr(), flags_peer=[t.data_ptr() for t in pages], cov=None,
                 counters=counters, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, wd=0.0, do_adam=True, grad_out=None,
                 err=err, grid=2, timeout_ns=int(0.2e9))
        t0 = time.time()
        plan.launch(0)
        torch.cuda.synchronize()
        assert time.time() - t0 < 30
        assert int(err.item()) & 8  # kErrPeerTimeout
    # the device barrier gives up the same way
    err.zero_()
    epoch = torch.zeros(1, dtype=torch.int64, device=dev)
    bflags = torch.zeros(2, dtype=torch.int32, device=dev)
    other = torch.zeros(2, dtype=torch.int32, device=dev)
    cu.peer_barrier(0, 2, bflags.data_ptr(), [bflags.data_ptr(), other.data_ptr()], epoch, int(0.2e9), err)
    torch.cuda.synchronize()
    assert int(err.item()) & 8
    # the context is still usable
    x = torch.ones(16, device=dev)
    assert float((x * 2).sum()) == 32.0
