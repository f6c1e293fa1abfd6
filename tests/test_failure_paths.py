"""Failure detection without faulting a GPU.

Host side (CPU, no device touched):
  - an injected status from the library (snnb_debug_inject_status) comes back from the
    entry point and the Python layer maps it to SnnbError;
  - snnb_set_wait_limit rejects a limit too short to be meaningful;
  - gloo ranks: a rank that never joins makes the others' rendezvous end with an error
    inside its timeout, and a rank that leaves before the all-gather makes the others'
    ShardedInference call end with an error instead of hanging.
GPU side (marked gpu):
  - a wait that nothing will complete runs out: with a short wait limit and the stall hook,
    the T-sequential conv kernel's MMA warp waits for a stage that CTA 0's producer
    withholds (no copy is in flight in that CTA); the launch returns, the device status
    reads SNNB_ERR_TIMEOUT once (reading clears it), the engine-level check raises
    SnnbError, and the next launch with the default limit is correct.
"""
import datetime
import os
import socket
import time

import pytest
import torch


def test_injected_status_is_returned_and_raised():
    from snn_compiler import _lib
    L = _lib.lib()
    assert L.snnb_debug_inject_status(-4, 1) == 0
    try:
        # any entry: the injected status comes back before the arguments are looked at
        st = L.snnb_neuron_multistep(None, 0, 4, 16, None, None, 1, 1, 0, 0.5, 0.5, None, 1,
                                     0.0, 0, 1.0, None, None, None, 0, None, None, None, None)
        assert st == -4
        with pytest.raises(_lib.SnnbError, match="timed out"):
            _lib.check(st, "snnb_neuron_multistep")
        # consumed: the next call validates its arguments again (null x -> invalid argument)
        st2 = L.snnb_neuron_multistep(None, 0, 4, 16, None, None, 1, 1, 0, 0.5, 0.5, None, 1,
                                      0.0, 0, 1.0, None, None, None, 0, None, None, None, None)
        assert st2 == -1
        # a count covers that many calls, across entry points
        assert L.snnb_debug_inject_status(-3, 2) == 0
        assert L.snnb_bgemm(None, None, None, 1, 1, 1, 1, 1, 0, None) == -3
        assert L.snnb_conv3x3_lif(None, 4, 1, 8, 8, 64, None, None, 64, 0.5, 0.5, 1.0, 0.0, 1,
                                  0, 0, 0, 1, None, 0, None, None) == -3
        assert L.snnb_bgemm(None, None, None, 1, 1, 1, 1, 1, 0, None) == -1
    finally:
        L.snnb_debug_inject_status(-1, 0)
    assert L.snnb_debug_inject_status(1, 1) == -1        # only error statuses
    assert L.snnb_debug_inject_status(-4, -1) == -1


def test_wait_limit_rejects_meaningless_values():
    from snn_compiler import _lib
    L = _lib.lib()
    assert L.snnb_set_wait_limit(10) == -1
    assert L.snnb_set_wait_limit(-5) == -1
    assert L.snnb_debug_inject_stall(-1) == -1


# ---- gloo ranks --------------------------------------------------------------------------
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _lonely_rank(port, q):
    import torch.distributed as dist
    t0 = time.time()
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0,
                                world_size=2, timeout=datetime.timedelta(seconds=3))
        q.put(("joined", time.time() - t0))
    except Exception as e:                      # rank 1 never came
        q.put((type(e).__name__, time.time() - t0))


def test_rank_that_never_joins_times_out_cleanly():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(_free_port(), q))
    p.start()
    what, dt = q.get(timeout=120)
    p.join(timeout=60)
    assert what != "joined"
    assert dt < 60
    assert p.exitcode == 0


def _leaving_rank(rank, port, q):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..",
                                    "triton-pass-analysis_b200"))
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=2, timeout=datetime.timedelta(seconds=5))
    from snn_compiler.sharding import ShardedInference
    sh = ShardedInference(lambda x: x.flatten(1).sum(1, keepdim=True))
    x = torch.arange(8.0).reshape(8, 1)
    assert torch.equal(sh(x), x)               # both ranks: one step together
    def report(item):
        q.put(item)
        q.close()
        q.join_thread()                        # flushed before the process ends

    if rank == 1:
        report(("left", 0.0))
        os._exit(0)                            # leaves between steps, no collective in flight
    t0 = time.time()
    try:
        sh(x)
        report(("completed", time.time() - t0))
    except Exception as e:
        report((type(e).__name__, time.time() - t0))
    os._exit(0)


def test_rank_that_leaves_makes_the_next_collective_fail():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    outcomes = {w for w, _ in got}
    assert "left" in outcomes
    other = [g for g in got if g[0] != "left"][0]
    assert other[0] != "completed", other
    assert other[1] < 60


# ---- GPU: a wait that runs out -----------------------------------------------------------
@pytest.mark.gpu
def test_wait_timeout_reports_and_recovers():
    from snn_compiler import _lib
    from snn_compiler.kernels import conv as KC
    L = _lib.lib()
    dev = "cuda"
    g = torch.Generator().manual_seed(3)
    T, B, C, H = 4, 2, 64, 16
    x = (torch.rand(T, B, H, H, C, generator=g) < 0.2).to(torch.bfloat16).to(dev)
    w = (torch.randn(64, 3, 3, C, generator=g) * 0.06).to(torch.bfloat16).to(dev)
    b = (torch.rand(64, generator=g) * 0.9 + 0.3).to(dev)
    kw = dict(tau=2.0, v_threshold=1.0, variant=1, block_n=64)
    ref = KC.conv3x3_lif(x, w, b, **kw)
    assert KC.device_status() == 0
    torch.cuda.synchronize()
    try:
        _lib.check(L.snnb_set_wait_limit(200_000), "snnb_set_wait_limit")     # ~0.1 ms
        _lib.check(L.snnb_debug_inject_stall(1), "snnb_debug_inject_stall")
        t0 = time.time()
        KC.conv3x3_lif(x, w, b, **kw)
        torch.cuda.synchronize()
        dt = time.time() - t0
        assert KC.device_status() == -4               # SNNB_ERR_TIMEOUT, cleared by the read
        assert KC.device_status() == 0
        assert dt < 1.0                               # ended by the short limit, not the default
        # the engine-level check turns the status into an exception
        _lib.check(L.snnb_debug_inject_stall(1), "snnb_debug_inject_stall")
        KC.conv3x3_lif(x, w, b, **kw)
        with pytest.raises(_lib.SnnbError, match="timed out"):
            KC.raise_on_device_status("conv3x3_lif")
    finally:
        L.snnb_debug_inject_stall(0)
        L.snnb_set_wait_limit(0)
    y = KC.conv3x3_lif(x, w, b, **kw)                 # the context is usable and correct
    assert KC.device_status() == 0
    assert torch.equal(y, ref)
