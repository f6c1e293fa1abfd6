"""Multi-rank host logic of batch-sharded inference, on CPU with gloo (world size 2 and 3):
sharded + all-gathered results equal the single-process result on the full batch."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _fake_engine(x):
    # per-sample "logits": deterministic function of the sample only
    return torch.stack([x.flatten(1).sum(1), x.flatten(1).amax(1)], 1)


def _worker(rank, world, port, B, q):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..",
                                    "triton-pass-analysis_b200"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from snn_compiler.sharding import ShardedInference
        g = torch.Generator().manual_seed(0)
        x = torch.rand(B, 3, 4, 4, generator=g)
        if B < world:
            # too few samples for the ranks: every rank refuses before any collective
            try:
                ShardedInference(_fake_engine)(x)
                q.put("no error")
            except ValueError:
                if rank == 0:
                    q.put("rejected")
            return
        sh = ShardedInference(_fake_engine)
        y = sh(x)
        # a second call reuses the preallocated slots and gives the same result
        y2 = sh(x)
        assert torch.equal(y, y2)
        if rank == 0:
            q.put(y)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,B", [(2, 8), (3, 10), (3, 3), (2, 1), (3, 2)])
def test_sharded_gather_equals_full_batch(world, B):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, q)) for r in range(world)]
    for p in procs:
        p.start()
    y = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    if B < world:
        assert y == "rejected"
        return
    g = torch.Generator().manual_seed(0)
    x = torch.rand(B, 3, 4, 4, generator=g)
    assert torch.equal(y, _fake_engine(x))


def test_shard_ranges_cover_batch():
    from snn_compiler.sharding import shard_range
    for B in (0, 1, 7, 64, 512):
        for world in (1, 2, 3, 8):
            spans = [shard_range(B, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == B
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)
