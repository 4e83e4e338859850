"""Data-parallel gradient exchange of the decoder (scope_b200.decoder.
BucketedAllReduce) as world_size-2 gloo groups on the CPU: gradients live in
flat buckets, each bucket is all-reduced when its last gradient arrives
during the backward, and after wait() every rank holds the mean of the
ranks' gradients (what the reference's per-parameter all_reduce with AVG
gives, scoped_medium.py:2523-2524)."""
import os
import socket

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


def _model():
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.ReLU(), torch.nn.Linear(32, 8),
                               torch.nn.Linear(8, 4, bias=False))


def _grads(x):
    m = _model()
    m(x).square().sum().backward()
    return [p.grad.clone() for p in m.parameters()]


def _batch(rank):
    return torch.randn(5, 16, generator=torch.Generator().manual_seed(10 + rank))


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        from scope_b200.decoder import BucketedAllReduce
        dist.init_process_group("gloo", rank=rank, world_size=world)
        m = _model()
        dp = BucketedAllReduce(m.parameters(), bucket_mb=0.001)   # several buckets
        ok = len(dp.buckets) > 1
        for step in range(2):                                   # the buckets are reused
            dp.zero_grad()
            m(_batch(rank)).square().sum().backward()
            dp.wait()
            want = [sum(g) / world for g in zip(*[_grads(_batch(r)) for r in range(world)])]
            ok = ok and all(torch.allclose(p.grad, w, atol=1e-6) for p, w in zip(m.parameters(), want))
        q.put((rank, ok, None))
    except Exception as e:  # reported to the parent
        q.put((rank, False, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_bucketed_allreduce_averages_gradients_over_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in sorted(res):
        assert err is None, (rank, err)
        assert ok, f"rank {rank}: averaged gradients differ"
