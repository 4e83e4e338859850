"""Head sharding across ranks (scope_b200.shard) as world_size-2 gloo process
groups on the CPU: each rank takes its heads of a seeded layer output and
its own pointer-statistics histogram; the all-gather must rebuild the full
[H, T, D] output (no permute) and the gathered histograms must be the
ranks' own, in rank order.
The GPU run of the same path is bench.py --gpus N (NCCL)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from scope_b200 import shard

T, H, D = 256, 8, 64


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _full_output():
    g = torch.Generator().manual_seed(7)
    return torch.randn(H, T, D, generator=g).to(torch.bfloat16)


def _stats(rank):
    g = torch.Generator().manual_seed(100 + rank)
    return torch.randint(0, 50, (97,), generator=g, dtype=torch.int32)


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        full = _full_output()
        hs = shard.head_slice(H, rank, world)
        # the attention writes this rank's heads head-major: [H/N, T, D]
        local = full[hs].contiguous()
        buf = shard.gather_buffer(T, H, D, world, torch.bfloat16, "cpu")
        out, work = shard.gather_heads(local, buf, async_op=True)
        mine = _stats(rank)
        sbuf = shard.stats_buffer(mine, world)
        st, work2 = shard.gather_stats(mine, sbuf, async_op=True)
        work.wait()
        work2.wait()
        ok_out = torch.equal(out, full) and out.data_ptr() == buf.data_ptr()
        ok_st = torch.equal(st, torch.stack([_stats(r) for r in range(world)]))
        q.put((rank, ok_out, ok_st, None))
    except Exception as e:  # reported to the parent
        q.put((rank, False, False, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_head_shards_gather_outputs_and_stats_over_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok_out, ok_st, err in sorted(res):
        assert err is None, (rank, err)
        assert ok_out, f"rank {rank}: gathered output differs"
        assert ok_st, f"rank {rank}: gathered statistics differ"


def test_head_slice_rules():
    assert shard.head_slice(16, 3, 4) == slice(12, 16)
    with pytest.raises(ValueError):
        shard.head_slice(16, 0, 3)
    with pytest.raises(ValueError):
        shard.head_slice(16, 4, 4)
