"""Multi-rank host logic on CPU: world_size-2 gloo ranks shard the sessions without overlap and
agree on the max-over-ranks time and the token total (the only cross-rank traffic)."""
import os
import socket

import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, total, out):
    import sys
    import datetime
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "gpt-sovits.cpp_b200"))
    import torch.distributed as dist
    import shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    lo, hi = shard.session_shard(total, world, rank)
    t_max = shard.max_over_ranks(1.0 + rank)
    n = shard.sum_over_ranks(float(hi - lo))
    out.put((rank, lo, hi, t_max, n))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("total", [2048, 7])
def test_gloo_two_ranks_shard_and_reduce(total):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, total, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, lo0, hi0, t0, n0), (r1, lo1, hi1, t1, n1) = res
    assert lo0 == 0 and hi0 == lo1 and hi1 == total
    assert abs((hi0 - lo0) - (hi1 - lo1)) <= 1
    assert t0 == t1 == 2.0 and n0 == n1 == float(total)


def test_shard_sizes():
    import shard
    for total, world in [(2048, 8), (2048, 3), (5, 8)]:
        spans = [shard.session_shard(total, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
