"""Multi-process host logic of the multi-GPU bench on CPU (gloo, world size 2):
token sharding and the max-over-ranks timing reduction."""
import os

import pytest


def _worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    from powerinfer_x64_b200 import dist

    r, lr, w = dist.init(backend="gloo")
    lo, hi = dist.shard_range(1001, r, w)
    m = dist.max_over_ranks(1.5 + r)
    dist.barrier()
    q.put((r, lo, hi, m))
    import torch.distributed as td

    td.destroy_process_group()


def test_gloo_two_ranks():
    import multiprocessing as mp
    import socket

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][1:3] == (0, 501) and res[1][1:3] == (501, 1001)
    assert all(r[3] == 2.5 for r in res)


def test_shard_range_covers_everything():
    from powerinfer_x64_b200.dist import shard_range

    for n in (0, 1, 7, 64, 1000):
        for w in (1, 2, 3, 8):
            parts = [shard_range(n, r, w) for r in range(w)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(w - 1))
