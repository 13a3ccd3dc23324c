"""Resident LM-head / projection matvec with its rows split over GPUs
(src/cuda/mod.rs:462-537): slice bookkeeping and the gather on CPU (gloo,
world size 2); the resident matvec against the oracle on the GPU."""
import os

import numpy as np
import pytest


def test_lm_head_slices_follow_the_reference():
    from powerinfer_x64_b200.lmhead import lm_head_slices

    for n_out in (1, 7, 1000, 151936):
        for g in (1, 2, 3, 8):
            sl = lm_head_slices(n_out, g)
            per = -(-n_out // g)
            assert len(sl) == g and sum(n for _, n in sl) == n_out
            for i, (lo, n) in enumerate(sl):
                # rows_per_gpu = div_ceil(n_out, n_gpus); GPU i takes [i*per, min((i+1)*per, n_out))
                assert lo == min(i * per, n_out) and n == max(0, min(lo + per, n_out) - lo)


def _worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    import torch

    from powerinfer_x64_b200 import dist
    from powerinfer_x64_b200.lmhead import gather_slices, lm_head_slices

    r, _, w = dist.init(backend="gloo")
    n_out, T = 11, 3
    full = torch.arange(T * n_out, dtype=torch.float32).reshape(T, n_out)
    sl = lm_head_slices(n_out, w)
    lo, n = sl[r]
    got = gather_slices(full[:, lo:lo + n].contiguous(), sl)
    q.put((r, bool(torch.equal(got, full))))
    import torch.distributed as td

    td.destroy_process_group()


def test_gather_two_ranks_gloo():
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
    assert all(ok for _, ok in res)


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", [8, 0])
def test_lm_head_resident_vs_oracle(orc, qtype):
    import torch

    from powerinfer_x64_b200.lmhead import LmHead

    rng = np.random.default_rng(5)
    n_in, n_out, T = 1024, 3000, 3
    w = rng.normal(0, 0.02, (n_out, n_in)).astype(np.float32)
    raw = orc.quantize_q8_0(w.reshape(-1)) if qtype == 8 else w.tobytes()
    x = rng.normal(0, 1, (T, n_in)).astype(np.float32)
    want = np.stack([orc.matvec_col_major(x[t], raw, qtype, n_in, n_out) for t in range(T)])
    for world in (1, 3):  # every rank's slice on this one GPU, assembled on the host
        parts = [LmHead(raw, qtype, n_out, n_in, rank=r, world=world).forward_local(torch.from_numpy(x).cuda())
                 for r in range(world)]
        got = torch.cat(parts, dim=1).cpu().numpy()
        assert got.shape == (T, n_out)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"world {world}"
