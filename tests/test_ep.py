"""Expert parallelism: the row exchange's bookkeeping on CPU (gloo, two ranks),
and on GPUs the sharded layer against the one-GPU layer, bit for bit."""
import os
import socket

import numpy as np
import pytest


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


# ---------------------------------------------------------------- CPU (gloo)
def _exchange_worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    import torch
    import torch.distributed as td

    from powerinfer_x64_b200 import dist
    from powerinfer_x64_b200.ep import RowExchange

    dist.init(backend="gloo")
    ex = RowExchange()
    # rank r sends (r + 1) * (dst + 1) rows to rank dst; each row tagged (src, dst, i)
    counts = torch.tensor([(rank + 1) * (dst + 1) for dst in range(world)], dtype=torch.int32)
    rows = torch.tensor([[rank, dst, i] for dst in range(world) for i in range((rank + 1) * (dst + 1))],
                        dtype=torch.int64)
    send, recv = ex.counts(counts)
    got = ex.rows(rows, send, recv)
    back = ex.rows(got, recv, send)
    q.put((rank, send, recv, got.tolist(), bool(torch.equal(back, rows))))
    td.destroy_process_group()


def test_row_exchange_two_ranks_gloo():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=180) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, send, recv, got, round_trip in res:
        assert send == [(rank + 1) * (d + 1) for d in range(2)]
        assert recv == [(s + 1) * (rank + 1) for s in range(2)]
        # received rows: grouped by source rank ascending, each source's rows for this rank in order
        want = [[s, rank, i] for s in range(2) for i in range((s + 1) * (rank + 1))]
        assert got == want
        assert round_trip


# ---------------------------------------------------------------- GPU
@pytest.fixture(scope="module")
def torch():
    import torch as t

    assert t.cuda.is_available()
    return t


@pytest.fixture(scope="module")
def pkg():
    from powerinfer_x64_b200 import build

    build.build()
    import powerinfer_x64_b200 as p

    return p


@pytest.mark.gpu
@pytest.mark.parametrize("T", [40, 300])
def test_ep_one_rank_equals_layer(pkg, torch, T):
    """world = 1: the staged expert-parallel forward equals MoeLayer.forward bit for bit
    (GEMV experts at T = 40, tensor-core experts at T = 300), with RMSNorm + residual."""
    from powerinfer_x64_b200 import synth
    from powerinfer_x64_b200.ep import EPMoeLayer

    c = synth.C2
    L, t = synth.moe_layer(c, seed=3, keep_tensors=True)
    x = synth.tokens_dev(c.d, T, seed=5)
    ref = L.forward(x, rmsnorm=True, residual=True).cpu().numpy()
    ep = EPMoeLayer(t["router"], t["gate_exps"], t["up_exps"], t["down_exps"], c.d, c.f, c.E, c.k, rank=0, world=1,
                    shared=t["shared"])
    got = ep.forward(x, rmsnorm=True, residual=True).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def _ep_worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        import torch
        import torch.distributed as td

        from powerinfer_x64_b200 import dist, synth
        from powerinfer_x64_b200.ep import EPMoeLayer, local_expert_bytes

        dist.init(backend="nccl")
        c = synth.C2
        L, t = synth.moe_layer(c, seed=3, keep_tensors=True)  # every rank builds the same full layer
        loc = lambda a: local_expert_bytes(a, c.E, rank, world)
        ep = EPMoeLayer(t["router"], loc(t["gate_exps"]), loc(t["up_exps"]), loc(t["down_exps"]), c.d, c.f, c.E,
                        c.k, rank=rank, world=world, shared=t["shared"])
        ok = True
        for T in (37, 300):
            x = synth.tokens_dev(c.d, T, seed=10 + rank)  # each rank its own home tokens
            ref = L.forward(x, rmsnorm=True, residual=True).cpu().numpy()
            got = ep.forward(x, rmsnorm=True, residual=True).cpu().numpy()
            ok &= bool(np.array_equal(got.view(np.uint32), ref.view(np.uint32)))
        dist.barrier(rank)
        td.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, False, repr(exc)))


@pytest.mark.gpu
def test_ep_two_ranks_nccl(pkg, torch):
    """Two ranks over NCCL (child processes, one GPU each): each rank's home tokens
    through the sharded layer equal the one-GPU layer's output bit for bit."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_ep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=600) for _ in ps)
    for p in ps:
        p.join(timeout=120)
    assert all(ok for _, ok, _ in res), res


@pytest.mark.gpu
@pytest.mark.parametrize("T", [5, 64])
def test_q8_decode_experts_bit_exact(pkg, torch, T):
    """The decode (GEMV) expert kernels sum Q8_0 block terms in the reference's order too:
    a top-1 layer (gate exactly 1) gives the reference restatement's output bit for bit."""
    import pi_oracle as orc
    from powerinfer_x64_b200 import moe

    orc.build()
    rng = np.random.default_rng(22)
    d, E, k, f = 1024, 8, 1, 512
    router = (rng.standard_normal(E * d) * 0.02).astype(np.float32)
    g, u, dn = (orc.quantize_q8_0((rng.standard_normal(E * f * d) * 0.02).astype(np.float32)) for _ in range(3))
    x = rng.standard_normal((T, d)).astype(np.float32)
    L = moe.MoeLayer(router, g, u, dn, 8, d, f, E, k)
    got = L.forward(torch.from_numpy(x).cuda(), path="gemv").cpu().numpy()
    ref = orc.moe_layer(x, d, f, E, k, 8, router, g, u, dn, threads=1)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), int(np.count_nonzero(got != ref))


# ------------------------------------------------- NVLink data plane (pi_ep_comm)
@pytest.mark.gpu
@pytest.mark.parametrize("T", [37, 300])
def test_ep_nvlink_self_equals_layer(pkg, torch, T):
    """world = 1 through the peer-memory data plane (rows pushed to this rank's own
    exchange memory, experts, partial rows returned, combine): a single partial per
    token is the whole combine sum, so the output equals MoeLayer.forward bit for bit."""
    from powerinfer_x64_b200 import synth
    from powerinfer_x64_b200.ep import EPComm, EPMoeLayer

    c = synth.C2
    L, t = synth.moe_layer(c, seed=3, keep_tensors=True)
    comm = EPComm(0, 1, 512, c.d, c.k)
    ep = EPMoeLayer(t["router"], t["gate_exps"], t["up_exps"], t["down_exps"], c.d, c.f, c.E, c.k, rank=0, world=1,
                    shared=t["shared"], comm=comm)
    for rep in range(3):  # epochs of both parities, buffer reuse
        x = synth.tokens_dev(c.d, T, seed=5 + rep)
        ref = L.forward(x, rmsnorm=True, residual=True, path="gemm").cpu().numpy()
        got = ep.forward(x, rmsnorm=True, residual=True).cpu().numpy()
        ep.ctx.sync_check()
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), rep


@pytest.mark.gpu
def test_ep_nvlink_wait_times_out(pkg, torch):
    """A forward whose peers never acknowledge (the test hook skips epochs) gives up
    after its bounded waits and reports PI_ERR_TIMEOUT; the device stays usable."""
    from powerinfer_x64_b200 import PiError, synth
    from powerinfer_x64_b200._lib import PI_ERR_TIMEOUT, lib
    from powerinfer_x64_b200.ep import EPComm, EPMoeLayer

    c = synth.C2
    L, t = synth.moe_layer(c, seed=3, keep_tensors=True)
    comm = EPComm(0, 1, 64, c.d, c.k)
    ep = EPMoeLayer(t["router"], t["gate_exps"], t["up_exps"], t["down_exps"], c.d, c.f, c.E, c.k, rank=0, world=1,
                    shared=t["shared"], comm=comm)
    x = synth.tokens_dev(c.d, 16, seed=1)
    ep.forward(x)
    ep.ctx.sync_check()
    assert lib().pi_ep_comm_debug_skip(comm.h, 3) == 0
    ep.forward(x)
    with pytest.raises(PiError) as ei:
        ep.ctx.sync_check()
    assert ei.value.code == PI_ERR_TIMEOUT
    y = L.forward(x)  # the context still runs kernels
    ep.ctx.sync_check()
    assert np.all(np.isfinite(y.cpu().numpy()))


def _ep_nvlink_worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        import torch
        import torch.distributed as td

        from powerinfer_x64_b200 import dist, synth
        from powerinfer_x64_b200.ep import EPComm, EPMoeLayer, local_expert_bytes

        dist.init(backend="nccl")
        c = synth.C2
        L, t = synth.moe_layer(c, seed=3, keep_tensors=True)  # every rank builds the same full layer
        loc = lambda a: local_expert_bytes(a, c.E, rank, world)
        comm = EPComm(rank, world, 512, c.d, c.k)
        ep = EPMoeLayer(t["router"], loc(t["gate_exps"]), loc(t["up_exps"]), loc(t["down_exps"]), c.d, c.f, c.E,
                        c.k, rank=rank, world=world, shared=t["shared"], comm=comm)
        worst = 0.0
        for rep, T in enumerate((37, 300, 512, 0, 100)):  # ragged, empty and full batches
            x = synth.tokens_dev(c.d, max(T, 1), seed=10 + rank + 7 * rep)[:T]
            ref = L.forward(x, rmsnorm=True, residual=True, path="gemm").cpu().numpy() if T else np.zeros((0, c.d))
            got = ep.forward(x, rmsnorm=True, residual=True).cpu().numpy()
            ep.ctx.sync_check()
            if T:
                f_ref, f_got = ref - x.cpu().numpy(), got - x.cpu().numpy()
                worst = max(worst, float(np.max(np.abs(f_got - f_ref)) / np.sqrt(np.mean(f_ref ** 2))))
        dist.barrier(rank)
        td.destroy_process_group()
        q.put((rank, worst < 1e-5, f"max-abs/rms {worst:.2e}"))
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, False, repr(exc)))


@pytest.mark.gpu
def test_ep_two_ranks_nvlink(pkg, torch):
    """Two ranks (child processes, one GPU each) over the peer-memory data plane: each
    rank's home tokens through the sharded layer match the one-GPU layer to f32
    rounding of the regrouped combine sum (max-abs below 1e-5 of the RMS)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_ep_nvlink_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=600) for _ in ps)
    for p in ps:
        p.join(timeout=120)
    assert all(ok for _, ok, _ in res), res
