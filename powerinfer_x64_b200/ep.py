"""Expert parallelism for the MoE layer.

Rank r of `world` holds experts [r*P, (r+1)*P), P = E / world, plus the full
router and the shared expert; tokens are data-parallel (each rank routes its
own home tokens). The reference has no counterpart (it runs one process,
model/mod.rs:1245-1571).

Two transports carry a layer forward:

* ``EPComm`` (the default on GPUs): NVLink peer memory, one C call per layer
  (``pi_moe_ep_forward``). Each home token's Q8_0 row goes once to every rank
  holding one of its experts; the destination runs its experts over all rows it
  received (and the shared expert over its home tokens) in one grouped GEMM,
  sums gate x output per row and stores that one partial row back; the home rank
  adds the partials in ascending rank order. No host synchronisation, no
  collective library; results equal ``MoeLayer.forward`` up to the regrouping
  of the combine sum by rank.
* ``RowExchange``: torch.distributed all_to_all_single over the staged calls
  ``pi_moe_ep_route`` / ``pi_moe_experts_q8`` / ``pi_moe_ep_combine`` (one row per
  (token, expert) slot, outputs returned per slot, the combine in the
  reference's order: bit for bit the one-GPU layer). Used when no comm is given,
  and by the gloo tests of the exchange bookkeeping on CPU.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import quant
from ._lib import PI_EP_HANDLE_BYTES, PI_FWD_FAST_SUM, PI_FWD_RESIDUAL, PI_FWD_RMSNORM, PI_QT_Q8_0, Context, PiError, PI_ERR_ARG, PiMoeLayerDesc, lib, ptr, \
    stream_ptr


def _torch():
    import torch

    return torch


class RowExchange:
    """All-to-all-v of row blocks over a process group (identity for one rank).

    ``counts(send_counts)`` exchanges the per-destination row counts and returns
    (send_splits, recv_splits) as host lists; ``rows(send, send_splits,
    recv_splits)`` sends rows [sum(send_splits), ...] (grouped by destination,
    ascending rank) and returns the received rows grouped by source rank.
    """

    def __init__(self, group=None):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1

    def counts(self, send_counts):
        torch = _torch()
        import torch.distributed as dist

        send = [int(v) for v in send_counts.cpu().tolist()]
        if self.world == 1:
            return send, list(send)
        sc = send_counts.to(torch.int64)
        rc = torch.empty_like(sc)
        dist.all_to_all_single(rc, sc, group=self.group)
        return send, [int(v) for v in rc.cpu().tolist()]

    def rows(self, send, send_splits, recv_splits):
        torch = _torch()
        import torch.distributed as dist

        if self.world == 1:
            return send[: sum(recv_splits)]
        out = torch.empty((sum(recv_splits),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        dist.all_to_all_single(out, send[: sum(send_splits)], output_split_sizes=recv_splits,
                               input_split_sizes=send_splits, group=self.group)
        return out


class EPComm:
    """This rank's exchange memory for expert-parallel layers over NVLink (pi_ep_comm).

    Every rank of the group builds one (collectively: the constructor exchanges the
    exported memory handles over ``group`` with all_gather_object) and passes it to
    each of its EPMoeLayer objects; one comm serves every layer. max_tokens bounds
    the home tokens of one forward.
    """

    def __init__(self, rank: int, world: int, max_tokens: int, n_embd: int, top_k: int, group=None,
                 device: int | None = None):
        import torch.distributed as dist

        self.ctx = Context.default(device)
        self.rank, self.world, self.max_tokens = rank, world, max_tokens
        h = C.c_void_p()
        self.ctx.check(lib().pi_ep_comm_create(self.ctx.h, rank, world, max_tokens, n_embd, top_k, C.byref(h)))
        self.h = h
        buf = (C.c_char * PI_EP_HANDLE_BYTES)()
        self.ctx.check(lib().pi_ep_comm_ipc_handle(h, buf))
        handles = [bytes(buf)]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, bytes(buf), group=group)
        allh = (C.c_char * (PI_EP_HANDLE_BYTES * world)).from_buffer_copy(b"".join(handles))
        self.ctx.check(lib().pi_ep_comm_open(h, allh))

    def __del__(self):
        try:
            if getattr(self, "h", None):
                lib().pi_ep_comm_destroy(self.h)
        except Exception:
            pass


class EPMoeLayer:
    """One MoE layer sharded by experts over `world` ranks (Q8_0 experts).

    gate/up/down_exps hold this rank's experts only (GGUF bytes of experts
    [rank*P, (rank+1)*P)); router, router_bias and shared are the full tensors.
    """

    def __init__(self, router, gate_exps, up_exps, down_exps, n_embd: int, n_ff: int, n_expert: int, top_k: int,
                 rank: int, world: int, shared=None, router_bias=None, exchange: RowExchange | None = None,
                 device: int | None = None, comm: EPComm | None = None):
        torch = _torch()
        if n_expert % world:
            raise PiError(PI_ERR_ARG, "n_expert must be a multiple of the world size")
        self.ctx = Context.default(device)
        self.d, self.f, self.E, self.k = n_embd, n_ff, n_expert, top_k
        self.rank, self.world, self.P = rank, world, n_expert // world
        self.has_shared = shared is not None
        self.exchange = exchange or RowExchange()
        self.comm = comm  # NVLink data plane (pi_moe_ep_forward); None: the all-to-all exchange
        keep = []

        def dev(a, dt):
            t = quant._dev(a, dt)
            keep.append(t)
            return ptr(t)

        desc = PiMoeLayerDesc()
        desc.n_embd, desc.n_ff_exp, desc.n_ff_shexp = n_embd, n_ff, n_ff
        desc.n_expert, desc.n_expert_used, desc.qtype, desc.src_on_host = n_expert, top_k, PI_QT_Q8_0, 0
        desc.router = dev(router, np.float32)
        desc.router_bias = dev(router_bias, np.float32) if router_bias is not None else None
        desc.gate_exps, desc.up_exps, desc.down_exps = (dev(gate_exps, np.uint8), dev(up_exps, np.uint8),
                                                        dev(down_exps, np.uint8))
        if shared is not None:
            g, u, d_, gi = shared
            desc.gate_shexp, desc.up_shexp, desc.down_shexp = dev(g, np.uint8), dev(u, np.uint8), dev(d_, np.uint8)
            desc.gate_inp_shexp = dev(gi, np.float32) if gi is not None else None
        h = C.c_void_p()
        torch.cuda.synchronize()
        self.ctx.check(lib().pi_moe_layer_create_ep(self.ctx.h, C.byref(desc), rank * self.P, self.P, C.byref(h)))
        self.h = h

    def __del__(self):
        try:
            if getattr(self, "h", None):
                lib().pi_moe_layer_destroy(self.h)
        except Exception:
            pass

    def forward(self, x, out=None, rmsnorm: bool = False, residual: bool = False, fast: bool = False):
        """MoE FFN of the home tokens x [T, d] (device f32) -> out [T, d]."""
        torch = _torch()
        L, s = lib(), stream_ptr()
        xd = quant._f32(x)
        T, d, k = xd.numel() // self.d, self.d, self.k
        if out is None:
            out = torch.empty((T, d), dtype=torch.float32, device="cuda")
        flags = (PI_FWD_RMSNORM if rmsnorm else 0) | (PI_FWD_RESIDUAL if residual else 0)
        flags |= PI_FWD_FAST_SUM if fast else 0
        if self.comm is not None:
            if T > self.comm.max_tokens:
                raise PiError(PI_ERR_ARG, "more home tokens than the comm's max_tokens")
            self.ctx.check(L.pi_moe_ep_forward(self.ctx.h, self.h, self.comm.h, ptr(xd), T, ptr(out), flags, s))
            return out
        if self.world == 1:
            # one rank holds every expert: nothing to exchange, the fused layer forward
            # (routed and shared experts in the same grouped launches) is the whole step
            if T:
                self.ctx.check(L.pi_moe_forward(self.ctx.h, self.h, ptr(xd), T, ptr(out), flags, s))
            return out
        dv = xd.device
        e = lambda *shape, dt=torch.float32: torch.empty(shape, dtype=dt, device=dv)
        idx, gates, shscale = e(T * k, dt=torch.int32), e(T * k), e(max(T, 1))
        xq, xs = e(T, d, dt=torch.int8), e(T, d // 32)
        send_counts = e(self.world, dt=torch.int32)
        send_xq, send_xs = e(T * k, d, dt=torch.int8), e(T * k, d // 32)
        send_eid, slot_row = e(T * k, dt=torch.int32), e(T * k, dt=torch.int32)
        self.ctx.check(L.pi_moe_ep_route(self.ctx.h, self.h, ptr(xd), T, flags, self.world, ptr(idx), ptr(gates),
                                         ptr(shscale), ptr(xq), ptr(xs), ptr(send_counts), ptr(send_xq), ptr(send_xs),
                                         ptr(send_eid), ptr(slot_row), s))
        # the shared expert needs only the home tokens: it runs on a side stream while
        # the counts and rows are exchanged and the routed experts run
        y_sh = None
        if self.has_shared and T:
            y_sh = e(T, d)
            cur = torch.cuda.current_stream()
            self._side = getattr(self, "_side", None) or torch.cuda.Stream(device=dv)
            self._side.wait_stream(cur)
            with torch.cuda.stream(self._side):
                self.ctx.check(L.pi_moe_experts_q8(self.ctx.h, self.h, T, ptr(xq), ptr(xs), None, ptr(y_sh),
                                                   stream_ptr(self._side)))
            for t_ in (xq, xs, y_sh):
                t_.record_stream(self._side)
        ex = self.exchange
        send_splits, recv_splits = ex.counts(send_counts)
        r_xq = ex.rows(send_xq, send_splits, recv_splits)
        r_xs = ex.rows(send_xs, send_splits, recv_splits)
        r_eid = ex.rows(send_eid, send_splits, recv_splits)
        n_recv = sum(recv_splits)
        y = e(max(n_recv, 1), d)
        self.ctx.check(L.pi_moe_experts_q8(self.ctx.h, self.h, n_recv, ptr(r_xq), ptr(r_xs), ptr(r_eid), ptr(y), s))
        y_back = ex.rows(y, recv_splits, send_splits)
        if y_sh is not None:
            torch.cuda.current_stream().wait_stream(self._side)
        self.ctx.check(L.pi_moe_ep_combine(self.ctx.h, self.h, ptr(xd), T, flags, ptr(gates), ptr(shscale),
                                           ptr(slot_row), ptr(y_back), ptr(y_sh) if y_sh is not None else None,
                                           ptr(out), s))
        return out


def local_expert_bytes(exps, n_expert: int, rank: int, world: int):
    """GGUF bytes of experts [rank*P, (rank+1)*P) out of an [E] expert tensor (equal slices)."""
    b = exps.reshape(-1)
    per = b.numel() // n_expert if hasattr(b, "numel") else b.size // n_expert
    P = n_expert // world
    return b[rank * P * per:(rank + 1) * P * per]
