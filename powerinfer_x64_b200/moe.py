"""Host-side mirror of the reference's MoE operators.

* ``MoeLayer`` — the MoE FFN that actually runs in the reference
  (model/mod.rs:1245-1571): f32 router over GGUF ``ffn_gate_inp``
  [ne0=d, ne1=E], softmax -> top-k -> ascending -> renormalised gates,
  Q8_0/Q4_0 SwiGLU experts and the sigmoid-gated shared expert. Weights are
  repacked once into HBM; ``route`` and ``forward`` run on the GPU.
* ``MoeRouter`` / ``RoutingResult`` / ``moe_forward`` / ``ExpertWeights`` —
  the standalone operator API of src/moe/mod.rs:24-219 (row-major [d, E]
  router, top-k on logits, softmax over the selected k, descending order).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import quant
from ._lib import (PI_FWD_FAST_SUM, PI_FWD_FORCE_GEMM, PI_FWD_FORCE_GEMV, PI_FWD_RESIDUAL, PI_FWD_RMSNORM, PI_QT_F32, Context, PiError, PiMoeLayerDesc, PI_ERR_ARG, lib,
                   ptr, stream_ptr)


def _torch():
    import torch

    return torch


class MoeLayer:
    """Device-resident MoE FFN layer built from GGUF-layout tensors.

    Tensors may be numpy arrays / bytes (host) or CUDA torch tensors:
      router      f32 [E*d]   (ffn_gate_inp, row e = expert e)
      gate_exps   GGUF bytes [ne0=d, ne1=f, ne2=E]; up_exps likewise
      down_exps   GGUF bytes [ne0=f, ne1=d, ne2=E]
      shared      optional (gate_shexp, up_shexp, down_shexp, gate_inp_shexp)
      router_bias optional f32 [E] added to the logits.
    """

    def __init__(self, router, gate_exps, up_exps, down_exps, qtype, n_embd: int, n_ff: int, n_expert: int,
                 top_k: int, shared=None, router_bias=None, device: int | None = None):
        torch = _torch()
        self.ctx = Context.default(device)
        self.n_embd, self.n_ff, self.n_expert, self.top_k = n_embd, n_ff, n_expert, top_k
        self.qtype = int(qtype)
        self.has_shared = shared is not None
        keep = []

        def dev(a, dt):
            t = quant._dev(a, dt)
            keep.append(t)
            return ptr(t)

        desc = PiMoeLayerDesc()
        desc.n_embd, desc.n_ff_exp, desc.n_ff_shexp = n_embd, n_ff, n_ff
        desc.n_expert, desc.n_expert_used, desc.qtype, desc.src_on_host = n_expert, top_k, self.qtype, 0
        desc.router = dev(router, np.float32)
        desc.router_bias = dev(router_bias, np.float32) if router_bias is not None else None
        desc.gate_exps = dev(gate_exps, np.uint8)
        desc.up_exps = dev(up_exps, np.uint8)
        desc.down_exps = dev(down_exps, np.uint8)
        if shared is not None:
            g, u, d_, gi = shared
            desc.gate_shexp, desc.up_shexp, desc.down_shexp = dev(g, np.uint8), dev(u, np.uint8), dev(d_, np.uint8)
            desc.gate_inp_shexp = dev(gi, np.float32) if gi is not None else None
        h = C.c_void_p()
        torch.cuda.synchronize()
        self.ctx.check(lib().pi_moe_layer_create(self.ctx.h, C.byref(desc), C.byref(h)))
        self.h = h

    def __del__(self):
        try:
            if getattr(self, "h", None):
                lib().pi_moe_layer_destroy(self.h)
        except Exception:
            pass

    # -- routing -----------------------------------------------------------
    def route(self, x, T: int | None = None):
        """Routing for tokens x [T, d] -> dict(idx, gates, counts, offsets, perm) (device tensors)."""
        torch = _torch()
        xd = quant._f32(x)
        T = xd.numel() // self.n_embd if T is None else T
        E, k = self.n_expert, self.top_k
        o = dict(idx=torch.empty((T, k), dtype=torch.int32, device="cuda"),
                 gates=torch.empty((T, k), dtype=torch.float32, device="cuda"),
                 counts=torch.empty(E, dtype=torch.int32, device="cuda"),
                 offsets=torch.empty(E, dtype=torch.int32, device="cuda"),
                 perm=torch.empty(T * k, dtype=torch.int32, device="cuda"))
        self.ctx.check(lib().pi_moe_route(self.ctx.h, self.h, ptr(xd), T, ptr(o["idx"]), ptr(o["gates"]),
                                          ptr(o["counts"]), ptr(o["offsets"]), ptr(o["perm"]), stream_ptr()))
        return o

    # -- forward -----------------------------------------------------------
    def forward(self, x, out=None, rmsnorm: bool = False, residual: bool = False, stream=None, path: str = "auto",
                fast: bool = False):
        """MoE FFN of tokens x [T, d] (device f32) -> out [T, d].

        path: "auto" (tensor-core GEMM for prefill-sized Q4_0 batches, else GEMV),
        "gemv" or "gemm" to force one. fast: the Q8_0 prefill GEMM adds each block
        term with a fused multiply-add (PI_FWD_FAST_SUM; within the parity tolerance,
        not bit-identical).
        """
        torch = _torch()
        xd = quant._f32(x)
        T = xd.numel() // self.n_embd
        if out is None:
            out = torch.empty((T, self.n_embd), dtype=torch.float32, device="cuda")
        if T == 0:
            return out
        flags = (PI_FWD_RMSNORM if rmsnorm else 0) | (PI_FWD_RESIDUAL if residual else 0)
        flags |= {"auto": 0, "gemv": PI_FWD_FORCE_GEMV, "gemm": PI_FWD_FORCE_GEMM}[path]
        flags |= PI_FWD_FAST_SUM if fast else 0
        self.ctx.check(lib().pi_moe_forward(self.ctx.h, self.h, ptr(xd), T, ptr(out), flags, stream_ptr(stream)))
        return out

    def forward_routed(self, x, out=None, rmsnorm: bool = False, residual: bool = False, stream=None,
                       path: str = "auto", fast: bool = False):
        """``forward`` that also returns the routing it used: (out, dict(idx, gates,
        counts, offsets, perm)) as ``route`` returns them, computed on the
        (optionally RMS-normed) tokens the forward itself routed."""
        torch = _torch()
        xd = quant._f32(x)
        T = xd.numel() // self.n_embd
        E, k = self.n_expert, self.top_k
        if out is None:
            out = torch.empty((T, self.n_embd), dtype=torch.float32, device="cuda")
        o = dict(idx=torch.empty((T, k), dtype=torch.int32, device="cuda"),
                 gates=torch.empty((T, k), dtype=torch.float32, device="cuda"),
                 counts=torch.zeros(E, dtype=torch.int32, device="cuda"),
                 offsets=torch.zeros(E, dtype=torch.int32, device="cuda"),
                 perm=torch.empty(T * k, dtype=torch.int32, device="cuda"))
        if T == 0:
            return out, o
        flags = (PI_FWD_RMSNORM if rmsnorm else 0) | (PI_FWD_RESIDUAL if residual else 0)
        flags |= {"auto": 0, "gemv": PI_FWD_FORCE_GEMV, "gemm": PI_FWD_FORCE_GEMM}[path]
        flags |= PI_FWD_FAST_SUM if fast else 0
        self.ctx.check(lib().pi_moe_forward_routed(self.ctx.h, self.h, ptr(xd), T, ptr(out), flags, ptr(o["idx"]),
                                                   ptr(o["gates"]), ptr(o["counts"]), ptr(o["offsets"]),
                                                   ptr(o["perm"]), stream_ptr(stream)))
        return out, o


# --------------------------------------------------------------------------
# src/moe operator API
# --------------------------------------------------------------------------
@dataclass
class RoutingResult:
    """moe/mod.rs:24-29."""

    expert_indices: list
    expert_weights: list


class MoeRouter:
    """moe/mod.rs:35-108: router over a row-major [n_embd, n_experts] f32 gate.

    ``route`` computes logits[j] = sum_i x[i] * gate[i*E + j] (ops::matvec_t,
    sequential in i), keeps the top-k logits (ties to the lowest index), orders
    them by descending logit and applies ops::softmax over the selected k.
    """

    def __init__(self, gate_weight, n_embd: int, n_experts: int, top_k: int):
        gw = np.asarray(gate_weight, dtype=np.float32).reshape(-1)
        if gw.size != n_embd * n_experts:
            raise PiError(PI_ERR_ARG, "gate_weight must have n_embd * n_experts elements")
        if not (1 <= top_k <= n_experts):
            raise PiError(PI_ERR_ARG, "top_k must be in 1..=n_experts")
        self.n_embd, self._n_experts, self._top_k = n_embd, n_experts, top_k
        # expert-major copy: row e = column e of the row-major gate (same values, same i order)
        wt = np.ascontiguousarray(gw.reshape(n_embd, n_experts).T)
        self._layer = _RouterOnly(wt, n_embd, n_experts, top_k)

    def n_experts(self) -> int:
        return self._n_experts

    def top_k(self) -> int:
        return self._top_k

    def route(self, x) -> RoutingResult:
        idx, w = self._layer.route_api(np.asarray(x, dtype=np.float32).reshape(1, -1))
        return RoutingResult(expert_indices=[int(i) for i in idx[0]], expert_weights=[float(v) for v in w[0]])


class _RouterOnly:
    """A router-only pi_moe_layer (dummy single-block experts are never run)."""

    def __init__(self, w_expert_major, n_embd, n_experts, top_k):
        self.n_embd, self.E, self.k = n_embd, n_experts, top_k
        self.w = np.asarray(w_expert_major, dtype=np.float32)

    def route_api(self, x):
        torch = _torch()
        ctx = Context.default()
        T = x.shape[0]
        wd = torch.from_numpy(self.w).cuda()
        xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        idx = torch.empty((T, self.k), dtype=torch.int32, device="cuda")
        wts = torch.empty((T, self.k), dtype=torch.float32, device="cuda")
        ctx.check(lib().pi_router_topk_softmax(ctx.h, ptr(xd), T, ptr(wd), self.n_embd, self.E, self.k, ptr(idx),
                                               ptr(wts), stream_ptr()))
        torch.cuda.synchronize()
        return idx.cpu().numpy(), wts.cpu().numpy()


class ExpertWeights:
    """moe/mod.rs:226-266: f32 experts, gate/up [n_embd, f] row-major, down [f, n_embd]."""

    def __init__(self, expert_gate, expert_up, expert_down):
        if not (len(expert_gate) == len(expert_up) == len(expert_down)):
            raise PiError(PI_ERR_ARG, "expert lists differ in length")
        self.expert_gate, self.expert_up, self.expert_down = expert_gate, expert_up, expert_down

    def get_expert(self, idx: int):
        return self.expert_gate[idx], self.expert_up[idx], self.expert_down[idx]

    def get_expert_f32(self, idx: int):
        return self.get_expert(idx)

    def n_experts(self) -> int:
        return len(self.expert_gate)


def expert_forward(x, gate_w, up_w, down_w, n_embd: int, expert_ffn_dim: int):
    """moe/mod.rs:134-145 (ops::ffn_swiglu) on the GPU through the F32 drop-ins.

    gate/up [n_embd, f] row-major are the transpose of GGUF [ne0=n_embd,
    ne1=f]; down [f, n_embd] row-major is GGUF [ne0=f, ne1=n_embd] as is.
    """
    g = np.ascontiguousarray(np.asarray(gate_w, np.float32).reshape(n_embd, expert_ffn_dim).T)
    u = np.ascontiguousarray(np.asarray(up_w, np.float32).reshape(n_embd, expert_ffn_dim).T)
    d = np.ascontiguousarray(np.asarray(down_w, np.float32).reshape(n_embd, expert_ffn_dim))
    out = np.zeros(n_embd, np.float32)
    quant.ffn_swiglu_q(out, np.asarray(x, np.float32), g.view(np.uint8), u.view(np.uint8), d.view(np.uint8),
                       PI_QT_F32, n_embd, expert_ffn_dim)
    return out


def moe_forward(x, router: MoeRouter, expert_provider, n_embd: int, expert_ffn_dim: int):
    """moe/mod.rs:193-219: route, run the k experts, weighted sum in routing order.

    The routing and every expert's SwiGLU run on the GPU (``pi_router_topk_softmax``,
    ``pi_ffn_swiglu_q``); like the reference, the caller's vector lives on the host, so
    the k-term weighted sum is done there in f32, multiply then add per term, in the
    routing order (moe/mod.rs:211-216)."""
    routing = router.route(x)
    out = np.zeros(n_embd, np.float32)
    for i, e in enumerate(routing.expert_indices):
        g, u, d = expert_provider.get_expert_f32(e)
        eo = expert_forward(x, g, u, d, n_embd, expert_ffn_dim)
        out = out + np.float32(routing.expert_weights[i]) * eo
    return out
