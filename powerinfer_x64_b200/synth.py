"""Seeded synthetic inputs for the benchmark configurations.

The reference publishes no dataset for this path; every configuration is
synthetic (weights N(0, 0.02) quantised with the repo's own quantisers,
activations N(0, 1)). Values come from SplitMix64 (the generator in the
reference, model/mod.rs:2041-2061) + Box-Muller, one independent stream per
tensor: stream seed = SplitMix64 output ``tensor_id`` of the config seed.

Large tensors are generated and quantised on the GPU (pi_synth_normal +
pi_quantize_*); ``host=True`` uses the host generator (for small fixtures).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from ._lib import PI_QT_Q4_0, PI_QT_Q8_0, Context, lib, ptr, stream_ptr

GAMMA = np.uint64(0x9E3779B97F4A7C15)
TENSOR_IDS = dict(router=1, gate_exps=2, up_exps=3, down_exps=4, gate_shexp=5, up_shexp=6, down_shexp=7,
                  gate_inp_shexp=8, x=9, bias=10, mask=11)


def splitmix_at(seed: int, j):
    """Output j (0-based) of SplitMix64 seeded with ``seed`` (vectorised over j)."""
    with np.errstate(over="ignore"):
        j = np.asarray(j, dtype=np.uint64)
        z = np.uint64(seed) + (j + np.uint64(1)) * GAMMA
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def stream_seed(seed: int, name: str, layer: int = 0) -> int:
    return int(splitmix_at(seed + 7919 * layer, TENSOR_IDS[name]))


@dataclass
class MoeConfig:
    name: str
    d: int
    E: int
    k: int
    f: int
    qtype: int
    shared: bool
    T: list
    zipf_bias: bool = False
    layers: int = 1
    rmsnorm: bool = False
    residual: bool = False
    seeds: list = field(default_factory=lambda: [0])


# BASELINE configs 1, 2, 3, 5 (MoE) and 4 (hot-neuron sparse FFN)
C1 = MoeConfig("c1_tiny_q8", d=1024, E=64, k=4, f=256, qtype=PI_QT_Q8_0, shared=False, T=[16])
C2 = MoeConfig("c2_decode_q8", d=2048, E=256, k=8, f=512, qtype=PI_QT_Q8_0, shared=True, T=[1, 4, 16, 64],
               seeds=[0, 1, 2, 3])
C3 = MoeConfig("c3_prefill_q4", d=2048, E=256, k=8, f=512, qtype=PI_QT_Q4_0, shared=True, T=[512, 2048, 4096],
               zipf_bias=True)
C5 = MoeConfig("c5_stack_q8", d=2048, E=256, k=8, f=512, qtype=PI_QT_Q8_0, shared=True, T=[8192], layers=40,
               rmsnorm=True, residual=True)


@dataclass
class SparseConfig:
    name: str = "c4_sparse_q4"
    d: int = 4096
    F: int = 12288
    qtype: int = PI_QT_Q4_0
    T: tuple = (1, 8)
    active_frac: float = 0.15
    hot_frac: float = 0.20
    hot_share: float = 0.80


C4 = SparseConfig()


def _torch():
    import torch

    return torch


def normal_dev(seed: int, n: int, std: float, out=None):
    torch = _torch()
    ctx = Context.default()
    if out is None:
        out = torch.empty(n, dtype=torch.float32, device="cuda")
    ctx.check(lib().pi_synth_normal(ctx.h, seed, 0, n, std, ptr(out), stream_ptr()))
    return out


def normal_host(seed: int, n: int, std: float) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().pi_synth_normal_host(seed, 0, n, std, out.ctypes.data)
    return out


def quantize_dev(x, qtype: int):
    torch = _torch()
    ctx = Context.default()
    n = x.numel()
    nb = n // 32 * (34 if qtype == PI_QT_Q8_0 else 18)
    out = torch.empty(nb, dtype=torch.uint8, device="cuda")
    fn = lib().pi_quantize_q8_0 if qtype == PI_QT_Q8_0 else lib().pi_quantize_q4_0
    ctx.check(fn(ctx.h, ptr(x), n, ptr(out), stream_ptr()))
    return out


def quant_weights_dev(seed: int, n_mats: int, rows: int, cols: int, qtype: int, std: float = 0.02):
    """GGUF bytes of n_mats [rows x cols] matrices ~ N(0, std) (generated matrix by matrix)."""
    torch = _torch()
    per = rows * cols
    bpm = per // 32 * (34 if qtype == PI_QT_Q8_0 else 18)
    out = torch.empty(n_mats * bpm, dtype=torch.uint8, device="cuda")
    chunk = max(1, (1 << 28) // per)  # <= 1 GiB of f32 at a time
    ctx = Context.default()
    buf = torch.empty(chunk * per, dtype=torch.float32, device="cuda")
    for m0 in range(0, n_mats, chunk):
        m = min(chunk, n_mats - m0)
        ctx.check(lib().pi_synth_normal(ctx.h, seed, m0 * per, m * per, std, ptr(buf), stream_ptr()))
        fn = lib().pi_quantize_q8_0 if qtype == PI_QT_Q8_0 else lib().pi_quantize_q4_0
        ctx.check(fn(ctx.h, ptr(buf), m * per, ptr(out[m0 * bpm:(m0 + m) * bpm]), stream_ptr()))
    return out


def zipf_bias(seed: int, E: int) -> np.ndarray:
    """b_e = 2 ln(1/(rank_e + 1)), rank = a seeded permutation of 0..E-1."""
    keys = splitmix_at(stream_seed(seed, "bias"), np.arange(E))
    rank = np.empty(E, np.int64)
    rank[np.argsort(keys, kind="stable")] = np.arange(E)
    return (2.0 * np.log(1.0 / (rank + 1.0))).astype(np.float32)


def moe_tensors(cfg: MoeConfig, seed: int = 0, layer: int = 0):
    """Device tensors of one MoE layer of ``cfg`` (GGUF layout)."""
    torch = _torch()
    s = lambda n: stream_seed(seed, n, layer)
    t = dict(
        router=normal_dev(s("router"), cfg.E * cfg.d, 0.02),
        gate_exps=quant_weights_dev(s("gate_exps"), cfg.E, cfg.f, cfg.d, cfg.qtype),
        up_exps=quant_weights_dev(s("up_exps"), cfg.E, cfg.f, cfg.d, cfg.qtype),
        down_exps=quant_weights_dev(s("down_exps"), cfg.E, cfg.d, cfg.f, cfg.qtype),
    )
    if cfg.shared:
        t["shared"] = (quant_weights_dev(s("gate_shexp"), 1, cfg.f, cfg.d, cfg.qtype),
                       quant_weights_dev(s("up_shexp"), 1, cfg.f, cfg.d, cfg.qtype),
                       quant_weights_dev(s("down_shexp"), 1, cfg.d, cfg.f, cfg.qtype),
                       normal_dev(s("gate_inp_shexp"), cfg.d, 0.02))
    t["router_bias"] = torch.from_numpy(zipf_bias(seed, cfg.E)).cuda() if cfg.zipf_bias else None
    return t


def moe_layer(cfg: MoeConfig, seed: int = 0, layer: int = 0, keep_tensors: bool = False):
    from .moe import MoeLayer

    t = moe_tensors(cfg, seed, layer)
    L = MoeLayer(t["router"], t["gate_exps"], t["up_exps"], t["down_exps"], cfg.qtype, cfg.d, cfg.f, cfg.E, cfg.k,
                 shared=t.get("shared"), router_bias=t["router_bias"])
    return (L, t) if keep_tensors else L


def tokens_dev(cfg_d: int, T: int, seed: int = 0, layer: int = 0):
    return normal_dev(stream_seed(seed, "x", layer), T * cfg_d, 1.0).view(T, cfg_d)


def sparse_masks(cfg: SparseConfig, T: int, seed: int = 0):
    """Per-token ascending neuron lists: active_frac of F per token, hot_share of
    them from a fixed seeded hot subset of hot_frac * F neurons."""
    F = cfg.F
    ms = stream_seed(seed, "mask")
    order = np.argsort(splitmix_at(ms, np.arange(F)), kind="stable")
    n_hot = int(round(cfg.hot_frac * F))
    hot, cold = np.sort(order[:n_hot]), np.sort(order[n_hot:])
    n_act = int(round(cfg.active_frac * F))
    n_from_hot = int(round(cfg.hot_share * n_act))
    n_from_cold = n_act - n_from_hot
    lists = []
    for t in range(T):
        kh = splitmix_at(ms + 1 + 2 * t, np.arange(hot.size))
        kc = splitmix_at(ms + 2 + 2 * t, np.arange(cold.size))
        sel = np.concatenate([hot[np.argsort(kh, kind="stable")[:n_from_hot]],
                              cold[np.argsort(kc, kind="stable")[:n_from_cold]]])
        lists.append(np.sort(sel).astype(np.int64))
    return lists


def sparse_tensors(cfg: SparseConfig, seed: int = 0):
    s = lambda n: stream_seed(seed, n)
    return dict(gate=quant_weights_dev(s("gate_exps"), 1, cfg.F, cfg.d, cfg.qtype),
                up=quant_weights_dev(s("up_exps"), 1, cfg.F, cfg.d, cfg.qtype),
                down=quant_weights_dev(s("down_exps"), 1, cfg.d, cfg.F, cfg.qtype))
