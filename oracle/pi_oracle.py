"""ctypes binding of the CPU oracle (oracle/pi_oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference legs, never by the product package.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libpi_oracle.so"

QT_F32, QT_F16, QT_Q4_0, QT_Q8_0 = 0, 1, 2, 8


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        _lib = C.CDLL(str(LIB))
        _lib.or_f16_to_f32.restype = C.c_float
        _lib.or_f16_to_f32.argtypes = [C.c_uint16]
        _lib.or_f32_to_f16.restype = C.c_uint16
        _lib.or_f32_to_f16.argtypes = [C.c_float]
    return _lib


class OrMoeLayer(C.Structure):
    _fields_ = [("d", C.c_int64), ("f", C.c_int64), ("f_sh", C.c_int64), ("E", C.c_int), ("k", C.c_int),
                ("qtype", C.c_int), ("router", C.c_void_p), ("bias", C.c_void_p), ("gate_exps", C.c_void_p),
                ("up_exps", C.c_void_p), ("down_exps", C.c_void_p), ("gate_sh", C.c_void_p),
                ("up_sh", C.c_void_p), ("down_sh", C.c_void_p), ("shared_gate", C.c_void_p)]


def _p(a):
    return C.c_void_p(None) if a is None else C.c_void_p(a.ctypes.data)


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, np.float32))


def _u8(a):
    if isinstance(a, (bytes, bytearray)):
        return np.frombuffer(a, np.uint8)
    return np.ascontiguousarray(np.asarray(a, np.uint8))


def _i64(a):
    return np.ascontiguousarray(np.asarray(a, np.int64))


def set_threads(n: int) -> None:
    lib().or_set_threads(C.c_int(n))


def set_scalar(on: bool) -> None:
    lib().or_set_scalar(C.c_int(1 if on else 0))


def f16_to_f32(h: int) -> float:
    return lib().or_f16_to_f32(h)


def f32_to_f16(x: float) -> int:
    return lib().or_f32_to_f16(x)


def quantize_q8_0(x) -> np.ndarray:
    x = _f32(x)
    out = np.empty(x.size // 32 * 34, np.uint8)
    lib().or_quantize_q8_0(_p(x), C.c_int64(x.size), _p(out))
    return out


def quantize_q4_0(x) -> np.ndarray:
    x = _f32(x)
    out = np.empty(x.size // 32 * 18, np.uint8)
    lib().or_quantize_q4_0(_p(x), C.c_int64(x.size), _p(out))
    return out


def quantize_act_q8_0(x):
    x = _f32(x)
    nb = (x.size + 31) // 32
    sc = np.empty(nb, np.float32)
    q = np.empty(nb * 32, np.int8)
    lib().or_quantize_act_q8_0(_p(x), C.c_int64(x.size), _p(sc), _p(q))
    return sc, q


def dequantize(raw, qtype, rows, cols, raw_len=None):
    raw = _u8(raw)
    out = np.empty(rows * cols, np.float32)
    rc = lib().or_dequantize(_p(raw), C.c_int64(raw.size if raw_len is None else raw_len), C.c_int(qtype),
                             C.c_int64(rows), C.c_int64(cols), _p(out))
    if rc:
        raise ValueError(f"dequantize failed ({rc})")
    return out


def matvec_col_major(x, raw, qtype, n_in, n_out):
    y = np.empty(n_out, np.float32)
    rc = lib().or_matvec_col_major(_p(y), _p(_f32(x)), _p(_u8(raw)), C.c_int(qtype), C.c_int64(n_in),
                                   C.c_int64(n_out))
    if rc:
        raise ValueError(rc)
    return y


def matvec_col_major_select(x, raw, qtype, n_in, n_out, idx):
    idx = _i64(idx)
    y = np.empty(idx.size, np.float32)
    rc = lib().or_matvec_col_major_select(_p(y), _p(_f32(x)), _p(_u8(raw)), C.c_int(qtype), C.c_int64(n_in),
                                          C.c_int64(n_out), _p(idx), C.c_int64(idx.size))
    if rc:
        raise IndexError(rc)
    return y


def matvec_col_major_sparse_input(x, idx, raw, qtype, n_in, n_out):
    idx = _i64(idx)
    y = np.empty(n_out, np.float32)
    rc = lib().or_matvec_col_major_sparse_input(_p(y), _p(_f32(x)), _p(idx), C.c_int64(idx.size), _p(_u8(raw)),
                                                C.c_int(qtype), C.c_int64(n_in), C.c_int64(n_out))
    if rc:
        raise IndexError(rc)
    return y


def ffn_swiglu_q(x, g, u, d, qtype, n_embd, n_ff):
    out = np.empty(n_embd, np.float32)
    rc = lib().or_ffn_swiglu_q(_p(out), _p(_f32(x)), _p(_u8(g)), _p(_u8(u)), _p(_u8(d)), C.c_int(qtype),
                               C.c_int64(n_embd), C.c_int64(n_ff))
    if rc:
        raise ValueError(rc)
    return out


def ffn_swiglu_q_selected(x, g, u, d, qtype, n_embd, n_ff, idx):
    idx = _i64(idx)
    out = np.empty(n_embd, np.float32)
    rc = lib().or_ffn_swiglu_q_selected(_p(out), _p(_f32(x)), _p(_u8(g)), _p(_u8(u)), _p(_u8(d)), C.c_int(qtype),
                                        C.c_int64(n_embd), C.c_int64(n_ff), _p(idx), C.c_int64(idx.size))
    if rc:
        raise IndexError(rc)
    return out


def moe_route(x, router, d, E, k, bias=None, threads=0):
    """Routing of T tokens (model/mod.rs:1254-1312); threads: 0 = all host cores."""
    x = _f32(x).reshape(-1, d)
    T = x.shape[0]
    router, bias = _f32(router), (None if bias is None else _f32(bias))
    logits = np.empty((T, E), np.float32)
    idx = np.empty((T, k), np.int32)
    gates = np.empty((T, k), np.float32)
    counts = np.empty(E, np.int32)
    offsets = np.empty(E, np.int32)
    perm = np.empty(T * k, np.int32)
    lib().or_moe_route_mt(_p(x), C.c_int64(T), _p(router), _p(bias), C.c_int64(d), C.c_int(E), C.c_int(k),
                          _p(logits), _p(idx), _p(gates), _p(counts), _p(offsets), _p(perm), C.c_int(threads))
    return dict(logits=logits, idx=idx, gates=gates, counts=counts, offsets=offsets, perm=perm)


def moe_layer(x, d, f, E, k, qtype, router, gate_exps, up_exps, down_exps, shared=None, bias=None, threads=1,
              residual=False, rmsnorm=False, eps=1e-6, token_threads=None):
    """Full MoE layer on T tokens (one at a time, as the reference).

    threads: 1 = single thread, 0 = the reference's own threading per token.
    token_threads: if given, tokens are spread over that many host threads
    (0 = all cores), each running the single-threaded path (same outputs)."""
    x = _f32(x).reshape(-1, d)
    keep = [_f32(router), _u8(gate_exps), _u8(up_exps), _u8(down_exps)]
    L = OrMoeLayer(d=d, f=f, f_sh=f, E=E, k=k, qtype=qtype)
    L.router, L.gate_exps, L.up_exps, L.down_exps = [_p(a) for a in keep]
    if bias is not None:
        b = _f32(bias)
        keep.append(b)
        L.bias = _p(b)
    if shared is not None:
        g, u, dn, gi = shared
        sh = [_u8(g), _u8(u), _u8(dn)] + ([_f32(gi)] if gi is not None else [])
        keep += sh
        L.gate_sh, L.up_sh, L.down_sh = _p(sh[0]), _p(sh[1]), _p(sh[2])
        if gi is not None:
            L.shared_gate = _p(sh[3])
    out = np.empty_like(x)
    if token_threads is not None:
        rc = lib().or_moe_layer_mt(C.byref(L), _p(x), C.c_int64(x.shape[0]), _p(out), C.c_int(1 if residual else 0),
                                   C.c_int(1 if rmsnorm else 0), C.c_float(eps), C.c_int(token_threads))
    else:
        rc = lib().or_moe_layer(C.byref(L), _p(x), C.c_int64(x.shape[0]), _p(out), C.c_int(threads),
                                C.c_int(1 if residual else 0), C.c_int(1 if rmsnorm else 0), C.c_float(eps))
    if rc:
        raise ValueError(rc)
    return out


def rms_norm(x, w, eps=1e-6):
    x, w = _f32(x), _f32(w)
    out = np.empty_like(x)
    lib().or_rms_norm(_p(out), _p(x), _p(w), C.c_int64(x.size), C.c_float(eps))
    return out


def sparse_ffn(x, g, u, dn, qtype, n_embd, n_ff, lists):
    x = _f32(x).reshape(-1, n_embd)
    T = x.shape[0]
    ptr = np.zeros(T + 1, np.int64)
    for t, l in enumerate(lists):
        ptr[t + 1] = ptr[t] + len(l)
    idx = np.concatenate([_i64(l) for l in lists]) if ptr[-1] else np.zeros(1, np.int64)
    out = np.empty_like(x)
    rc = lib().or_sparse_ffn(_p(x), C.c_int64(T), _p(_u8(g)), _p(_u8(u)), _p(_u8(dn)), C.c_int(qtype),
                             C.c_int64(n_embd), C.c_int64(n_ff), _p(ptr), _p(idx), _p(out))
    if rc:
        raise IndexError(rc)
    return out


def predictor(a, W1, b1, W2, b2):
    a, W1, b1, W2, b2 = map(_f32, (a, W1, b1, W2, b2))
    n_hidden, n_in = W1.shape
    n_out = W2.shape[0]
    probs = np.empty(n_out, np.float32)
    lib().or_predictor(_p(a), _p(W1), _p(b1), _p(W2), _p(b2), C.c_int64(n_in), C.c_int64(n_hidden),
                       C.c_int64(n_out), _p(probs))
    return probs


def moe_api_route(x, gate, d, E, k, threads=0):
    """MoeRouter::route (moe/mod.rs:69-108) for T tokens over a row-major [d, E]
    gate: (indices [T, k] in descending-logit order, softmax weights [T, k])."""
    x = _f32(x).reshape(-1, d)
    T = x.shape[0]
    g = _f32(gate)
    idx = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    lib().or_moe_api_route(_p(x), C.c_int64(T), _p(g), C.c_int64(d), C.c_int(E), C.c_int(k), _p(idx), _p(w),
                           C.c_int(threads))
    return idx, w


# ---------------------------------------------------------------------------
# Host-side synthetic inputs (the benchmark's seeded generator, restated so the
# CPU legs never load the GPU library): one SplitMix64 stream per tensor, stream
# seed = SplitMix64 output `tensor id` of (config seed + 7919 * layer).
# ---------------------------------------------------------------------------
_GAMMA = np.uint64(0x9E3779B97F4A7C15)
TENSOR_IDS = dict(router=1, gate_exps=2, up_exps=3, down_exps=4, gate_shexp=5, up_shexp=6, down_shexp=7,
                  gate_inp_shexp=8, x=9, bias=10, mask=11)


def splitmix_at(seed: int, j):
    with np.errstate(over="ignore"):
        j = np.asarray(j, dtype=np.uint64)
        z = np.uint64(seed) + (j + np.uint64(1)) * _GAMMA
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def stream_seed(seed: int, name: str, layer: int = 0) -> int:
    return int(splitmix_at(seed + 7919 * layer, TENSOR_IDS[name]))


def synth_normal(seed: int, n: int, std: float, offset: int = 0, threads: int = 0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().or_synth_normal(C.c_uint64(seed), C.c_uint64(offset), C.c_int64(n), C.c_float(std), _p(out),
                          C.c_int(threads))
    return out


def synth_quant(seed: int, n_mats: int, rows: int, cols: int, qtype: int, std: float = 0.02,
                threads: int = 0) -> np.ndarray:
    out = np.empty(n_mats * rows * cols // 32 * (34 if qtype == QT_Q8_0 else 18), np.uint8)
    lib().or_synth_quant(C.c_uint64(seed), C.c_int64(n_mats), C.c_int64(rows), C.c_int64(cols), C.c_int(qtype),
                         C.c_float(std), _p(out), C.c_int(threads))
    return out


def zipf_bias(seed: int, E: int) -> np.ndarray:
    keys = splitmix_at(stream_seed(seed, "bias"), np.arange(E))
    rank = np.empty(E, np.int64)
    rank[np.argsort(keys, kind="stable")] = np.arange(E)
    return (2.0 * np.log(1.0 / (rank + 1.0))).astype(np.float32)


def moe_tensors_host(d, E, f, qtype, shared, zipf=False, seed=0, layer=0):
    """Host GGUF tensors of one synthetic MoE layer: the same streams the GPU
    generator draws for (seed, layer)."""
    s = lambda n: stream_seed(seed, n, layer)
    t = dict(router=synth_normal(s("router"), E * d, 0.02),
             gate_exps=synth_quant(s("gate_exps"), E, f, d, qtype),
             up_exps=synth_quant(s("up_exps"), E, f, d, qtype),
             down_exps=synth_quant(s("down_exps"), E, d, f, qtype),
             shared=None, router_bias=zipf_bias(seed, E) if zipf else None)
    if shared:
        t["shared"] = (synth_quant(s("gate_shexp"), 1, f, d, qtype), synth_quant(s("up_shexp"), 1, f, d, qtype),
                       synth_quant(s("down_shexp"), 1, d, f, qtype), synth_normal(s("gate_inp_shexp"), d, 0.02))
    return t
