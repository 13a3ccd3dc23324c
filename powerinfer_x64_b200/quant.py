"""Host-side mirror of the reference's ``quant`` operator API (src/quant/mod.rs).

Each function keeps the reference's name, argument order and meaning, and its
error behaviour (an out-of-range index raises, like the reference's
``anyhow::Err``). Arguments may be host arrays (numpy / bytes; the output
array is filled in place like the Rust ``&mut [f32]``) or CUDA torch tensors
(the call is then asynchronous on torch's current stream and index errors are
reported by ``Context.sync_check``). All arithmetic runs in libpi_moe.so on the
GPU; there is no CPU path.
"""
from __future__ import annotations

import ctypes as C
import enum

import numpy as np

from ._lib import PI_QT_F16, PI_QT_F32, PI_QT_Q4_0, PI_QT_Q8_0, Context, PiError, PI_ERR_INDEX, PI_ERR_SHORT, lib, ptr, stream_ptr


class QuantizationType(enum.IntEnum):
    """GGML tensor types on this path (quant/mod.rs:12-40); values are ggml_type ids."""

    F32 = PI_QT_F32
    F16 = PI_QT_F16
    Q4_0 = PI_QT_Q4_0
    Q8_0 = PI_QT_Q8_0

    def block_size_bytes(self) -> int:  # quant/mod.rs:72-88
        return {self.F32: 4, self.F16: 2, self.Q4_0: 18, self.Q8_0: 34}[self]

    def values_per_block(self) -> int:  # quant/mod.rs:91-104
        return 1 if self in (self.F32, self.F16) else 32


def raw_nbytes(qtype: int, n: int) -> int:
    q = QuantizationType(qtype)
    return n // q.values_per_block() * q.block_size_bytes()


# --------------------------------------------------------------------------
# argument staging
# --------------------------------------------------------------------------
def _torch():
    import torch

    return torch


def _is_dev(a) -> bool:
    return hasattr(a, "is_cuda") and a.is_cuda


def _dev(a, dtype):
    """Device tensor view of a host array / bytes / device tensor."""
    torch = _torch()
    if a is None:
        return None
    if _is_dev(a):
        return a
    if isinstance(a, (bytes, bytearray, memoryview)):
        a = np.frombuffer(a, dtype=np.uint8)
    arr = np.ascontiguousarray(np.asarray(a, dtype=dtype))
    if not arr.flags.writeable:  # e.g. a window of a read-only memory map: upload a copy
        arr = arr.copy()
    return torch.from_numpy(arr).cuda()


def _u8(a):
    return _dev(a, np.uint8)


def _f32(a):
    return _dev(a, np.float32)


def _i64(a):
    return _dev(a, np.int64)


class _Call:
    """Runs one C-ABI call on device buffers and writes host outputs back."""

    def __init__(self):
        self.ctx = Context.default()
        self.host_out = []

    def out(self, y, n):
        torch = _torch()
        if _is_dev(y):
            return y
        t = torch.empty(n, dtype=torch.float32, device="cuda")
        self.host_out.append((y, t))
        return t

    def finish(self, rc, sync=False):
        self.ctx.check(rc)
        if self.host_out or sync:
            self.ctx.sync_check()
        for host, dev in self.host_out:
            host[...] = dev.cpu().numpy().reshape(host.shape)


def _check_indices_host(indices, limit, what):
    if _is_dev(indices):
        return
    arr = np.asarray(indices, dtype=np.int64)
    bad = np.nonzero((arr < 0) | (arr >= limit))[0]
    if bad.size:
        raise PiError(PI_ERR_INDEX, f"{what} {int(arr[bad[0]])} out of range for width {limit}")


# --------------------------------------------------------------------------
# operators
# --------------------------------------------------------------------------
def dequantize(data, qtype, rows: int, cols: int):
    """quant::dequantize (quant/mod.rs:110-143) -> float32 array of rows*cols."""
    call = _Call()
    raw = _u8(data)
    n = rows * cols
    out = _torch().empty(n, dtype=_torch().float32, device="cuda")
    rc = lib().pi_dequantize(call.ctx.h, ptr(raw), raw.numel(), int(qtype), rows, cols, ptr(out), stream_ptr())
    if rc == PI_ERR_SHORT:
        call.ctx.check(rc)
    call.finish(rc)
    return out if _is_dev(data) else out.cpu().numpy()


def quantize_q8_0(x):
    """GGUF Q8_0 bytes of x with the reference's quantiser (quant/mod.rs:698-736)."""
    call = _Call()
    xd = _f32(x)
    out = _torch().empty(raw_nbytes(PI_QT_Q8_0, xd.numel()), dtype=_torch().uint8, device="cuda")
    call.finish(lib().pi_quantize_q8_0(call.ctx.h, ptr(xd), xd.numel(), ptr(out), stream_ptr()))
    return out if _is_dev(x) else out.cpu().numpy()


def quantize_q4_0(x):
    """GGUF Q4_0 bytes (ggml-style quantiser, reference nibble order)."""
    call = _Call()
    xd = _f32(x)
    out = _torch().empty(raw_nbytes(PI_QT_Q4_0, xd.numel()), dtype=_torch().uint8, device="cuda")
    call.finish(lib().pi_quantize_q4_0(call.ctx.h, ptr(xd), xd.numel(), ptr(out), stream_ptr()))
    return out if _is_dev(x) else out.cpu().numpy()


def matvec_col_major(y, x, raw, qtype, n_in: int, n_out: int) -> None:
    """quant::matvec_col_major (quant/mod.rs:939-970): y[j] = x . W[:, j]."""
    call = _Call()
    yd = call.out(y, n_out)
    xd, rd = _f32(x), _u8(raw)  # keep the device copies alive until the launch is queued
    rc = lib().pi_matvec_col_major(call.ctx.h, ptr(yd), ptr(xd), ptr(rd), int(qtype), n_in, n_out, stream_ptr())
    call.finish(rc)


def matvec_col_major_select(y, x, raw, qtype, n_in: int, n_out: int, indices) -> None:
    """quant::matvec_col_major_select (quant/mod.rs:974-1068)."""
    if len(indices) == 0:
        return
    _check_indices_host(indices, n_out, "selected column")
    call = _Call()
    idx = _i64(indices)
    yd = call.out(y, idx.numel())
    xd, rd = _f32(x), _u8(raw)
    rc = lib().pi_matvec_col_major_select(call.ctx.h, ptr(yd), ptr(xd), ptr(rd), int(qtype), n_in, n_out,
                                          ptr(idx), idx.numel(), stream_ptr())
    call.finish(rc, sync=not _is_dev(y))


def matvec_col_major_sparse_input(y, x, indices, raw, qtype, n_in: int, n_out: int) -> None:
    """quant::matvec_col_major_sparse_input (quant/mod.rs:1073-1169)."""
    _check_indices_host(indices, n_in, "sparse input index")
    call = _Call()
    yd = call.out(y, n_out)
    idx = _i64(indices) if len(indices) else None
    n_idx = 0 if idx is None else idx.numel()
    xd = _f32(x) if n_idx else None
    rd = _u8(raw)
    rc = lib().pi_matvec_col_major_sparse_input(call.ctx.h, ptr(yd), ptr(xd), ptr(idx), n_idx, ptr(rd),
                                                int(qtype), n_in, n_out, stream_ptr())
    call.finish(rc, sync=not _is_dev(y))


def ffn_swiglu_q(out, x, gate_raw, up_raw, down_raw, qtype, n_embd: int, n_ff: int) -> None:
    """quant::ffn_swiglu_q (quant/mod.rs:1179-1204)."""
    call = _Call()
    od = call.out(out, n_embd)
    xd, g, u, d = _f32(x), _u8(gate_raw), _u8(up_raw), _u8(down_raw)
    rc = lib().pi_ffn_swiglu_q(call.ctx.h, ptr(od), ptr(xd), ptr(g), ptr(u), ptr(d), int(qtype), n_embd, n_ff,
                               stream_ptr())
    call.finish(rc)


def ffn_swiglu_q_selected(out, x, gate_raw, up_raw, down_raw, qtype, n_embd: int, n_ff: int,
                          selected_indices) -> None:
    """quant::ffn_swiglu_q_selected (quant/mod.rs:1208-1249)."""
    if len(selected_indices) < n_ff:
        _check_indices_host(selected_indices, n_ff, "selected column")
    call = _Call()
    od = call.out(out, n_embd)
    idx = _i64(selected_indices) if len(selected_indices) else None
    n_idx = 0 if idx is None else idx.numel()
    xd, g, u, d = _f32(x), _u8(gate_raw), _u8(up_raw), _u8(down_raw)
    rc = lib().pi_ffn_swiglu_q_selected(call.ctx.h, ptr(od), ptr(xd), ptr(g), ptr(u), ptr(d), int(qtype), n_embd,
                                        n_ff, ptr(idx), n_idx, stream_ptr())
    call.finish(rc, sync=not _is_dev(out))
