"""ctypes binding of ``libpi_moe.so`` (the C ABI declared in include/pi_moe.h).

The library is built in-tree (``powerinfer_x64_b200/_lib/libpi_moe.so``) by
``powerinfer_x64_b200.build``. There is no fallback: if the library is missing
or no CUDA device is present, every compute call raises.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libpi_moe.so"

PI_OK, PI_ERR_ARG, PI_ERR_INDEX, PI_ERR_SHORT, PI_ERR_OOM, PI_ERR_CUDA, PI_ERR_TIMEOUT = range(7)
PI_QT_F32, PI_QT_F16, PI_QT_Q4_0, PI_QT_Q8_0 = 0, 1, 2, 8
PI_EP_MAX_WORLD, PI_EP_HANDLE_BYTES = 64, 64
PI_FWD_RMSNORM, PI_FWD_RESIDUAL, PI_FWD_FORCE_GEMV, PI_FWD_FORCE_GEMM, PI_FWD_FAST_SUM = 1, 2, 4, 8, 16

_P = C.c_void_p
_I64 = C.c_int64
_I32 = C.c_int32
_INT = C.c_int


class PiError(RuntimeError):
    """A failed call into the C ABI; ``code`` is the PI_ERR_* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[pi status {code}] {msg}")
        self.code = code


class PiMoeLayerDesc(C.Structure):
    _fields_ = [
        ("n_embd", _I64), ("n_ff_exp", _I64), ("n_ff_shexp", _I64),
        ("n_expert", _I32), ("n_expert_used", _I32), ("qtype", _I32), ("src_on_host", _I32),
        ("router", _P), ("router_bias", _P),
        ("gate_exps", _P), ("up_exps", _P), ("down_exps", _P),
        ("gate_shexp", _P), ("up_shexp", _P), ("down_shexp", _P),
        ("gate_inp_shexp", _P),
    ]


# name -> (restype, argtypes); every symbol include/pi_moe.h declares.
SIGNATURES = {
    "pi_ctx_create": (_INT, [_INT, C.POINTER(_P)]),
    "pi_ctx_destroy": (None, [_P]),
    "pi_last_error": (C.c_char_p, [_P]),
    "pi_ctx_check": (_INT, [_P, _P]),
    "pi_ctx_reserve": (_INT, [_P, _P, C.c_uint64]),
    "pi_ctx_profile": (_INT, [_P, _INT]),
    "pi_ctx_profile_read": (_INT, [_P, _INT, C.c_char_p, C.POINTER(C.c_double), C.POINTER(_I64)]),
    "pi_dequantize": (_INT, [_P, _P, C.c_uint64, _INT, _I64, _I64, _P, _P]),
    "pi_quantize_q8_0": (_INT, [_P, _P, _I64, _P, _P]),
    "pi_quantize_q4_0": (_INT, [_P, _P, _I64, _P, _P]),
    "pi_matvec_col_major": (_INT, [_P, _P, _P, _P, _INT, _I64, _I64, _P]),
    "pi_matvec_col_major_q8_0_noalloc": (_INT, [_P, _P, _P, _I64, _I64, _P]),
    "pi_matvec_col_major_select": (_INT, [_P, _P, _P, _P, _INT, _I64, _I64, _P, _I64, _P]),
    "pi_matvec_col_major_sparse_input": (_INT, [_P, _P, _P, _P, _I64, _P, _INT, _I64, _I64, _P]),
    "pi_ffn_swiglu_q": (_INT, [_P, _P, _P, _P, _P, _P, _INT, _I64, _I64, _P]),
    "pi_ffn_swiglu_q_selected": (_INT, [_P, _P, _P, _P, _P, _P, _INT, _I64, _I64, _P, _I64, _P]),
    "pi_moe_layer_create": (_INT, [_P, C.POINTER(PiMoeLayerDesc), C.POINTER(_P)]),
    "pi_moe_layer_destroy": (None, [_P]),
    "pi_moe_route": (_INT, [_P, _P, _P, _I64, _P, _P, _P, _P, _P, _P]),
    "pi_moe_forward": (_INT, [_P, _P, _P, _I64, _P, _I32, _P]),
    "pi_moe_forward_routed": (_INT, [_P, _P, _P, _I64, _P, _I32, _P, _P, _P, _P, _P, _P]),
    "pi_moe_layer_create_ep": (_INT, [_P, C.POINTER(PiMoeLayerDesc), _I32, _I32, C.POINTER(_P)]),
    "pi_moe_ep_route": (_INT, [_P, _P, _P, _I64, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "pi_moe_experts_q8": (_INT, [_P, _P, _I64, _P, _P, _P, _P, _P]),
    "pi_moe_ep_combine": (_INT, [_P, _P, _P, _I64, _I32, _P, _P, _P, _P, _P, _P, _P]),
    "pi_router_topk_softmax": (_INT, [_P, _P, _I64, _P, _I64, _I32, _I32, _P, _P, _P]),
    "pi_ep_comm_create": (_INT, [_P, _I32, _I32, _I64, _I64, _I32, C.POINTER(_P)]),
    "pi_ep_comm_ipc_handle": (_INT, [_P, _P]),
    "pi_ep_comm_open": (_INT, [_P, _P]),
    "pi_ep_comm_destroy": (None, [_P]),
    "pi_moe_ep_forward": (_INT, [_P, _P, _P, _P, _I64, _P, _I32, _P]),
    "pi_ep_comm_debug_skip": (_INT, [_P, _I32]),
    "pi_sparse_ffn_create": (_INT, [_P, _P, _P, _P, _I32, _I64, _I64, _I32, C.POINTER(_P)]),
    "pi_sparse_ffn_destroy": (None, [_P]),
    "pi_sparse_ffn_forward": (_INT, [_P, _P, _P, _I64, _P, _P, _P, _P]),
    "pi_predictor_forward": (_INT, [_P, _P, _I64, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P]),
    "pi_hot_lists_from_probs": (_INT, [_P, _P, _I64, _I64, C.c_float, _I64, _I64, _P, _P, _P]),
    "pi_hot_lists_broadcast": (_INT, [_P, _P, _I64, _I64, _P, _P, _P]),
    "pi_synth_normal": (_INT, [_P, C.c_uint64, C.c_uint64, _I64, C.c_float, _P, _P]),
    "pi_synth_normal_host": (_INT, [C.c_uint64, C.c_uint64, _I64, C.c_float, _P]),
}

_lib = None
_lock = threading.Lock()


def lib() -> C.CDLL:
    """Loads the library (once). Raises if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise PiError(PI_ERR_CUDA, f"{LIB_PATH} is not built; run python -m powerinfer_x64_b200.build")
            L = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


class Context:
    """One CUDA device: wraps ``pi_ctx`` (error strings, per-stream scratch)."""

    _default: dict[int, "Context"] = {}

    def __init__(self, device: int = 0):
        self.device = device
        h = _P()
        rc = lib().pi_ctx_create(device, C.byref(h))
        if rc != PI_OK:
            raise PiError(rc, f"pi_ctx_create(device={device}) failed (no usable CUDA device?)")
        self.h = h

    @classmethod
    def default(cls, device: int | None = None) -> "Context":
        import torch

        if device is None:
            device = torch.cuda.current_device()
        with _lock:
            ctx = cls._default.get(device)
        if ctx is None:
            ctx = cls(device)
            with _lock:
                cls._default[device] = ctx
        return ctx

    def check(self, rc: int) -> None:
        if rc != PI_OK:
            msg = lib().pi_last_error(self.h)
            raise PiError(rc, msg.decode() if msg else "")

    def sync_check(self, stream=None) -> None:
        """Synchronises ``stream`` and raises on a device-side error (e.g. an index out of range)."""
        self.check(lib().pi_ctx_check(self.h, stream_ptr(stream)))

    def profile(self, enable: bool) -> None:
        """Starts (clearing previous totals) or stops per-kernel CUDA-event timing."""
        self.check(lib().pi_ctx_profile(self.h, 1 if enable else 0))

    def profile_read(self) -> dict:
        """{kernel name: (total ms, launches)} accumulated since profiling started."""
        n_max = 64
        names = C.create_string_buffer(32 * n_max)
        ms = (C.c_double * n_max)()
        cnt = (_I64 * n_max)()
        n = lib().pi_ctx_profile_read(self.h, n_max, names, ms, cnt)
        raw = names.raw
        return {raw[32 * i:32 * i + 32].split(b"\0")[0].decode(): (ms[i], int(cnt[i])) for i in range(min(n, n_max))}

    def __del__(self):
        try:
            if getattr(self, "h", None) and _lib is not None:
                _lib.pi_ctx_destroy(self.h)
        except Exception:
            pass


def stream_ptr(stream=None):
    """cudaStream_t of a torch stream (default: torch's current stream)."""
    import torch

    if stream is None:
        stream = torch.cuda.current_stream()
    return _P(stream.cuda_stream) if hasattr(stream, "cuda_stream") else _P(stream)


def ptr(t) -> _P:
    """Device pointer of a torch tensor (None -> NULL)."""
    if t is None:
        return _P(None)
    return _P(t.data_ptr())
