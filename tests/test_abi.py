"""CPU checks of the drop-in boundary: the C-ABI library loads and exports
every entry point include/pi_moe.h declares (no compute without a GPU)."""
import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def declared():
    src = (ROOT / "include" / "pi_moe.h").read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(pi_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared()
    for must in ("pi_ctx_create", "pi_matvec_col_major", "pi_ffn_swiglu_q_selected", "pi_moe_forward",
                 "pi_moe_route", "pi_sparse_ffn_forward", "pi_dequantize"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from powerinfer_x64_b200 import build

    lib_path = build.build()
    lib = ctypes.CDLL(str(lib_path))
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    from powerinfer_x64_b200._lib import SIGNATURES, lib

    assert sorted(SIGNATURES) == declared()
    L = lib()
    for n in SIGNATURES:
        assert getattr(L, n).argtypes is not None


def test_ctx_create_without_gpu_fails_cleanly():
    import torch

    if torch.cuda.is_available():
        return
    from powerinfer_x64_b200._lib import PiError, Context

    try:
        Context(0)
    except PiError as e:
        assert e.code != 0
    else:
        raise AssertionError("context creation should fail without a CUDA device")


def test_host_synth_matches_numpy_splitmix():
    """The host generator's SplitMix64 stream equals the numpy restatement."""
    import math

    import numpy as np
    from powerinfer_x64_b200 import synth

    vals = synth.normal_host(12345, 6, 1.0)
    u = synth.splitmix_at(12345, np.arange(6))
    for m in range(3):
        u1 = 1.0 - float(u[2 * m] >> np.uint64(11)) / 2.0 ** 53
        u2 = float(u[2 * m + 1] >> np.uint64(11)) / 2.0 ** 53
        r = math.sqrt(-2 * math.log(u1))
        assert np.float32(r * math.cos(2 * math.pi * u2)) == vals[2 * m]
        assert np.float32(r * math.sin(2 * math.pi * u2)) == vals[2 * m + 1]
