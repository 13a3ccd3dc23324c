"""B200-native (sm_100a) MoE feed-forward and hot-neuron sparse-FFN path for
PowerInfer_x64, behind the reference's quant / moe / predictor operator APIs.

Compute runs in ``_lib/libpi_moe.so`` (hand-written CUDA kernels, C ABI in
include/pi_moe.h). Submodules: ``quant``, ``moe``, ``predictor``, ``synth``.
"""
from ._lib import PiError, Context, LIB_PATH  # noqa: F401

__all__ = ["PiError", "Context", "LIB_PATH", "quant", "moe", "predictor", "synth"]
