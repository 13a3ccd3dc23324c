"""GPU check of the allocation-free Q8_0 matvec entry point.

pi_matvec_col_major_q8_0_noalloc serves callers that cannot allocate device
memory at call time (their allocator owns the device memory, or they must not
call cudaMalloc on the hot path): it keeps its scratch in a fixed device array
instead. Its output must equal the regular entry point's, on two calls in a
row through the shared array. This file sorts last so that a run stopping at
its first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_noalloc_matches_matvec_col_major_twice(orc):
    import torch

    from powerinfer_x64_b200 import build

    build.build()
    from powerinfer_x64_b200._lib import PI_OK, PI_QT_Q8_0, Context, lib, ptr, stream_ptr
    from test_gpu_parity import close

    ctx = Context.default()
    rng = np.random.default_rng(21)
    for n_in, n_out in ((2048, 512), (4096, 333)):  # second call reuses the array with a larger, ragged shape
        w = (rng.standard_normal(n_in * n_out) * 0.02).astype(np.float32)
        raw = torch.from_numpy(orc.quantize_q8_0(w)).cuda()
        x = torch.from_numpy(rng.standard_normal(n_in).astype(np.float32)).cuda()
        y_ref = torch.empty(n_out, dtype=torch.float32, device="cuda")
        y_new = torch.full((n_out,), float("nan"), dtype=torch.float32, device="cuda")
        ctx.check(lib().pi_matvec_col_major(ctx.h, ptr(y_ref), ptr(x), ptr(raw), PI_QT_Q8_0, n_in, n_out,
                                            stream_ptr()))
        rc = lib().pi_matvec_col_major_q8_0_noalloc(ptr(y_new), ptr(x), ptr(raw), n_in, n_out, stream_ptr())
        assert rc == PI_OK
        torch.cuda.synchronize()
        close(y_new.cpu().numpy(), y_ref.cpu().numpy())


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import torch

    from powerinfer_x64_b200 import build

    build.build()
    from powerinfer_x64_b200._lib import PI_ERR_ARG, lib

    p = C.c_void_p(torch.empty(1, device="cuda").data_ptr())
    assert lib().pi_matvec_col_major_q8_0_noalloc(p, p, p, 16384 + 32, 1, None) == PI_ERR_ARG
    assert lib().pi_matvec_col_major_q8_0_noalloc(p, p, p, 100, 1, None) == PI_ERR_ARG
