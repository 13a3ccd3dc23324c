"""Resident projection / LM-head matvec with its rows split over GPUs.

The reference's only GPU use uploads the LM head (f32, row-major
``[n_out][n_in]``) once and gives each GPU a contiguous slice of
``ceil(n_out / n_gpus)`` output rows; every call runs each slice's matvec and
assembles the logits (src/cuda/mod.rs:462-537, ``upload_lm_head`` /
``try_lm_head_matvec``). Here the weights stay in their GGUF encoding (F32,
Q8_0 or Q4_0 rows of ``n_in`` values, the layout ``quant::matvec_col_major``
reads, src/quant/mod.rs:939-970), one slice per rank (one process per GPU);
each rank runs ``pi_matvec_col_major`` over its resident slice for a batch of
tokens and, with more than one rank, the slices are all-gathered into the full
logits. With one rank the whole matrix is resident on the one GPU.
"""
from __future__ import annotations

import numpy as np

from . import quant
from ._lib import Context, lib, ptr, stream_ptr


def lm_head_slices(n_out: int, n_gpus: int):
    """[(row_start, n_rows)] per GPU: ceil(n_out / n_gpus) rows each, the last
    GPUs possibly short or empty (src/cuda/mod.rs:475-486)."""
    per = -(-n_out // n_gpus) if n_gpus else 0
    out = []
    for g in range(n_gpus):
        lo = min(g * per, n_out)
        hi = min(lo + per, n_out)
        out.append((lo, hi - lo))
    return out


class LmHead:
    """One rank's resident slice of a ``[n_out][n_in]`` projection.

    raw:   the whole matrix's GGUF bytes (host bytes / numpy, or a CUDA uint8 tensor),
           rows of n_in values in ``qtype`` encoding;
    rank, world: this process's slice; ``group`` the process group for the gather
           (the default group when world > 1).
    """

    def __init__(self, raw, qtype: int, n_out: int, n_in: int, rank: int = 0, world: int = 1, device=None,
                 group=None):
        import torch

        self.qtype, self.n_out, self.n_in, self.rank, self.world, self.group = int(qtype), n_out, n_in, rank, world, group
        self.dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        self.ctx = Context.default(self.dev.index)
        self.slices = lm_head_slices(n_out, world)
        self.row_start, self.n_rows = self.slices[rank]
        row_b = quant.raw_nbytes(self.qtype, n_in)
        lo, hi = self.row_start * row_b, (self.row_start + self.n_rows) * row_b
        if hasattr(raw, "is_cuda"):
            part = raw.reshape(-1)[lo:hi]
            self.w = part.to(self.dev, dtype=torch.uint8).contiguous()
        else:
            buf = np.frombuffer(raw, np.uint8) if isinstance(raw, (bytes, bytearray, memoryview)) else \
                np.asarray(raw).reshape(-1).view(np.uint8)
            if buf.size < n_out * row_b:
                raise ValueError(f"lm head: {buf.size} bytes for {n_out} rows of {row_b}")
            self.w = torch.from_numpy(np.ascontiguousarray(buf[lo:hi])).to(self.dev)

    def forward_local(self, x, out=None):
        """This rank's rows of W x for every token: x [T, n_in] (device f32) -> [T, n_rows]."""
        import torch

        x = x.reshape(-1, self.n_in)
        T = x.shape[0]
        if out is None:
            out = torch.empty((T, self.n_rows), dtype=torch.float32, device=self.dev)
        if self.n_rows == 0:
            return out
        L, s = lib(), stream_ptr()
        for t in range(T):  # one resident-weight matvec per token (decode batches are small)
            rc = L.pi_matvec_col_major(self.ctx.h, ptr(out[t]), ptr(x[t]), ptr(self.w), self.qtype, self.n_in,
                                       self.n_rows, s)
            self.ctx.check(rc)
        return out

    def forward(self, x):
        """Full logits [T, n_out]: the local slice, all-gathered over the ranks when world > 1
        (try_lm_head_matvec's assembly)."""
        local = self.forward_local(x)
        if self.world == 1:
            return local
        return gather_slices(local, self.slices, self.group)


def gather_slices(local, slices, group=None):
    """All-gathers each rank's [T, n_rows_r] slice (rows ``slices[r]``) into [T, n_out]; the
    slices are padded to the largest for the collective (any torch.distributed backend)."""
    import torch
    import torch.distributed as dist

    T, per = local.shape[0], max(n for _, n in slices)
    pad = torch.zeros((T, per), dtype=local.dtype, device=local.device)
    pad[:, :local.shape[1]] = local
    parts = [torch.empty_like(pad) for _ in slices]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[:, :n] for p, (_, n) in zip(parts, slices)], dim=1)
