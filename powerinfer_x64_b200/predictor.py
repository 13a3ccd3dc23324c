"""Host-side mirror of the reference's predictor and hot-neuron sparse FFN.

* ``Predictor`` — predictor/mod.rs:20-95: sigmoid(W2 relu(W1 a + b1) + b2)
  over neuron blocks, ``predict`` / ``predict_hot`` (threshold -> block ids).
  ``from_embedded`` gives the reference's zero-weight placeholder model.
* ``SparseFFN`` — the hot-neuron dense FFN of model/mod.rs:1573-1612
  (quant::ffn_swiglu_q_selected per token) on the GPU, with weights repacked
  once (down projection neuron-major).
* ``blocks_to_indices`` expands predictor block ids to the neuron index list
  the sparse FFN takes (64 neurons per block).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import quant
from ._lib import Context, PiError, PI_ERR_ARG, lib, ptr, stream_ptr


def _torch():
    import torch

    return torch


class PredictorConfig:
    """predictor/mod.rs:12-17."""

    def __init__(self, input_dim=256, hidden_dim=512, output_dim=128, n_layers=2):
        self.input_dim, self.hidden_dim, self.output_dim, self.n_layers = input_dim, hidden_dim, output_dim, n_layers


class Predictor:
    def __init__(self, config: PredictorConfig, weights1, bias1, weights2, bias2):
        torch = _torch()
        self.config = config
        f = lambda a: torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float32))).cuda()
        self.w1, self.b1, self.w2, self.b2 = f(weights1), f(bias1), f(weights2), f(bias2)

    @classmethod
    def from_embedded(cls) -> "Predictor":
        """predictor/mod.rs:31-54: the placeholder model (all weights zero)."""
        c = PredictorConfig()
        return cls(c, np.zeros((c.hidden_dim, c.input_dim)), np.zeros(c.hidden_dim),
                   np.zeros((c.output_dim, c.hidden_dim)), np.zeros(c.output_dim))

    def predict_batch(self, activations):
        """probabilities [T, output_dim] for activations [T, input_dim] (device tensor)."""
        torch = _torch()
        c = self.config
        a = quant._f32(activations)
        T = a.numel() // c.input_dim
        out = torch.empty((T, c.output_dim), dtype=torch.float32, device="cuda")
        ctx = Context.default()
        ctx.check(lib().pi_predictor_forward(ctx.h, ptr(a), T, ptr(self.w1), ptr(self.b1), ptr(self.w2),
                                             ptr(self.b2), c.input_dim, c.hidden_dim, c.output_dim, ptr(out),
                                             stream_ptr()))
        return out

    def predict(self, activations):
        """predictor/mod.rs:63-84; a dimension mismatch gives zeros (with a warning), as the reference."""
        a = np.asarray(activations, np.float32).reshape(-1)
        if a.size != self.config.input_dim:
            import sys

            print(f"Warning: predictor input dim mismatch, expected {self.config.input_dim}, got {a.size}",
                  file=sys.stderr)
            return np.zeros(self.config.output_dim, np.float32)
        return self.predict_batch(a.reshape(1, -1)).cpu().numpy()[0]

    def predict_hot(self, activations, threshold: float):
        """predictor/mod.rs:87-95: ids of blocks with probability >= threshold."""
        probs = self.predict(activations)
        return [int(i) for i in np.nonzero(probs >= np.float32(threshold))[0]]


def blocks_to_indices(blocks, block_size: int = 64, n_ff: int | None = None):
    """Ascending neuron ids covered by the given block ids."""
    ids = np.concatenate([np.arange(b * block_size, (b + 1) * block_size) for b in sorted(set(blocks))]) \
        if len(blocks) else np.zeros(0, np.int64)
    if n_ff is not None:
        ids = ids[ids < n_ff]
    return ids.astype(np.int64)


class SparseFFN:
    """Hot-neuron sparse SwiGLU FFN (gate/up [ne0=n_embd, ne1=n_ff], down [ne0=n_ff, ne1=n_embd])."""

    def __init__(self, gate_raw, up_raw, down_raw, qtype, n_embd: int, n_ff: int, device: int | None = None):
        torch = _torch()
        self.ctx = Context.default(device)
        self.n_embd, self.n_ff, self.qtype = n_embd, n_ff, int(qtype)
        g, u, d = quant._u8(gate_raw), quant._u8(up_raw), quant._u8(down_raw)
        torch.cuda.synchronize()
        h = C.c_void_p()
        self.ctx.check(lib().pi_sparse_ffn_create(self.ctx.h, ptr(g), ptr(u), ptr(d), self.qtype, n_embd, n_ff, 0,
                                                  C.byref(h)))
        self.h = h

    def __del__(self):
        try:
            if getattr(self, "h", None):
                lib().pi_sparse_ffn_destroy(self.h)
        except Exception:
            pass

    @staticmethod
    def csr(index_lists):
        """(ptr, idx) int64 arrays from per-token ascending index lists."""
        ptr_ = np.zeros(len(index_lists) + 1, np.int64)
        for t, l in enumerate(index_lists):
            ptr_[t + 1] = ptr_[t] + len(l)
        idx = np.concatenate([np.asarray(l, np.int64) for l in index_lists]) if ptr_[-1] else np.zeros(1, np.int64)
        return ptr_, idx

    def forward(self, x, index_lists=None, csr=None, out=None, stream=None):
        """out [T, n_embd] = ffn_swiglu_q_selected(x[t], S_t) for each token t."""
        torch = _torch()
        xd = quant._f32(x)
        T = xd.numel() // self.n_embd
        if csr is None:
            if index_lists is None or len(index_lists) != T:
                raise PiError(PI_ERR_ARG, "need one index list per token")
            for l in index_lists:
                a = np.asarray(l, np.int64)
                if a.size and (a.min() < 0 or a.max() >= self.n_ff) and a.size < self.n_ff:
                    raise PiError(2, f"selected column {int(a[(a < 0) | (a >= self.n_ff)][0])} out of range for "
                                     f"output width {self.n_ff}")
            p, i = self.csr(index_lists)
            csr = (torch.from_numpy(p).cuda(), torch.from_numpy(i).cuda())
        if out is None:
            out = torch.empty((T, self.n_embd), dtype=torch.float32, device="cuda")
        self.ctx.check(lib().pi_sparse_ffn_forward(self.ctx.h, self.h, ptr(xd), T, ptr(csr[0]), ptr(csr[1]), ptr(out),
                                                   stream_ptr(stream)))
        return out
