"""Host-side mirror of the reference's predictor and hot-neuron sparse FFN.

* ``Predictor`` — predictor/mod.rs:20-95: sigmoid(W2 relu(W1 a + b1) + b2)
  over neuron blocks, ``predict`` / ``predict_hot`` (threshold -> block ids).
  ``from_embedded`` gives the reference's zero-weight placeholder model.
* ``SparseFFN`` — the hot-neuron dense FFN of model/mod.rs:1573-1612
  (quant::ffn_swiglu_q_selected per token) on the GPU, with weights repacked
  once (down projection neuron-major).
* ``blocks_to_indices`` expands predictor block ids to the neuron index list
  the sparse FFN takes (64 neurons per block); ``hot_lists_from_probs`` does the
  same on the device for a batch, and ``SparseFFN.forward_predicted`` chains
  predictor probabilities -> lists -> sparse FFN without leaving the device.
* ``HotNeuronIndex`` — activation/mod.rs:246-325, the profiler's per-layer hot
  lists, applied as Model::set_hot_index does (model/mod.rs:1743-1802);
  ``SparseFFN.forward_hot`` runs one static list for every token.
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


# --------------------------------------------------------------------------
# Hot-neuron lists on the device
# --------------------------------------------------------------------------
def hot_lists_from_probs(probs, threshold: float, n_ff: int, block: int = 64, stream=None):
    """Predictor::predict_hot (predictor/mod.rs:87-95) for every token of a device
    probability matrix [T, n_blocks], expanded to neuron ids (block b = neurons
    [b*block, (b+1)*block) below n_ff), as device CSR (ptr [T+1], idx) int64."""
    torch = _torch()
    p = quant._f32(probs)
    T, nb = (p.shape[0], p.shape[1]) if p.dim() == 2 else (1, p.numel())
    ptr_ = torch.empty(T + 1, dtype=torch.int64, device=p.device)
    idx = torch.empty(max(T * n_ff, 1), dtype=torch.int64, device=p.device)
    ctx = Context.default()
    ctx.check(lib().pi_hot_lists_from_probs(ctx.h, ptr(p), T, nb, float(threshold), block, n_ff, ptr(ptr_), ptr(idx),
                                            stream_ptr(stream)))
    return ptr_, idx


def hot_lists_broadcast(hot_list, T: int, stream=None):
    """One static hot list for each of T tokens, as device CSR (ptr, idx)."""
    torch = _torch()
    lst = torch.as_tensor(np.asarray(hot_list, np.int64)).cuda()
    n = lst.numel()
    ptr_ = torch.empty(T + 1, dtype=torch.int64, device="cuda")
    idx = torch.empty(max(T * n, 1), dtype=torch.int64, device="cuda")
    ctx = Context.default()
    ctx.check(lib().pi_hot_lists_broadcast(ctx.h, ptr(lst), n, T, ptr(ptr_), ptr(idx), stream_ptr(stream)))
    return ptr_, idx


class HotNeuronIndex:
    """activation/mod.rs:246-330: per-layer hot neuron lists (JSON), loaded the way
    Model::set_hot_index does (model/mod.rs:1743-1761): each list sorted and
    de-duplicated, then validated against the model's layer widths."""

    def __init__(self, version: int, threshold: float, min_hotness: float, total_samples: int, layers: list):
        self.version, self.threshold, self.min_hotness, self.total_samples = version, threshold, min_hotness, \
            total_samples
        self.layers = [dict(layer_idx=int(l["layer_idx"]), hot_indices=sorted(set(int(i) for i in l["hot_indices"])),
                            n_ff=int(l["n_ff"])) for l in layers]

    @classmethod
    def load(cls, path) -> "HotNeuronIndex":
        import json
        from pathlib import Path

        d = json.loads(Path(path).read_text())
        return cls(d["version"], d["threshold"], d["min_hotness"], d["total_samples"], d["layers"])

    def save(self, path) -> None:
        import json
        from pathlib import Path

        Path(path).parent.mkdir(parents=True, exist_ok=True)
        Path(path).write_text(json.dumps(dict(version=self.version, threshold=self.threshold,
                                              min_hotness=self.min_hotness, total_samples=self.total_samples,
                                              layers=self.layers), indent=2))

    def layer(self, layer_idx: int):
        """The entry of `layer_idx` or None (activation/mod.rs:265-270)."""
        return next((l for l in self.layers if l["layer_idx"] == layer_idx), None)

    def validate_against_dims(self, layer_dims) -> None:
        """activation/mod.rs:287-325: every entry names a layer of the model once, with
        the model's width and indices inside it."""
        seen = [False] * len(layer_dims)
        for l in self.layers:
            li = l["layer_idx"]
            if li >= len(layer_dims):
                raise PiError(PI_ERR_ARG, f"hot index layer {li} is out of range for model with {len(layer_dims)} layers")
            if seen[li]:
                raise PiError(PI_ERR_ARG, f"hot index contains duplicate entries for layer {li}")
            seen[li] = True
            if l["n_ff"] != layer_dims[li]:
                raise PiError(PI_ERR_ARG, f"hot index layer {li} expects width {l['n_ff']}, but model layer width is "
                                          f"{layer_dims[li]}")
            bad = [i for i in l["hot_indices"] if i >= l["n_ff"]]
            if bad:
                raise PiError(PI_ERR_ARG, f"hot index layer {li} contains out-of-range index {bad[0]} for width "
                                          f"{l['n_ff']}")

    def sparse_hot_indices(self, layer_idx: int, dense_width: int):
        """model/mod.rs:1799-1802: the layer's list when it is narrower than the dense
        width, else None (the dense path)."""
        l = self.layer(layer_idx)
        if l is None or len(l["hot_indices"]) >= dense_width:
            return None
        return l["hot_indices"]


def _sparse_forward_predicted(self, x, probs, threshold: float, block: int = 64, out=None, stream=None):
    """The FFN over the neurons the predictor marks hot for each token: device
    probabilities [T, n_blocks] -> device CSR lists -> the sparse FFN, with no
    host round trip."""
    csr = hot_lists_from_probs(probs, threshold, self.n_ff, block, stream=stream)
    return self.forward(x, csr=csr, out=out, stream=stream)


def _sparse_forward_hot(self, x, hot_list, out=None, stream=None):
    """The FFN over one static hot list for every token (a HotNeuronIndex layer)."""
    xd = quant._f32(x)
    T = xd.numel() // self.n_embd
    lst = np.asarray(hot_list, np.int64)
    if lst.size and (lst.min() < 0 or lst.max() >= self.n_ff):
        raise PiError(2, "hot index out of range for the FFN width")
    return self.forward(xd, csr=hot_lists_broadcast(lst, T, stream=stream), out=out, stream=stream)


SparseFFN.forward_predicted = _sparse_forward_predicted
SparseFFN.forward_hot = _sparse_forward_hot
