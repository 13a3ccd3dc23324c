"""GPU parity at the benchmark's own sizes, against the CPU oracle.

* Config 3 (Q4_0, Zipf-biased router) at T = 512, 2048 and 4096: expert
  indices, per-expert counts, offsets and the permutation bit-exact on every
  token, taken from the forward that produced the output (the tensor-core
  grouped-GEMM path); outputs on a 64-token sample that includes the tokens of
  the two most-loaded (Zipf-hot) experts.
* Config 5 (Q8_0, RMSNorm before the layer, residual after) at T = 8192, the
  size that runs the 4-token-per-thread dispatch: the same checks, routing on
  all 8192 tokens.
* The 40-layer config-5 stack, teacher-forced: each layer's GPU input is the
  previous GPU layer's output, and the oracle routes that same input. The
  per-layer routing agreement is reported and must be 100%.
* MoeRouter::route (src/moe/mod.rs:69-108) against its oracle restatement.

Bars: routing bit-exact; outputs within rel-L2 <= 1e-3 and max-abs <= 2e-3
after normalising by the oracle output's RMS. The layer-output bar applies to
the FFN part (output minus residual) where a residual is added.
"""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_L2, MAX_ABS = 1e-3, 2e-3


def close(got, ref, rel_l2=REL_L2, max_abs=MAX_ABS):
    got = np.asarray(got, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    rms = np.sqrt(np.mean(ref ** 2)) or 1.0
    rl2 = np.linalg.norm(got - ref) / (np.linalg.norm(ref) or 1.0)
    ma = np.max(np.abs(got - ref)) / rms if ref.size else 0.0
    assert rl2 <= rel_l2 and ma <= max_abs, f"rel_l2={rl2:.3e} max_abs/rms={ma:.3e}"
    return rl2, ma


def _host(t):
    return t.cpu().numpy() if hasattr(t, "cpu") else t


def _routing_equal(got, ref, what=""):
    for key in ("idx", "counts", "offsets", "perm"):
        g = _host(got[key]).ravel()
        r = np.asarray(ref[key]).ravel()
        assert g.shape == r.shape and np.array_equal(g, r), f"{what}: {key} differs at {np.flatnonzero(g != r)[:8]}"


def _report(name, obj):
    d = os.environ.get("PI_REPORT_DIR")
    if d:
        os.makedirs(d, exist_ok=True)
        with open(os.path.join(d, name), "w") as f:
            json.dump(obj, f, indent=1)


def _sample(route, T, n=64):
    """n tokens: 16 routed to each of the two most-loaded experts, the rest evenly spaced."""
    counts = _host(route["counts"])
    offs = _host(route["offsets"])
    perm = _host(route["perm"])
    hot = np.argsort(-counts, kind="stable")[:2]
    pick = []
    for e in hot:
        toks = perm[offs[e]:offs[e] + counts[e]]
        pick += list(toks[np.linspace(0, len(toks) - 1, 16).astype(int)])
    pick += list(np.linspace(0, T - 1, n - len(pick)).astype(int))
    return np.unique(np.asarray(pick, np.int64)), hot


def _oracle_layer(orc, cfg, t, x, **kw):
    sh = tuple(_host(a) for a in t["shared"]) if cfg.shared else None
    bias = None if t.get("router_bias") is None else _host(t["router_bias"])
    return orc.moe_layer(x, cfg.d, cfg.f, cfg.E, cfg.k, cfg.qtype, _host(t["router"]), _host(t["gate_exps"]),
                         _host(t["up_exps"]), _host(t["down_exps"]), shared=sh, bias=bias, token_threads=0, **kw)


@pytest.fixture(scope="module")
def torch():
    import torch as t

    assert t.cuda.is_available()
    return t


@pytest.fixture(scope="module")
def pkg():
    from powerinfer_x64_b200 import build

    build.build()
    import powerinfer_x64_b200 as p

    return p


@pytest.fixture(scope="module")
def c3(pkg, torch):
    from powerinfer_x64_b200 import synth

    L, t = synth.moe_layer(synth.C3, seed=0, keep_tensors=True)
    host = {k: (tuple(_host(a) for a in v) if isinstance(v, tuple) else _host(v)) for k, v in t.items()
            if v is not None}
    host["router_bias"] = _host(t["router_bias"])
    del t
    torch.cuda.empty_cache()
    return L, host


@pytest.mark.parametrize("T", [512, 2048, 4096])
def test_c3_baseline_sizes_vs_oracle(pkg, orc, torch, c3, T):
    from powerinfer_x64_b200 import synth

    c = synth.C3
    L, t = c3
    x = synth.tokens_dev(c.d, T, seed=20 + T)
    out, r = L.forward_routed(x)  # auto path: the tensor-core router and grouped GEMMs at these sizes
    xh = _host(x)
    ref = orc.moe_route(xh, t["router"], c.d, c.E, c.k, bias=t["router_bias"])
    _routing_equal(r, ref, f"c3 T={T}")
    close(_host(r["gates"]), ref["gates"], rel_l2=1e-6, max_abs=1e-5)
    counts = _host(r["counts"])
    assert counts.max() > 2 * counts.mean()  # the Zipf bias skews the load
    pick, hot = _sample(r, T)
    got = _host(out)[pick]
    want = _oracle_layer(orc, c, t, xh[pick])
    rl2, ma = close(got, want)
    _report(f"c3_T{T}_parity.json", dict(T=T, routing_bit_exact=True, sample=len(pick), hot_experts=hot.tolist(),
                                        hot_counts=counts[hot].tolist(), rel_l2=rl2, max_abs_over_rms=ma))


@pytest.mark.parametrize("fast", [False, True])
def test_c5_T8192_vs_oracle(pkg, orc, torch, fast):
    """fast: the grouped GEMM adds the block terms with fused multiply-adds
    (PI_FWD_FAST_SUM); the bars are the same."""
    from powerinfer_x64_b200 import synth

    c = synth.C5
    T = 8192
    L, t = synth.moe_layer(c, seed=0, layer=0, keep_tensors=True)
    x = synth.tokens_dev(c.d, T, seed=0, layer=0)
    out, r = L.forward_routed(x, rmsnorm=True, residual=True, fast=fast)
    xh = _host(x)
    normed = np.stack([orc.rms_norm(row, np.ones(c.d, np.float32)) for row in xh])
    ref = orc.moe_route(normed, _host(t["router"]), c.d, c.E, c.k)
    _routing_equal(r, ref, "c5 T=8192")
    close(_host(r["gates"]), ref["gates"], rel_l2=1e-6, max_abs=1e-5)
    pick, hot = _sample(r, T)
    got = _host(out)[pick]
    want = _oracle_layer(orc, c, t, xh[pick], residual=True, rmsnorm=True)
    rl2, ma = close(got - xh[pick], want - xh[pick])
    same = float(np.mean(got.view(np.uint32) == want.view(np.uint32)))
    _report(f"c5_T8192{'_fast' if fast else ''}_parity.json", dict(T=T, routing_bit_exact=True, sample=len(pick), rel_l2=rl2,
                                         max_abs_over_rms=ma, bitwise_equal_fraction=same))


def test_c5_stack_40_layers_teacher_forced(pkg, orc, torch):
    """40 layers at the config-5 shape, chained on the GPU (RMSNorm -> MoE ->
    residual). At every layer the oracle routes the GPU's own layer input, so
    each layer's routing is checked on all tokens independently of the others;
    outputs are checked on a token sample at four layers."""
    from powerinfer_x64_b200 import synth

    c = synth.C5
    T = int(os.environ.get("PI_STACK_TOKENS", "8192"))
    x = synth.tokens_dev(c.d, T, seed=0, layer=0)
    agree, checks = [], []
    out_layers = (0, 13, 26, 39)
    for layer in range(c.layers):
        L, t = synth.moe_layer(c, seed=0, layer=layer, keep_tensors=True)
        y, r = L.forward_routed(x, rmsnorm=True, residual=True)
        xh = _host(x)
        normed = np.stack([orc.rms_norm(row, np.ones(c.d, np.float32)) for row in xh])
        ref = orc.moe_route(normed, _host(t["router"]), c.d, c.E, c.k)
        idx = _host(r["idx"])
        tok_ok = np.all(idx == ref["idx"], axis=1)
        agree.append(float(tok_ok.mean()))
        if layer in out_layers:
            pick = np.linspace(0, T - 1, 16).astype(np.int64)
            want = _oracle_layer(orc, c, t, xh[pick], residual=True, rmsnorm=True)
            got = _host(y)[pick]
            checks.append(dict(layer=layer, rel_l2_max_abs=close(got - xh[pick], want - xh[pick])))
        x = y
        del L, t
        torch.cuda.empty_cache()
    _report("c5_stack_teacher_forced.json", dict(T=T, layers=c.layers, routing_agreement=agree, outputs=checks))
    assert all(a == 1.0 for a in agree), agree


def test_moe_router_api_vs_oracle(pkg, orc, torch):
    """MoeRouter::route (row-major [d, E] gate, top-k on logits in descending
    order, softmax over the k) against its oracle restatement, 64 tokens."""
    from powerinfer_x64_b200 import moe

    rng = np.random.default_rng(31)
    d, E, k = 2048, 256, 8
    gate = (rng.standard_normal(d * E) * 0.02).astype(np.float32)
    x = rng.standard_normal((64, d)).astype(np.float32)
    R = moe.MoeRouter(gate, d, E, k)
    idx, w = R._layer.route_api(x)
    ridx, rw = orc.moe_api_route(x, gate, d, E, k)
    assert np.array_equal(idx, ridx)
    close(w, rw, rel_l2=1e-6, max_abs=1e-6)
    one = R.route(x[5])
    assert one.expert_indices == ridx[5].tolist()
