"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle on the
same seeded inputs, and against the committed golden fixture.

Bars (north star): routing indices, per-expert counts, offsets and the
permutation bit-exact; float outputs within rel-L2 <= 1e-3 and
max-abs <= 2e-3 after normalising by the oracle output's RMS. The
per-function drop-ins keep the reference's exact summation order and are held
to bitwise equality (SwiGLU outputs to 1 ulp-level, see the exp note).
"""
import json

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


def bits(a):
    return np.ascontiguousarray(np.asarray(a, np.float32)).view(np.uint32)


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
    from powerinfer_x64_b200 import moe, predictor, quant, synth  # noqa: F401

    return p


@pytest.fixture(scope="module")
def kat(golden_dir):
    return json.loads((golden_dir / "reference_kat.json").read_text())


# ---------------------------------------------------------------------------
# quant drop-ins
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name,qt", [("q4_0_zero_nibbles", 2), ("q8_0_ones_half_scale", 8), ("q4_0_soak_pattern", 2)])
def test_dequant_kat_gpu(pkg, orc, kat, name, qt):
    from powerinfer_x64_b200 import quant

    k = kat[name]
    raw = np.frombuffer(bytes.fromhex(k["block_hex"]), np.uint8)
    got = quant.dequantize(raw, qt, 1, 32)
    assert np.array_equal(bits(got), bits(orc.dequantize(raw, qt, 1, 32)))


def test_dequant_short_raises(pkg):
    from powerinfer_x64_b200 import PiError, quant

    with pytest.raises(PiError):
        quant.dequantize(np.zeros(17, np.uint8), 2, 1, 32)


@pytest.mark.parametrize("qt", [2, 8])
def test_quantisers_bitwise(pkg, orc, qt):
    from powerinfer_x64_b200 import quant

    rng = np.random.default_rng(10)
    x = (rng.standard_normal(32 * 4096) * 0.02).astype(np.float32)
    x[:32] = 0.0  # an all-zero block
    x[64:96] = -x[64:96]
    got = (quant.quantize_q8_0 if qt == 8 else quant.quantize_q4_0)(x)
    ref = (orc.quantize_q8_0 if qt == 8 else orc.quantize_q4_0)(x)
    bs = 34 if qt == 8 else 18
    bad = np.nonzero((got.reshape(-1, bs) != ref.reshape(-1, bs)).any(1))[0]
    assert bad.size == 0, (bad[:8], got.reshape(-1, bs)[bad[0]], ref.reshape(-1, bs)[bad[0]], x[32 * bad[0]:32 * bad[0] + 32])
    assert np.array_equal(bits(quant.dequantize(got, qt, 1, x.size)), bits(orc.dequantize(ref, qt, 1, x.size)))


@pytest.mark.parametrize("qt,n_in,n_out", [(8, 2048, 512), (8, 512, 2048), (2, 1024, 256), (0, 300, 64)])
def test_matvec_col_major_bitwise(pkg, orc, qt, n_in, n_out):
    from powerinfer_x64_b200 import quant

    rng = np.random.default_rng(11)
    w = (rng.standard_normal(n_in * n_out) * 0.02).astype(np.float32)
    raw = {8: orc.quantize_q8_0, 2: orc.quantize_q4_0, 0: lambda a: a.view(np.uint8)}[qt](w)
    x = rng.standard_normal(n_in).astype(np.float32)
    y = np.zeros(n_out, np.float32)
    quant.matvec_col_major(y, x, raw, qt, n_in, n_out)
    assert np.array_equal(bits(y), bits(orc.matvec_col_major(x, raw, qt, n_in, n_out)))


@pytest.mark.parametrize("qt", [0, 2, 8])
def test_select_and_sparse_input_bitwise(pkg, orc, qt):
    from powerinfer_x64_b200 import PiError, quant

    rng = np.random.default_rng(12)
    n_in, n_out = 1024, 768
    w = (rng.standard_normal(n_in * n_out) * 0.02).astype(np.float32)
    raw = {8: orc.quantize_q8_0, 2: orc.quantize_q4_0, 0: lambda a: a.view(np.uint8)}[qt](w)
    x = rng.standard_normal(n_in).astype(np.float32)
    idx = np.sort(rng.choice(n_out, 100, replace=False)).astype(np.int64)
    y = np.zeros(idx.size, np.float32)
    quant.matvec_col_major_select(y, x, raw, qt, n_in, n_out, idx)
    assert np.array_equal(bits(y), bits(orc.matvec_col_major_select(x, raw, qt, n_in, n_out, idx)))
    with pytest.raises(PiError):
        quant.matvec_col_major_select(y, x, raw, qt, n_in, n_out, [n_out])
    # sparse input over the rows of a [ne0=n_in, ne1=n_out] matrix used transposed
    sidx = np.sort(rng.choice(n_in, 150, replace=False)).astype(np.int64)
    xs = rng.standard_normal(sidx.size).astype(np.float32)
    ys = np.zeros(n_out, np.float32)
    quant.matvec_col_major_sparse_input(ys, xs, sidx, raw, qt, n_in, n_out)
    assert np.array_equal(bits(ys), bits(orc.matvec_col_major_sparse_input(xs, sidx, raw, qt, n_in, n_out)))
    quant.matvec_col_major_sparse_input(ys, [], [], raw, qt, n_in, n_out)
    assert np.all(ys == 0)


def test_f32_known_answers_gpu(pkg, kat):
    from powerinfer_x64_b200 import quant

    k = kat["select_f32"]
    raw = np.asarray(k["w"], np.float32).view(np.uint8)
    y = np.zeros(2, np.float32)
    quant.matvec_col_major_select(y, k["x"], raw, 0, k["n_in"], k["n_out"], k["indices"])
    assert np.allclose(y, k["expect"], atol=k["tol"])
    k = kat["sparse_input_f32"]
    raw = np.asarray(k["w"], np.float32).view(np.uint8)
    y = np.zeros(3, np.float32)
    quant.matvec_col_major_sparse_input(y, k["x"], k["indices"], raw, 0, k["n_in"], k["n_out"])
    assert np.allclose(y, k["expect"], atol=k["tol"])


@pytest.mark.parametrize("qt", [0, 2, 8])
def test_ffn_swiglu_q_and_selected(pkg, orc, qt):
    from powerinfer_x64_b200 import quant

    rng = np.random.default_rng(13)
    n_embd, n_ff = 1024, 512
    q = {8: orc.quantize_q8_0, 2: orc.quantize_q4_0, 0: lambda a: a.view(np.uint8)}[qt]
    g = q((rng.standard_normal(n_embd * n_ff) * 0.02).astype(np.float32))
    u = q((rng.standard_normal(n_embd * n_ff) * 0.02).astype(np.float32))
    d = q((rng.standard_normal(n_embd * n_ff) * 0.02).astype(np.float32))
    x = rng.standard_normal(n_embd).astype(np.float32)
    out = np.zeros(n_embd, np.float32)
    quant.ffn_swiglu_q(out, x, g, u, d, qt, n_embd, n_ff)
    ref = orc.ffn_swiglu_q(x, g, u, d, qt, n_embd, n_ff)
    close(out, ref, rel_l2=1e-6, max_abs=1e-5)
    idx = np.sort(rng.choice(n_ff, 77, replace=False)).astype(np.int64)
    quant.ffn_swiglu_q_selected(out, x, g, u, d, qt, n_embd, n_ff, idx)
    close(out, orc.ffn_swiglu_q_selected(x, g, u, d, qt, n_embd, n_ff, idx), rel_l2=1e-6, max_abs=1e-5)
    quant.ffn_swiglu_q_selected(out, x, g, u, d, qt, n_embd, n_ff, [])
    assert np.all(out == 0)
    quant.ffn_swiglu_q_selected(out, x, g, u, d, qt, n_embd, n_ff, np.arange(n_ff))  # dense fallback
    close(out, ref, rel_l2=1e-6, max_abs=1e-5)


def test_ffn_selected_kat_gpu(pkg, kat):
    from test_oracle import _f32_ffn_masked
    from powerinfer_x64_b200 import quant

    k = kat["ffn_selected_f32"]
    pk = lambda a: np.asarray(a, np.float32).view(np.uint8)
    out = np.zeros(k["n_embd"], np.float32)
    quant.ffn_swiglu_q_selected(out, k["x"], pk(k["gate"]), pk(k["up"]), pk(k["down"]), 0, k["n_embd"], k["n_ff"],
                                k["indices"])
    assert np.allclose(out, _f32_ffn_masked(k), atol=k["tol"])


# ---------------------------------------------------------------------------
# MoE layer
# ---------------------------------------------------------------------------
def _routing_equal(got, ref):
    for key in ("idx", "counts", "offsets", "perm"):
        g = got[key].cpu().numpy().ravel() if hasattr(got[key], "cpu") else np.asarray(got[key]).ravel()
        assert np.array_equal(g, np.asarray(ref[key]).ravel()), key


def test_c1_against_golden_fixture(pkg, torch, golden_dir):
    import make_golden
    from powerinfer_x64_b200 import moe, synth

    c = synth.C1
    fx = np.load(golden_dir / "c1_seed0.npz")
    inp = make_golden.c1_inputs(0)
    assert make_golden.digest(inp) == str(fx["input_sha256"])
    L = moe.MoeLayer(inp["router"], inp["gate_exps"], inp["up_exps"], inp["down_exps"], c.qtype, c.d, c.f, c.E, c.k)
    x = torch.from_numpy(inp["x"]).cuda()
    r = L.route(x)
    _routing_equal(r, fx)
    close(r["gates"].cpu().numpy(), fx["gates"], rel_l2=1e-4, max_abs=1e-4)
    out = L.forward(x).cpu().numpy()
    close(out, fx["out"])


def _host(t):
    return t.cpu().numpy() if hasattr(t, "cpu") else t


def _oracle_layer(orc, cfg, t, x, **kw):
    sh = None
    if cfg.shared:
        sh = tuple(_host(a) for a in t["shared"])
    return orc.moe_layer(_host(x), cfg.d, cfg.f, cfg.E, cfg.k, cfg.qtype, _host(t["router"]), _host(t["gate_exps"]),
                         _host(t["up_exps"]), _host(t["down_exps"]), shared=sh,
                         bias=None if t["router_bias"] is None else _host(t["router_bias"]), threads=0, **kw)


@pytest.fixture(scope="module")
def c2_layer(pkg, torch):
    from powerinfer_x64_b200 import synth

    return synth.moe_layer(synth.C2, seed=0, keep_tensors=True)


@pytest.mark.parametrize("T", [1, 4, 16, 64])
def test_c2_decode_parity(pkg, orc, torch, c2_layer, T):
    from powerinfer_x64_b200 import synth

    c = synth.C2
    L, t = c2_layer
    x = synth.tokens_dev(c.d, T, seed=0)
    r = L.route(x)
    ref_r = orc.moe_route(_host(x), _host(t["router"]), c.d, c.E, c.k)
    _routing_equal(r, ref_r)
    close(r["gates"].cpu().numpy(), ref_r["gates"], rel_l2=1e-4, max_abs=1e-4)
    out = L.forward(x).cpu().numpy()
    close(out, _oracle_layer(orc, c, t, x))


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_c2_other_seeds(pkg, orc, torch, seed):
    from powerinfer_x64_b200 import synth

    c = synth.C2
    L, t = synth.moe_layer(c, seed=seed, keep_tensors=True)
    x = synth.tokens_dev(c.d, 16, seed=seed)
    _routing_equal(L.route(x), orc.moe_route(_host(x), _host(t["router"]), c.d, c.E, c.k))
    close(L.forward(x).cpu().numpy(), _oracle_layer(orc, c, t, x))


def test_c3_shape_q4_zipf_parity(pkg, orc, torch):
    from powerinfer_x64_b200 import synth

    c = synth.C3
    L, t = synth.moe_layer(c, seed=0, keep_tensors=True)
    x = synth.tokens_dev(c.d, 24, seed=0)
    ref_r = orc.moe_route(_host(x), _host(t["router"]), c.d, c.E, c.k, bias=_host(t["router_bias"]))
    _routing_equal(L.route(x), ref_r)
    close(L.forward(x).cpu().numpy(), _oracle_layer(orc, c, t, x))


@pytest.fixture(scope="module")
def c3_layer(pkg, torch):
    from powerinfer_x64_b200 import synth

    return synth.moe_layer(synth.C3, seed=0, keep_tensors=True)


def test_c3_prefill_gemm_vs_oracle(pkg, orc, torch, c3_layer):
    """Prefill-sized batch: the tcgen05 GEMM path against the reference restatement."""
    from powerinfer_x64_b200 import synth

    c = synth.C3
    L, t = c3_layer
    x = synth.tokens_dev(c.d, 160, seed=3)
    got = L.forward(x, path="gemm").cpu().numpy()
    close(got, _oracle_layer(orc, c, t, x))


@pytest.mark.parametrize("T", [256, 300])
def test_c3_prefill_router_exact(pkg, orc, torch, c3_layer, T):
    """Prefill-sized batches take the wide exact router: indices, counts,
    offsets and permutation bit-exact against the reference restatement
    (Zipf-biased logits, a ragged final token tile), the shared-expert gate
    through the layer output."""
    from powerinfer_x64_b200 import synth

    c = synth.C3
    L, t = c3_layer
    x = synth.tokens_dev(c.d, T, seed=7)
    ref_r = orc.moe_route(_host(x), _host(t["router"]), c.d, c.E, c.k, bias=_host(t["router_bias"]))
    r = L.route(x)
    _routing_equal(r, ref_r)
    close(r["gates"].cpu().numpy(), ref_r["gates"], rel_l2=1e-6, max_abs=1e-6)


@pytest.mark.parametrize("T", [512, 2048])
def test_c3_prefill_gemm_vs_gemv(pkg, torch, c3_layer, T):
    """Same inputs through both expert paths (Zipf-skewed routing: experts with
    more than 128 tokens span several GEMM work items)."""
    from powerinfer_x64_b200 import synth

    L, _ = c3_layer
    x = synth.tokens_dev(synth.C3.d, T, seed=4)
    a = L.forward(x, path="gemm").cpu().numpy()
    b = L.forward(x, path="gemv").cpu().numpy()
    close(a, b)
    r = L.route(x)
    assert int(r["counts"].max()) > 128


@pytest.mark.parametrize("T", [40, 300])
def test_q8_prefill_gemm_bit_exact(pkg, orc, torch, T):
    """Q8_0 prefill GEMM (int8 block sums exact on the tensor cores, scales in
    block order, SwiGLU and Q8_0 h in the epilogue) is bit-exact with the
    reference restatement. A top-1 layer makes the renormalised gate exactly 1,
    so the layer output is the expert FFN output itself; T = 300 also takes the
    tensor-core router and multi-item experts."""
    from powerinfer_x64_b200 import moe

    rng = np.random.default_rng(21)
    d, E, k, f = 1024, 8, 1, 512
    router = (rng.standard_normal(E * d) * 0.02).astype(np.float32)
    g, u, dn = (orc.quantize_q8_0((rng.standard_normal(E * f * d) * 0.02).astype(np.float32)) for _ in range(3))
    x = rng.standard_normal((T, d)).astype(np.float32)
    L = moe.MoeLayer(router, g, u, dn, 8, d, f, E, k)
    got = L.forward(torch.from_numpy(x).cuda(), path="gemm").cpu().numpy()
    ref = orc.moe_layer(x, d, f, E, k, 8, router, g, u, dn, threads=1)
    close(got, ref)
    assert np.array_equal(bits(got), bits(ref)), f"{np.count_nonzero(bits(got) != bits(ref))} outputs differ"


def test_q8_prefill_gemm_vs_gemv(pkg, torch, c2_layer):
    """A batch large enough for multi-item experts: GEMM and GEMV paths agree."""
    from powerinfer_x64_b200 import synth

    L, _ = c2_layer
    x = synth.tokens_dev(synth.C2.d, 1024, seed=12)
    close(L.forward(x, path="gemm").cpu().numpy(), L.forward(x, path="gemv").cpu().numpy())


def test_c5_rmsnorm_residual_teacher_forced(pkg, orc, torch):
    """Two layers of the C5 stack: each GPU layer gets the oracle's previous output."""
    from powerinfer_x64_b200 import synth

    c = synth.C5
    x = _host(synth.tokens_dev(c.d, 32, seed=0))
    for layer in range(2):
        L, t = synth.moe_layer(c, seed=0, layer=layer, keep_tensors=True)
        ref = _oracle_layer(orc, c, t, x, residual=True, rmsnorm=True)
        got = L.forward(torch.from_numpy(x).cuda(), rmsnorm=True, residual=True).cpu().numpy()
        close(got - x, ref - x)  # the FFN part, normalised by its own RMS
        x = ref


@pytest.mark.parametrize("T", [48, 300])
def test_routing_exact_fallback_on_ties(pkg, orc, torch, T):
    """Pairs of identical router rows give exactly tied logits: such tokens cannot
    be certified by the fast router and must take the exact path, which breaks
    the tie to the lowest expert index like the reference restatement. At
    T = 300 the wide exact router (64 of 128 tile rows live) takes the batch."""
    from powerinfer_x64_b200 import moe

    rng = np.random.default_rng(16)
    d, E, k, f = 1024, 64, 4, 256
    router = (rng.standard_normal((E // 2, d)) * 0.02).astype(np.float32).repeat(2, axis=0).reshape(-1)
    g, u, dn = (orc.quantize_q8_0((rng.standard_normal(E * f * d) * 0.02).astype(np.float32)) for _ in range(3))
    x = rng.standard_normal((T, d)).astype(np.float32)
    L = moe.MoeLayer(router, g, u, dn, 8, d, f, E, k)
    r = L.route(torch.from_numpy(x).cuda())
    ref = orc.moe_route(x, router, d, E, k)
    _routing_equal(r, ref)
    close(r["gates"].cpu().numpy(), ref["gates"], rel_l2=1e-4, max_abs=1e-4)
    close(L.forward(torch.from_numpy(x).cuda()).cpu().numpy(),
          orc.moe_layer(x, d, f, E, k, 8, router, g, u, dn, threads=1))


def test_moe_edge_cases(pkg, torch, c2_layer):
    L, _ = c2_layer
    out = L.forward(torch.zeros((0, 2048), device="cuda"))
    assert out.shape == (0, 2048)
    z = L.forward(torch.zeros((3, 2048), device="cuda")).cpu().numpy()  # all-zero tokens: all logits tie
    assert np.all(np.isfinite(z))
    r = L.route(torch.zeros((3, 2048), device="cuda"))
    assert r["idx"].cpu().numpy().tolist() == [list(range(8))] * 3  # ties break to the lowest indices


# ---------------------------------------------------------------------------
# hot-neuron sparse FFN
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("qt", [2, 8])
def test_sparse_ffn_small(pkg, orc, torch, qt):
    from powerinfer_x64_b200 import PiError, predictor

    rng = np.random.default_rng(14)
    n_embd, n_ff = 1024, 2048
    q = orc.quantize_q8_0 if qt == 8 else orc.quantize_q4_0
    g, u, d = (q((rng.standard_normal(n_embd * n_ff) * 0.02).astype(np.float32)) for _ in range(3))
    F = predictor.SparseFFN(g, u, d, qt, n_embd, n_ff)
    T = 11
    x = rng.standard_normal((T, n_embd)).astype(np.float32)
    lists = [np.sort(rng.choice(n_ff, m, replace=False)).astype(np.int64) for m in
             (0, 1, 5, 300, 307, 2047, 100, 31, 64, 900, 10)]
    lists[5] = np.arange(n_ff)  # dense
    got = F.forward(torch.from_numpy(x).cuda(), lists).cpu().numpy()
    ref = orc.sparse_ffn(x, g, u, d, qt, n_embd, n_ff, lists)
    assert np.all(got[0] == 0)
    for t in range(1, T):
        close(got[t], ref[t])
    with pytest.raises(PiError):
        F.forward(torch.from_numpy(x[:1]).cuda(), [np.array([n_ff], np.int64)])


@pytest.mark.parametrize("qt", [2, 8])
def test_sparse_ffn_one_token_fused(pkg, orc, torch, qt, monkeypatch):
    """A one-token pass runs as one fused launch (gate/up straight from the
    token's list, grid barrier, down). Against the oracle: empty, short, long,
    unsorted and complete (dense) lists; a list with repeated entries gives the
    same output as the three-launch path (PI_SF_SPLIT=1), which marks each
    neuron once; an out-of-range entry is refused."""
    from powerinfer_x64_b200 import PiError, predictor

    rng = np.random.default_rng(21)
    n_embd, n_ff = 2048, 4096
    q = orc.quantize_q8_0 if qt == 8 else orc.quantize_q4_0
    g, u, d = (q((rng.standard_normal(n_embd * n_ff) * 0.02).astype(np.float32)) for _ in range(3))
    F = predictor.SparseFFN(g, u, d, qt, n_embd, n_ff)
    monkeypatch.setenv("PI_SF_SPLIT", "1")
    Fs = predictor.SparseFFN(g, u, d, qt, n_embd, n_ff)
    monkeypatch.delenv("PI_SF_SPLIT")
    x = rng.standard_normal((1, n_embd)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    for lst in (np.zeros(0, np.int64), np.array([7], np.int64), rng.permutation(n_ff)[:600],
                np.sort(rng.choice(n_ff, 3000, replace=False)), np.arange(n_ff)):
        lst = np.asarray(lst, np.int64)
        got = F.forward(xd, [lst]).cpu().numpy()
        if lst.size == 0:
            assert np.all(got == 0)
            continue
        close(got[0], orc.sparse_ffn(x, g, u, d, qt, n_embd, n_ff, [np.sort(lst)])[0])
    rep = np.concatenate([rng.choice(n_ff, 500, replace=False)] * 2)
    a = F.forward(xd, [rep]).cpu().numpy()
    b = Fs.forward(xd, [rep]).cpu().numpy()
    close(a[0], b[0], rel_l2=1e-5, max_abs=1e-5)
    close(a[0], orc.sparse_ffn(x, g, u, d, qt, n_embd, n_ff, [np.unique(rep)])[0])
    # an out-of-range entry reaches the device (the host check is for Python lists only)
    bad = (torch.tensor([0, 2], dtype=torch.int64, device="cuda"),
           torch.tensor([3, n_ff + 5], dtype=torch.int64, device="cuda"))
    F.forward(xd, csr=bad)
    with pytest.raises(PiError):
        F.ctx.sync_check()
    # the context is usable afterwards
    close(F.forward(xd, [np.array([7], np.int64)]).cpu().numpy()[0],
          orc.sparse_ffn(x, g, u, d, qt, n_embd, n_ff, [np.array([7], np.int64)])[0])


@pytest.mark.parametrize("T", [1, 8])
def test_c4_sparse_parity(pkg, orc, torch, T):
    from powerinfer_x64_b200 import predictor, synth

    c = synth.C4
    t = synth.sparse_tensors(c, seed=0)
    F = predictor.SparseFFN(t["gate"], t["up"], t["down"], c.qtype, c.d, c.F)
    lists = synth.sparse_masks(c, T, seed=0)
    assert all(l.size == round(c.active_frac * c.F) for l in lists)
    x = synth.tokens_dev(c.d, T, seed=0)
    got = F.forward(x, lists).cpu().numpy()
    orc.set_threads(0)
    ref = orc.sparse_ffn(_host(x), _host(t["gate"]), _host(t["up"]), _host(t["down"]), c.qtype, c.d, c.F, lists)
    for i in range(T):
        close(got[i], ref[i])


# ---------------------------------------------------------------------------
# predictor and the src/moe operator API
# ---------------------------------------------------------------------------
def test_predictor_gpu(pkg, orc, kat):
    from powerinfer_x64_b200 import predictor

    k = kat["predictor_zero_weights"]
    p = predictor.Predictor.from_embedded()
    probs = p.predict(np.full(256, 0.1, np.float32))
    assert probs.size == k["output_dim"] and np.all(probs == 0.5)
    assert len(p.predict_hot(np.zeros(256), 0.5)) == k["hot_at_0_5"]
    assert len(p.predict_hot(np.zeros(256), 0.6)) == k["hot_at_0_6"]
    rng = np.random.default_rng(15)
    W1, b1 = rng.standard_normal((512, 256)).astype(np.float32) * 0.05, rng.standard_normal(512).astype(np.float32)
    W2, b2 = rng.standard_normal((128, 512)).astype(np.float32) * 0.05, rng.standard_normal(128).astype(np.float32)
    a = rng.standard_normal(256).astype(np.float32)
    q = predictor.Predictor(predictor.PredictorConfig(), W1, b1, W2, b2)
    close(q.predict(a), orc.predictor(a, W1, b1, W2, b2), rel_l2=1e-6, max_abs=1e-5)


def test_moe_router_api_kats(pkg, kat):
    from powerinfer_x64_b200 import moe

    k = kat["router_identity"]
    gw = np.zeros(k["n_embd"] * k["n_experts"], np.float32)
    for i in range(min(k["n_embd"], k["n_experts"])):
        gw[i * k["n_experts"] + i] = 1.0
    r = moe.MoeRouter(gw, k["n_embd"], k["n_experts"], k["top_k"]).route(k["x"])
    assert len(r.expert_indices) == k["top_k"] and r.expert_indices[0] == k["expect_first"]
    assert abs(sum(r.expert_weights) - 1) < k["weight_sum_tol"]
    k = kat["router_different_inputs"]
    gw = np.zeros(k["n_embd"] * k["n_experts"], np.float32)
    for i in range(k["n_embd"]):
        gw[i * k["n_experts"] + i] = 1.0
    assert moe.MoeRouter(gw, k["n_embd"], k["n_experts"], k["top_k"]).route(k["x"]).expert_indices[0] == 2
    k = kat["router_normalised"]
    n, E = k["n_embd"], k["n_experts"]
    gw = np.sin(np.arange(n * E, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    x = np.cos(np.arange(n, dtype=np.float32) * np.float32(0.3)).astype(np.float32)
    r = moe.MoeRouter(gw, n, E, k["top_k"]).route(x)
    assert abs(sum(r.expert_weights) - 1) < k["weight_sum_tol"]
    assert all(w > 0 for w in r.expert_weights) and len(set(r.expert_indices)) == k["top_k"]


def test_moe_forward_api(pkg):
    from powerinfer_x64_b200 import moe

    n_embd, E, k, f = 4, 4, 2, 8
    gw = np.zeros(n_embd * E, np.float32)
    for i in range(n_embd):
        gw[i * E + i] = 1.0
    router = moe.MoeRouter(gw, n_embd, E, k)
    ew = moe.ExpertWeights([np.full(n_embd * f, 0.1, np.float32)] * E, [np.full(n_embd * f, 0.2, np.float32)] * E,
                           [np.full(f * n_embd, 0.05, np.float32)] * E)
    out = moe.moe_forward(np.array([1, 0, 0, 0], np.float32), router, ew, n_embd, f)
    assert out.shape == (n_embd,) and np.all(np.isfinite(out))
    # all experts equal -> output = single expert output (weights sum to 1)
    single = moe.expert_forward(np.array([1, 0, 0, 0], np.float32), *ew.get_expert(0), n_embd, f)
    assert np.allclose(out, single, rtol=1e-6)


@pytest.mark.gpu
def test_forward_rejects_misaligned_rows(pkg, torch):
    """The layer kernels read and write token rows with 16-byte accesses: a token
    batch that starts off a 16-byte boundary is refused with PI_ERR_ARG instead of
    reaching the GPU."""
    from powerinfer_x64_b200 import PiError, synth

    c = synth.C1
    L = synth.moe_layer(c, seed=1)
    buf = torch.zeros(4 * c.d + 1, dtype=torch.float32, device="cuda")
    with pytest.raises(PiError):
        L.forward(buf[1:].view(4, c.d))
    out = L.forward(buf[: 4 * c.d].view(4, c.d))
    torch.cuda.synchronize()
    assert tuple(out.shape) == (4, c.d)


@pytest.mark.gpu
def test_layer_rejects_unsupported_expert_width(pkg, orc, torch):
    """Expert widths outside 128, 256, 512, 1024 are refused when the layer is built."""
    from powerinfer_x64_b200 import PiError, moe

    rng = np.random.default_rng(3)
    d, E, k, f = 1024, 4, 2, 192
    router = (rng.standard_normal(E * d) * 0.02).astype(np.float32)
    g, u, dn = (orc.quantize_q8_0((rng.standard_normal(E * f * d) * 0.02).astype(np.float32)) for _ in range(3))
    with pytest.raises(PiError):
        moe.MoeLayer(router, g, u, dn, 8, d, f, E, k)


@pytest.mark.gpu
@pytest.mark.parametrize("qt,d", [(8, 1152), (8, 4096), (2, 1152), (2, 1536)])
def test_layer_rejects_unsupported_n_embd(pkg, orc, torch, qt, d):
    """n_embd outside the widths the decode kernels are built for (Q8_0: 1024, 2048;
    Q4_0: 1024, 2048, 4096) is refused when the layer is built, not summed in part."""
    from powerinfer_x64_b200 import PiError, moe

    rng = np.random.default_rng(4)
    E, k, f = 4, 2, 256
    router = (rng.standard_normal(E * d) * 0.02).astype(np.float32)
    qz = orc.quantize_q8_0 if qt == 8 else orc.quantize_q4_0
    g, u, dn = (qz((rng.standard_normal(E * f * d) * 0.02).astype(np.float32)) for _ in range(3))
    with pytest.raises(PiError):
        moe.MoeLayer(router, g, u, dn, qt, d, f, E, k)
