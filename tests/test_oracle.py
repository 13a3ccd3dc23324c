"""CPU checks of the oracle: the reference's own known-answer tests, the
committed golden fixture, and the oracle's internal cross-checks."""
import json
import math

import numpy as np
import pytest


@pytest.fixture(scope="module")
def kat(golden_dir):
    return json.loads((golden_dir / "reference_kat.json").read_text())


def test_f16_roundtrip_all_halves(orc):
    # the half crate's f16 -> f32 is exact; f32 -> f16 is RNE: check all 2^16 patterns
    h = np.arange(1 << 16, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([orc.f16_to_f32(int(v)) for v in h], np.float32)
    finite = np.isfinite(ref)
    assert np.array_equal(got[finite].view(np.uint32), ref[finite].view(np.uint32))
    assert np.all(np.isnan(got[~finite]) == np.isnan(ref[~finite]))
    back = np.array([orc.f32_to_f16(float(v)) for v in ref[finite]], np.uint16)
    assert np.array_equal(back, h[finite])


def test_f32_to_f16_rne_matches_numpy(orc):
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-7, 1e-4, 1, 1e3, 3e4)])
    got = np.array([orc.f32_to_f16(float(v)) for v in x], np.uint16)
    assert np.array_equal(got, x.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("name,qt", [("q4_0_zero_nibbles", 2), ("q8_0_ones_half_scale", 8), ("q4_0_soak_pattern", 2)])
def test_dequant_known_answers(orc, kat, name, qt):
    k = kat[name]
    raw = np.frombuffer(bytes.fromhex(k["block_hex"]), np.uint8)
    out = orc.dequantize(raw, qt, k["rows"], k["cols"])
    expect = np.full(32, k["expect_all"], np.float32) if "expect_all" in k else np.array(k["expect"], np.float32)
    assert np.allclose(out, expect, atol=k.get("tol", 0))


def test_dequant_short_buffer_errors(orc):
    with pytest.raises(ValueError):
        orc.dequantize(np.zeros(17, np.uint8), 2, 1, 32)


def test_select_f32_kat(orc, kat):
    k = kat["select_f32"]
    raw = np.asarray(k["w"], np.float32).view(np.uint8)
    sel = orc.matvec_col_major_select(k["x"], raw, 0, k["n_in"], k["n_out"], k["indices"])
    dense = orc.matvec_col_major(k["x"], raw, 0, k["n_in"], k["n_out"])
    assert np.allclose(sel, k["expect"], atol=k["tol"])
    assert np.allclose(sel, dense[k["indices"]], atol=k["tol"])
    with pytest.raises(IndexError):
        orc.matvec_col_major_select(k["x"], raw, 0, k["n_in"], k["n_out"], [4])


def test_sparse_input_f32_kat(orc, kat):
    k = kat["sparse_input_f32"]
    raw = np.asarray(k["w"], np.float32).view(np.uint8)
    y = orc.matvec_col_major_sparse_input(k["x"], k["indices"], raw, 0, k["n_in"], k["n_out"])
    assert np.allclose(y, k["expect"], atol=k["tol"])
    assert np.all(orc.matvec_col_major_sparse_input([], [], raw, 0, k["n_in"], k["n_out"]) == 0)


def _f32_ffn_masked(k):
    # independent float32 restatement: dense SwiGLU with unselected units zeroed
    f32 = np.float32
    n_embd, n_ff = k["n_embd"], k["n_ff"]
    g = np.asarray(k["gate"], f32).reshape(n_ff, n_embd)
    u = np.asarray(k["up"], f32).reshape(n_ff, n_embd)
    d = np.asarray(k["down"], f32).reshape(n_embd, n_ff)
    x = np.asarray(k["x"], f32)
    h = np.zeros(n_ff, f32)
    for j in range(n_ff):
        gs, us = f32(0), f32(0)
        for i in range(n_embd):
            gs = f32(gs + f32(x[i] * g[j, i]))
            us = f32(us + f32(x[i] * u[j, i]))
        sig = f32(1) / f32(f32(1) + f32(math.exp(-float(gs))))
        h[j] = f32(f32(gs * sig) * us) if j in k["indices"] else 0
    out = np.zeros(n_embd, f32)
    for c in range(n_embd):
        s = f32(0)
        for j in range(n_ff):
            s = f32(s + f32(h[j] * d[c, j]))
        out[c] = s
    return out


def test_ffn_selected_f32_kat(orc, kat):
    k = kat["ffn_selected_f32"]
    pk = lambda a: np.asarray(a, np.float32).view(np.uint8)
    got = orc.ffn_swiglu_q_selected(k["x"], pk(k["gate"]), pk(k["up"]), pk(k["down"]), 0, k["n_embd"], k["n_ff"],
                                    k["indices"])
    assert np.allclose(got, _f32_ffn_masked(k), atol=k["tol"])


def test_q8_0_sse_equals_scalar(orc):
    rng = np.random.default_rng(1)
    n_in, n_out = 2048, 64
    raw = orc.quantize_q8_0(rng.standard_normal(n_in * n_out).astype(np.float32) * 0.02)
    x = rng.standard_normal(n_in).astype(np.float32)
    a = orc.matvec_col_major(x, raw, 8, n_in, n_out)
    orc.set_scalar(True)
    try:
        b = orc.matvec_col_major(x, raw, 8, n_in, n_out)
    finally:
        orc.set_scalar(False)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_q8_0_matvec_within_quantisation_bound(orc):
    rng = np.random.default_rng(2)
    n_in, n_out = 1024, 32
    w = rng.standard_normal(n_in * n_out).astype(np.float32) * 0.02
    raw = orc.quantize_q8_0(w)
    x = rng.standard_normal(n_in).astype(np.float32)
    y = orc.matvec_col_major(x, raw, 8, n_in, n_out).astype(np.float64)
    exact = w.reshape(n_out, n_in).astype(np.float64) @ x.astype(np.float64)
    # |w - wq| <= d_w/2, |x - xq| <= d_x/2 per element
    bound = (np.abs(w).reshape(n_out, -1).max(1) / 127 * np.abs(x).sum() +
             np.abs(x).max() / 127 * np.abs(w).reshape(n_out, -1).sum(1))
    assert np.all(np.abs(y - exact) <= bound)


def test_q8_0_quantiser_error_bound(orc):
    rng = np.random.default_rng(3)
    x = rng.standard_normal(32 * 100).astype(np.float32)
    deq = orc.dequantize(orc.quantize_q8_0(x), 8, 1, x.size)
    amax = np.abs(x.reshape(-1, 32)).max(1, keepdims=True)
    d = amax / 127
    # rounding (d/2) plus the f16 rounding of the stored scale (|q| <= 127, rel 2^-11)
    assert np.all(np.abs(deq.reshape(-1, 32) - x.reshape(-1, 32)) <= d * (0.5 + 127 * 2.0 ** -11) + 1e-12)


def test_q4_0_quantiser_roundtrip(orc):
    rng = np.random.default_rng(4)
    x = rng.standard_normal(32 * 100).astype(np.float32)
    deq = orc.dequantize(orc.quantize_q4_0(x), 2, 1, x.size)
    amax = np.abs(x.reshape(-1, 32)).max(1, keepdims=True)
    # one quantisation step at most: the clamp to q <= 15 costs a full step at x = -m
    assert np.all(np.abs(deq.reshape(-1, 32) - x.reshape(-1, 32)) <= amax / 8 * (1 + 16 * 2.0 ** -11) + 1e-6)


def test_routing_properties(orc):
    rng = np.random.default_rng(5)
    d, E, k, T = 256, 64, 4, 32
    router = rng.standard_normal(E * d).astype(np.float32) * 0.02
    x = rng.standard_normal((T, d)).astype(np.float32)
    r = orc.moe_route(x, router, d, E, k)
    assert np.all(np.diff(r["idx"], axis=1) > 0)  # ascending, distinct
    assert np.allclose(r["gates"].sum(1), 1, atol=1e-5)
    assert r["counts"].sum() == T * k
    assert np.array_equal(r["offsets"], np.concatenate([[0], np.cumsum(r["counts"])[:-1]]))
    for e in range(E):
        toks = r["perm"][r["offsets"][e]:r["offsets"][e] + r["counts"][e]]
        assert np.all(np.diff(toks) > 0)
        assert all(e in r["idx"][t] for t in toks)
    # selected experts carry the k largest probabilities (ties -> lowest index)
    lg = r["logits"]
    for t in range(T):
        order = sorted(range(E), key=lambda e: (-lg[t, e], e))[:k]
        assert sorted(order) == list(r["idx"][t])


def test_routing_tie_breaks_to_lowest_index(orc):
    d, E, k = 32, 8, 2
    router = np.zeros(E * d, np.float32)
    for e in (1, 3, 5):  # three equal best logits
        router[e * d] = 1.0
    r = orc.moe_route(np.eye(1, d, dtype=np.float32), router, d, E, k)
    assert list(r["idx"][0]) == [1, 3]


def test_golden_c1_fixture(orc, golden_dir):
    import make_golden

    fx = np.load(golden_dir / "c1_seed0.npz")
    inp = make_golden.c1_inputs(0)
    assert make_golden.digest(inp) == str(fx["input_sha256"])
    from powerinfer_x64_b200 import synth

    c = synth.C1
    r = orc.moe_route(inp["x"], inp["router"], c.d, c.E, c.k)
    for key in ("idx", "counts", "offsets", "perm"):
        assert np.array_equal(r[key], fx[key]), key
    assert np.array_equal(r["gates"].view(np.uint32), fx["gates"].view(np.uint32))
    out = orc.moe_layer(inp["x"], c.d, c.f, c.E, c.k, c.qtype, inp["router"], inp["gate_exps"], inp["up_exps"],
                        inp["down_exps"], threads=0)
    assert np.array_equal(out.view(np.uint32), fx["out"].view(np.uint32))  # threaded == single-thread, bitwise


def test_rms_norm_lane_order(orc):
    rng = np.random.default_rng(6)
    x = rng.standard_normal(2048).astype(np.float32)
    out = orc.rms_norm(x, np.ones_like(x))
    f32 = np.float32
    lanes = [f32(0)] * 4
    for i in range(0, 2048, 4):
        for j in range(4):
            lanes[j] = f32(lanes[j] + f32(x[i + j] * x[i + j]))
    ss = f32(f32(lanes[0] + lanes[1]) + f32(lanes[2] + lanes[3]))
    inv = f32(1) / np.sqrt(f32(ss / f32(2048) + f32(1e-6)), dtype=f32)
    assert np.array_equal(out, (x * inv).astype(f32))


def test_predictor_zero_weights(orc, kat):
    k = kat["predictor_zero_weights"]
    probs = orc.predictor(np.full(256, 0.1, np.float32), np.zeros((512, 256)), np.zeros(512), np.zeros((128, 512)),
                          np.zeros(128))
    assert probs.size == k["output_dim"] and np.all(probs == k["expect_prob"])
