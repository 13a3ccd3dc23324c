"""GGUF ingest (src/gguf/mod.rs, src/weights.rs restated): a synthetic GGUF written by
tests/golden/make_gguf.py is parsed on CPU, and on the GPU a layer built from it
matches the oracle on the same bytes."""
import numpy as np
import pytest

import make_gguf as mg


@pytest.fixture(scope="module")
def q8_file(tmp_path_factory, orc):
    path = tmp_path_factory.mktemp("gguf") / "moe_q8.gguf"
    meta, tensors, ref = mg.moe_model(qtype=mg.GGML_Q8_0)
    mg.write_gguf(path, meta, tensors)
    return path, meta, tensors, ref


@pytest.fixture(scope="module")
def q4_file(tmp_path_factory, orc):
    path = tmp_path_factory.mktemp("gguf") / "moe_q4_ggml.gguf"
    meta, tensors, ref = mg.moe_model(qtype=mg.GGML_Q4_0, q4_order="ggml", d=1024, f=256)
    mg.write_gguf(path, meta, tensors)
    return path, meta, tensors, ref


def test_gguf_parse(q8_file):
    from powerinfer_x64_b200.gguf import GgufFile

    path, meta, tensors, _ = q8_file
    gf = GgufFile(path)
    assert gf.version == 3 and gf.architecture() == "qwen35moe"
    assert gf.embedding_length() == 1024 and gf.block_count() == 2
    assert gf.moe_config() == (8, 2, 256)
    assert len(gf.tensors) == len(tensors)
    for name, shape, t, data in tensors:
        ti = gf.tensor(name)
        assert ti.shape == tuple(shape) and ti.ggml_type == t
        assert np.array_equal(gf.raw(name), np.asarray(data, np.uint8))
    # expert slices (weights.rs:78-113): expert e = bytes [e * B, (e + 1) * B)
    raw = gf.raw("blk.1.ffn_down_exps.weight")
    per = 1024 * 256 // 32 * 34
    assert np.array_equal(gf.expert_raw_slice("blk.1.ffn_down_exps.weight", 5), raw[5 * per:6 * per])
    with pytest.raises(ValueError):
        gf.expert_raw_slice("blk.1.ffn_down_exps.weight", 8)
    with pytest.raises(ValueError):
        gf.expert_raw_slice("blk.0.ffn_gate_inp.weight", 0)
    gf.close()


def test_gguf_moe_config_from_shape(tmp_path):
    """Without expert_feed_forward_length the width comes from ffn_gate_exps ne1."""
    from powerinfer_x64_b200.gguf import GgufFile

    meta = {"general.architecture": "qwen35moe", "qwen35moe.expert_count": 4, "qwen35moe.expert_used_count": 2,
            "qwen35moe.embedding_length": 64}
    t = [("blk.0.ffn_gate_exps.weight", (64, 96, 4), mg.GGML_Q8_0, np.zeros(64 * 96 * 4 // 32 * 34, np.uint8))]
    mg.write_gguf(tmp_path / "m.gguf", meta, t)
    assert GgufFile(tmp_path / "m.gguf").moe_config() == (4, 2, 96)


def test_gguf_rejects_bad_files(tmp_path):
    from powerinfer_x64_b200.gguf import GgufError, GgufFile

    (tmp_path / "bad.gguf").write_bytes(b"GGML" + b"\0" * 60)
    with pytest.raises(GgufError):
        GgufFile(tmp_path / "bad.gguf")
    meta = {"general.architecture": "qwen35moe"}
    t = [("w", (64,), mg.GGML_F32, np.zeros(256, np.uint8))]
    mg.write_gguf(tmp_path / "short.gguf", meta, t)
    data = (tmp_path / "short.gguf").read_bytes()
    (tmp_path / "short.gguf").write_bytes(data[:-100])  # truncated tensor data
    with pytest.raises(GgufError):
        GgufFile(tmp_path / "short.gguf")


def test_q4_nibble_order_round_trip(orc):
    """GGML's Q4_0 nibble order, rewritten by the loader, decodes with the reference's
    decoder to the same values GGML's layout means (element j low / j + 16 high)."""
    from powerinfer_x64_b200.gguf import q4_0_ggml_to_reference

    rng = np.random.default_rng(5)
    x = (rng.standard_normal(32 * 64) * 0.02).astype(np.float32)
    ref_order = orc.quantize_q4_0(x)
    ggml = mg.q4_reference_to_ggml(ref_order)
    assert np.array_equal(q4_0_ggml_to_reference(ggml), ref_order)
    # GGML semantics read directly from the GGML-order bytes
    b = ggml.reshape(-1, 18)
    d = b[:, :2].copy().view(np.float16).astype(np.float32).reshape(-1)
    qs = b[:, 2:]
    q = np.concatenate([qs & 0x0F, qs >> 4], axis=1).astype(np.float32) - 8.0
    assert np.array_equal((q * d[:, None]).reshape(-1), orc.dequantize(ref_order, 2, 1, x.size))


@pytest.mark.gpu
@pytest.mark.parametrize("which", ["q8", "q4"])
def test_gguf_layer_vs_oracle(orc, q8_file, q4_file, which):
    """A device layer built from the file (Q4_0 read in GGML order) against the oracle
    on the reference-order tensors, both layers of the file."""
    import torch

    from powerinfer_x64_b200 import gguf

    path, meta, tensors, ref = q8_file if which == "q8" else q4_file
    qt = 8 if which == "q8" else 2
    gf = gguf.GgufFile(path)
    rng = np.random.default_rng(7)
    x = rng.standard_normal((16, 1024)).astype(np.float32)
    for li in range(2):
        L = gguf.moe_layer(gf, li, q4_order="ggml")
        got = L.forward(torch.from_numpy(x).cuda(), rmsnorm=True, residual=True).cpu().numpy()
        r = ref[li]
        want = orc.moe_layer(x, 1024, 256, 8, 2, qt, r["router"], r["gate_exps"], r["up_exps"], r["down_exps"],
                             shared=r["shared"], threads=1, rmsnorm=True, residual=True)
        f_got, f_want = got - x, want - x
        rl2 = np.linalg.norm(f_got - f_want) / np.linalg.norm(f_want)
        ma = np.max(np.abs(f_got - f_want)) / np.sqrt(np.mean(f_want ** 2))
        assert rl2 <= 1e-3 and ma <= 2e-3, (li, rl2, ma)
