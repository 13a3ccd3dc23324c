"""Hot-neuron index producer: HotNeuronIndex (activation/mod.rs:246-325) applied as
Model::set_hot_index (model/mod.rs:1743-1802) on the host, and the device lists
from predictor probabilities (predictor/mod.rs:87-95, 64-neuron blocks) feeding
the sparse FFN with no host round trip, against the oracle."""
import numpy as np
import pytest


def _index(layers):
    from powerinfer_x64_b200.predictor import HotNeuronIndex

    return HotNeuronIndex(1, 0.5, 0.1, 100, layers)


def test_hot_index_sort_dedup_and_json(tmp_path):
    from powerinfer_x64_b200.predictor import HotNeuronIndex

    idx = _index([dict(layer_idx=1, hot_indices=[9, 3, 3, 7, 9], n_ff=16)])
    assert idx.layer(1)["hot_indices"] == [3, 7, 9] and idx.layer(0) is None
    idx.save(tmp_path / "sub" / "hot.json")
    back = HotNeuronIndex.load(tmp_path / "sub" / "hot.json")
    assert back.layers == idx.layers and back.threshold == 0.5
    assert idx.sparse_hot_indices(1, 16) == [3, 7, 9]
    assert idx.sparse_hot_indices(1, 3) is None  # as wide as the layer: dense path
    idx.validate_against_dims([16, 16])


@pytest.mark.parametrize("layers,dims,msg", [
    ([dict(layer_idx=2, hot_indices=[0], n_ff=8)], [8, 8], "out of range for model"),
    ([dict(layer_idx=0, hot_indices=[0], n_ff=8), dict(layer_idx=0, hot_indices=[1], n_ff=8)], [8], "duplicate"),
    ([dict(layer_idx=0, hot_indices=[0], n_ff=4)], [8], "expects width"),
    ([dict(layer_idx=0, hot_indices=[8], n_ff=8)], [8], "out-of-range index"),
])
def test_hot_index_validation(layers, dims, msg):
    from powerinfer_x64_b200 import PiError

    with pytest.raises(PiError, match=msg):
        _index(layers).validate_against_dims(dims)


def _expand(probs, thr, n_ff, block):
    """predict_hot per token, blocks expanded to ascending neuron ids below n_ff."""
    from powerinfer_x64_b200.predictor import blocks_to_indices

    return [blocks_to_indices(list(np.nonzero(p >= np.float32(thr))[0]), block, n_ff) for p in probs]


@pytest.mark.gpu
def test_device_lists_from_probs():
    import torch

    from powerinfer_x64_b200 import build
    from powerinfer_x64_b200.predictor import hot_lists_from_probs

    build.build()
    rng = np.random.default_rng(8)
    T, nb, block, n_ff = 5, 300, 64, 300 * 64 - 40  # last block partly past n_ff
    probs = rng.random((T, nb)).astype(np.float32)
    probs[0, :10] = 0.5  # exactly at the threshold: kept (>=)
    probs[1, 5] = np.nan  # never hot
    probs[2, :] = 0.0  # an empty list
    ptr, idx = hot_lists_from_probs(torch.from_numpy(probs).cuda(), 0.5, n_ff, block)
    ptr, idx = ptr.cpu().numpy(), idx.cpu().numpy()
    want = _expand(probs, 0.5, n_ff, block)
    assert ptr[0] == 0 and list(np.diff(ptr)) == [len(w) for w in want]
    for t in range(T):
        assert np.array_equal(idx[ptr[t]:ptr[t + 1]], want[t])


@pytest.mark.gpu
@pytest.mark.parametrize("qt", [2, 8])
def test_predicted_sparse_ffn_vs_oracle(orc, qt):
    """predictor (device) -> device lists -> sparse FFN, against the oracle's
    ffn_swiglu_q_selected on the host-expanded lists; and a static hot list."""
    import torch

    from powerinfer_x64_b200 import build, predictor

    build.build()
    rng = np.random.default_rng(9)
    n_embd, n_ff, T = 1024, 4096, 6
    q = orc.quantize_q8_0 if qt == 8 else orc.quantize_q4_0
    g, u, d = (q((rng.standard_normal(n_embd * n_ff) * 0.02).astype(np.float32)) for _ in range(3))
    F = predictor.SparseFFN(g, u, d, qt, n_embd, n_ff)
    cfg = predictor.PredictorConfig(input_dim=256, hidden_dim=512, output_dim=n_ff // 64)
    W1, b1 = rng.standard_normal((512, 256)).astype(np.float32) * 0.05, rng.standard_normal(512).astype(np.float32)
    W2, b2 = rng.standard_normal((cfg.output_dim, 512)).astype(np.float32) * 0.2, \
        rng.standard_normal(cfg.output_dim).astype(np.float32)
    P = predictor.Predictor(cfg, W1, b1, W2, b2)
    a = rng.standard_normal((T, 256)).astype(np.float32)
    probs = P.predict_batch(torch.from_numpy(a).cuda())
    x = rng.standard_normal((T, n_embd)).astype(np.float32)
    got = F.forward_predicted(torch.from_numpy(x).cuda(), probs, 0.6).cpu().numpy()
    lists = _expand(probs.cpu().numpy(), 0.6, n_ff, 64)
    assert 0 < sum(len(l) for l in lists) < T * n_ff
    ref = orc.sparse_ffn(x, g, u, d, qt, n_embd, n_ff, lists)
    for t in range(T):
        if len(lists[t]) == 0:
            assert np.all(got[t] == 0)
            continue
        err = np.linalg.norm(got[t] - ref[t]) / np.linalg.norm(ref[t])
        assert err <= 1e-3, (t, err)
    hot = np.sort(rng.choice(n_ff, 700, replace=False)).astype(np.int64)
    got = F.forward_hot(torch.from_numpy(x).cuda(), hot).cpu().numpy()
    ref = orc.sparse_ffn(x, g, u, d, qt, n_embd, n_ff, [hot] * T)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-3
