"""Weight I/O (src/utils/serialization.ts) and the model zoo's parameter
layout, on CPU: the cases of the reference's tests/serialization.test.ts,
plus the oracle's restatements of the nn building blocks against plain numpy
and the reference's own activation cases (tests/tensor.test.ts:118-148)."""
import json

import numpy as np
import pytest

import browsergnn_b200 as bg
from oracle import oracle as orc


def test_serialize_gcn_layer():
    layer = bg.GCNConv(inChannels=4, outChannels=8)
    s = bg.serializeModel(layer, "test-gcn")
    assert s["name"] == "test-gcn" and s["version"]
    assert len(s["parameters"]) > 0
    assert s["metadata"]["numParameters"] == layer.numParameters()
    s2 = bg.serializeModel(layer, "m", {"description": "Test model", "author": "Dr. Lee"})
    assert s2["metadata"]["description"] == "Test model" and s2["metadata"]["author"] == "Dr. Lee"
    sd = bg.deserializeModel(s)
    assert len(sd) > 0


def test_parameter_values_survive():
    layer = bg.GCNConv(inChannels=4, outChannels=8)
    s = bg.serializeModel(layer)
    s["parameters"][0]["data"][0] = 999.5
    sd = bg.deserializeModel(s)
    assert sd[s["parameters"][0]["name"]]["tensor"].reshape(-1)[0] == 999.5


def test_state_dict_roundtrip_and_reports():
    layer = bg.GCNConv(inChannels=4, outChannels=8)
    sd = bg.getStateDict(layer)
    assert sd["weight"]["tensor"].shape == (4, 8)
    other = bg.GCNConv(inChannels=4, outChannels=8)
    sd["weight"]["tensor"][0, 0] = 0.5
    missing, unexpected = bg.loadStateDict(other, sd)
    assert missing == [] and unexpected == []
    assert bg.getStateDict(other)["weight"]["tensor"][0, 0] == 0.5
    only_w = {"weight": sd["weight"]}
    missing, _ = bg.loadStateDict(bg.GCNConv(inChannels=4, outChannels=8), only_w, strict=False)
    assert "bias" in missing
    extra = dict(sd)
    extra["extra_key"] = {"tensor": np.zeros(3, np.float32)}
    _, unexpected = bg.loadStateDict(bg.GCNConv(inChannels=4, outChannels=8), extra, strict=False)
    assert "extra_key" in unexpected
    with pytest.raises(ValueError, match="State dict mismatch"):
        bg.loadStateDict(bg.GCNConv(inChannels=4, outChannels=8), only_w)
    bad = {"weight": {"tensor": np.zeros((8, 4), np.float32)}, "bias": sd["bias"]}
    with pytest.raises(ValueError, match='Shape mismatch for parameter "weight"'):
        bg.loadStateDict(bg.GCNConv(inChannels=4, outChannels=8), bad)


def test_json_roundtrip_and_sequential():
    layer = bg.GCNConv(inChannels=4, outChannels=8)
    sd = bg.getStateDict(layer)
    sd["weight"]["tensor"][0, 0] = 123.456
    bg.loadStateDict(layer, sd)
    text = bg.saveModelToJSON(layer, "json-test")
    layer2 = bg.GCNConv(inChannels=4, outChannels=8)
    res = bg.loadModelFromJSON(layer2, text)
    assert res["missing"] == [] and res["unexpected"] == [] and res["model"]["name"] == "json-test"
    assert abs(float(layer2.parameters()[0].tensor.reshape(-1)[0]) - 123.456) < 1e-3
    model = bg.Sequential([bg.Linear(inFeatures=10, outFeatures=8), bg.ReLU(),
                           bg.Linear(inFeatures=8, outFeatures=4)])
    parsed = json.loads(bg.saveModelToJSON(model, "sequential-test"))
    assert parsed["name"] == "sequential-test" and len(parsed["parameters"]) == 4
    assert [p["name"] for p in parsed["parameters"]] == ["0.weight", "0.bias", "2.weight",
                                                         "2.bias"]


def test_model_size():
    size = bg.getModelSize(bg.GCNConv(inChannels=16, outChannels=8))
    assert (size["parameters"], size["bytes"], size["formatted"]) == (136, 544, "544 B")
    model = bg.Sequential([bg.Linear(inFeatures=256, outFeatures=512),
                           bg.Linear(inFeatures=512, outFeatures=256)])
    size = bg.getModelSize(model)
    assert size["parameters"] == 262912 and size["bytes"] == 1051648 and "MB" in size["formatted"]


def test_browser_only_helpers():
    with pytest.raises(RuntimeError, match="only available in browser environment"):
        bg.serialization.downloadModel(bg.Linear(inFeatures=2, outFeatures=2))
    assert bg.serialization.listSavedModels() == []
    assert bg.serialization.deleteSavedModel("x") is False


def test_model_zoo_parameter_names():
    """Names follow the reference's registerModule / registerParameter order,
    so a state dict saved by the reference loads unchanged."""
    sm = bg.StudentMasteryPredictor(inputFeatures=11, hiddenDim=16)
    assert [n for n, _ in sm.namedParameters()] == [
        "inputProj.weight", "inputProj.bias", "gnn_0.weight", "gnn_0.bias", "gnn_1.weight",
        "gnn_1.bias", "outputHead.0.weight", "outputHead.0.bias"]
    assert tuple(dict(sm.namedParameters())["inputProj.weight"].tensor.shape) == (16, 11)
    lp = bg.LearningPathRecommender(inputFeatures=11, hiddenDim=16, useGIN=True, numLayers=1)
    assert [n for n, _ in lp.namedParameters()] == [
        "inputProj.0.weight", "inputProj.0.bias", "gnn_0.epsilon", "gnn_0.mlp_weight1",
        "gnn_0.mlp_bias1", "gnn_0.mlp_weight2", "gnn_0.mlp_bias2", "scoringHead.0.weight",
        "scoringHead.0.bias", "scoringHead.2.weight", "scoringHead.2.bias"]
    cm = bg.ConceptPrerequisiteMapper(inputFeatures=20, hiddenDim=16, linkPredictor="bilinear",
                                      numLayers=1)
    assert [n for n, _ in cm.namedParameters()][:1] == ["bilinearWeight"]
    cm = bg.ConceptPrerequisiteMapper(inputFeatures=20, hiddenDim=16, numLayers=1)
    names = [n for n, _ in cm.namedParameters()]
    assert names[-4:] == ["linkPredictor.0.weight", "linkPredictor.0.bias",
                          "linkPredictor.3.weight", "linkPredictor.3.bias"]
    assert tuple(dict(cm.namedParameters())["linkPredictor.0.weight"].tensor.shape) == (16, 48)
    assert str(cm) == "ConceptPrerequisiteMapper(20 -> GATx1 -> mlp)"
    with pytest.raises(ValueError, match="Invalid typed array length"):
        bg.LearningPathRecommender(inputFeatures=11, hiddenDim=15)


# ---- oracle restatements of the nn building blocks ---------------------------
def test_oracle_linear_is_double_sum():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((17, 33)).astype(np.float32)
    w = rng.standard_normal((5, 33)).astype(np.float32)
    b = rng.standard_normal(5).astype(np.float32)
    want = (x.astype(np.float64) @ w.T.astype(np.float64)).astype(np.float32)
    want = (want.astype(np.float64) + b).astype(np.float32)
    got = orc.linear(x, w, b)
    # numpy's double matmul may reassociate; the sums agree to double rounding
    assert np.array_equal(got, want) or np.abs(got - want).max() <= 1e-6


def test_oracle_activation_kats():
    # tests/tensor.test.ts:119-148
    assert orc.relu(np.array([-1, 0, 1, 2], np.float32)).tolist() == [0, 0, 1, 2]
    assert abs(float(orc.sigmoid(np.array([0], np.float32))[0]) - 0.5) < 1e-7
    sm = orc.softmax_rows(np.array([[1, 2, 3]], np.float32))[0]
    assert abs(float(sm.sum()) - 1) < 1e-6 and sm[0] < sm[1] < sm[2]
    ls = orc.softmax_rows(np.array([[1, 2, 3]], np.float32), log=True)[0]
    assert np.allclose(np.exp(ls.astype(np.float64)), sm, atol=1e-6)
    x = np.linspace(-6, 6, 101).astype(np.float32)
    assert np.allclose(orc.tanh(x), np.tanh(x.astype(np.float64)), atol=1e-7)
    assert np.allclose(orc.silu(x), x / (1 + np.exp(-x.astype(np.float64))), atol=1e-6)
    g = 0.5 * x * (1 + np.tanh(np.sqrt(2 / np.pi) * (x + 0.044715 * x.astype(np.float64) ** 3)))
    assert np.allclose(orc.gelu(x), g, atol=1e-6)
    assert orc.prelu(np.array([-2, 3], np.float32), np.array([0.25], np.float32)).tolist() == [-0.5, 3]


def test_oracle_masked_softmax():
    x = np.array([[0.5, 2.0, 1.0, -1.0]], np.float32)
    m = np.array([0, 1, 0, 0], np.uint8)
    got = orc.softmax_rows(x, col_mask=m, mask_value=-1e9)[0]
    assert got[1] == 0.0
    e = np.exp(np.array([0.5, 1.0, -1.0]) - 1.0)
    assert np.allclose(got[[0, 2, 3]], e / e.sum(), atol=1e-7)


def test_oracle_dropout_draws():
    u = np.array([orc.uniform(42, i) for i in range(20000)])
    assert 0.0 <= u.min() and u.max() < 1.0 and abs(u.mean() - 0.5) < 0.01
    x = np.ones(20000, np.float32)
    d = orc.dropout(x, 0.25, 42)
    kept = d != 0
    assert abs(kept.mean() - 0.75) < 0.01
    assert np.all(d[kept] == np.float32(1 / 0.75))
    assert np.array_equal(kept, u > 0.25)


def test_oracle_link_dot_matches_numpy():
    rng = np.random.default_rng(3)
    emb = rng.standard_normal((10, 6)).astype(np.float32)
    src, tgt = np.array([0, 3, 9]), np.array([1, 3, 2])
    got = orc.link_scores(emb, src, tgt, "dot")
    dots = np.array([float(np.dot(emb[s].astype(np.float64), emb[t].astype(np.float64)))
                     for s, t in zip(src, tgt)])
    assert np.allclose(got, 1 / (1 + np.exp(-dots)), rtol=1e-14)
