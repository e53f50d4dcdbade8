"""Model zoo and nn building blocks on the cuda backend against the oracle.

Linear, PReLU and Dropout (same counter-based draw on both sides) are
bit-exact; Sigmoid/Tanh/GELU/SiLU, softmax and the link scorers call exp,
tanh or log, whose last double ulp can differ between CUDA and the host libm,
and the models chain them, so those are held to the 1e-6 abs / 1e-5 rel bar
(f32 outputs) or 1e-12 rel (the double link scores).
"""
import numpy as np
import pytest

from oracle import model_zoo as mz
from oracle import oracle as orc
from tests.helpers import assert_bits_equal, assert_close, rand_graph

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bg():
    import browsergnn_b200 as bg

    bg.init_browsergnn()
    return bg


def _dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _inject(bg, model, rng, scale=0.3):
    """Random weights under the model's own parameter names; returns them."""
    P = {}
    for name, p in model.namedParameters():
        shape = tuple(p.tensor.shape)
        if name.endswith("epsilon"):
            P[name] = np.array([0.25], np.float32)
        else:
            P[name] = (scale * rng.standard_normal(shape)).astype(np.float32)
    model.loadStateDict(P)
    return P


# ---- building blocks -------------------------------------------------------
@pytest.mark.parametrize("m,k,n", [(1, 11, 64), (130, 77, 65), (1000, 64, 1), (257, 192, 33)])
@pytest.mark.parametrize("bias", [True, False])
def test_dense_bits(bg, m, k, n, bias):
    rng = np.random.default_rng(m * 7 + k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((n, k)).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32) if bias else None
    lin = bg.Linear(inFeatures=k, outFeatures=n, bias=bias)
    lin.loadStateDict({"weight": w, **({"bias": b} if bias else {})})
    got = lin.forward(_dev(x)).cpu().numpy()
    assert_bits_equal(got, orc.linear(x, w, b), "Linear")
    # 1-D input: [in] -> [out]
    got1 = lin.forward(_dev(x[0])).cpu().numpy()
    assert got1.shape == (n,)
    assert_bits_equal(got1, orc.linear(x[:1], w, b).reshape(n), "Linear 1-D")


def test_linear_errors(bg):
    lin = bg.Linear(inFeatures=4, outFeatures=2)
    with pytest.raises(ValueError, match="Expected input size 4, got 3"):
        lin.forward(_dev(np.zeros((2, 3), np.float32)))
    with pytest.raises(ValueError, match="expects 1D or 2D"):
        lin.forward(_dev(np.zeros((2, 2, 4), np.float32)))


@pytest.mark.parametrize("name", ["sigmoid", "tanh", "gelu", "silu"])
def test_new_activations(bg, name):
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(5000) * 4, [0.0, -0.0, 30.0, -30.0, 90.0, -90.0,
                                                        np.inf, -np.inf]]).astype(np.float32)
    mod = {"sigmoid": bg.Sigmoid, "tanh": bg.Tanh, "gelu": bg.GELU, "silu": bg.SiLU}[name]()
    got = mod.forward(_dev(x)).cpu().numpy()
    want = getattr(orc, name)(x)
    assert_close(got, want, name)


def test_sigmoid_softmax_reference_cases(bg):
    # tests/tensor.test.ts:129-148
    s = bg.Sigmoid().forward(_dev(np.array([0.0], np.float32))).cpu().numpy()
    assert abs(float(s[0]) - 0.5) < 1e-7
    sm = bg.Softmax().forward(_dev(np.array([[1, 2, 3]], np.float32))).cpu().numpy()[0]
    assert abs(float(sm.sum()) - 1) < 1e-6 and sm[0] < sm[1] < sm[2]


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 7), (1, 50000), (64, 1025)])
@pytest.mark.parametrize("log", [False, True])
def test_softmax_rows(bg, rows, cols, log):
    import torch

    rng = np.random.default_rng(rows * 31 + cols)
    x = (rng.standard_normal((rows, cols)) * 5).astype(np.float32)
    mask = (rng.random(cols) < 0.2).astype(np.uint8)
    for m in (None, mask):
        out = torch.empty((rows, cols), dtype=torch.float32, device="cuda")
        mt = None if m is None else _dev(m)
        bg.get_context().call("bgnn_softmax_rows", _dev(x).data_ptr(), rows, cols,
                              None if mt is None else mt.data_ptr(), -1e9, int(log),
                              out.data_ptr())
        want = orc.softmax_rows(x, col_mask=m, mask_value=-1e9, log=log)
        assert_close(out.cpu().numpy(), want, f"softmax log={log} mask={m is not None}")


def test_softmax_nan_and_errors(bg):
    x = np.array([[1.0, np.nan, 2.0], [0.0, -0.0, 0.0]], np.float32)
    got = bg.Softmax().forward(_dev(x)).cpu().numpy()
    want = orc.softmax_rows(x)
    assert np.isnan(got[0]).all() and np.isnan(want[0]).all()
    assert_close(got[1], want[1], "zeros")
    with pytest.raises(ValueError, match="only supports 2D"):
        bg.Softmax().forward(_dev(np.zeros(3, np.float32)))


@pytest.mark.parametrize("p", [0.0, 0.1, 0.5, 1.0])
def test_dropout_bits(bg, p):
    rng = np.random.default_rng(9)
    x = rng.standard_normal(100003).astype(np.float32)
    d = bg.Dropout(p)
    got = d.forward(_dev(x), seed=1234).cpu().numpy()
    if p == 0.0:
        assert_bits_equal(got, x, "p=0 identity")
    else:
        assert_bits_equal(got, orc.dropout(x, p, 1234), f"dropout p={p}")
    d.eval()
    assert_bits_equal(d.forward(_dev(x)).cpu().numpy(), x, "eval identity")
    with pytest.raises(ValueError):
        bg.Dropout(1.5)


def test_prelu_bits(bg):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((33, 7)).astype(np.float32)
    for k in (1, 7):
        mod = bg.PReLU(k, 0.25)
        w = rng.standard_normal(k).astype(np.float32)
        mod.loadStateDict({"weight": w})
        got = mod.forward(_dev(x)).cpu().numpy()
        assert_bits_equal(got, orc.prelu(x, w), f"prelu k={k}")


@pytest.mark.parametrize("mode", ["dot", "bilinear", "mlp"])
def test_link_scores(bg, mode):
    import torch

    rng = np.random.default_rng(3)
    n, d, q = 300, 48, 5000
    emb = rng.standard_normal((n, d)).astype(np.float32) * 0.3
    src = rng.integers(0, n, q).astype(np.uint32)
    tgt = rng.integers(0, n, q).astype(np.uint32)
    wb = (rng.standard_normal((d, d)) * 0.2).astype(np.float32)
    w1 = (rng.standard_normal((d, 3 * d)) * 0.2).astype(np.float32)
    b1 = rng.standard_normal(d).astype(np.float32) * 0.1
    w2 = (rng.standard_normal((1, d)) * 0.2).astype(np.float32)
    b2 = rng.standard_normal(1).astype(np.float32) * 0.1
    want = orc.link_scores(emb, src, tgt, mode, w_bilinear=wb, w1=w1, b1=b1, w2=w2, b2=b2)
    out = torch.empty(q, dtype=torch.float64, device="cuda")
    dv = {k: _dev(v) for k, v in dict(emb=emb, src=src.view(np.int32), tgt=tgt.view(np.int32),
                                       wb=wb, w1=w1, b1=b1, w2=w2, b2=b2).items()}
    bg.get_context().call("bgnn_link_scores", dv["emb"].data_ptr(), n, d, dv["src"].data_ptr(),
                          dv["tgt"].data_ptr(), q, {"dot": 0, "bilinear": 1, "mlp": 2}[mode],
                          dv["wb"].data_ptr(), dv["w1"].data_ptr(), dv["b1"].data_ptr(),
                          dv["w2"].data_ptr(), dv["b2"].data_ptr(), out.data_ptr())
    got = out.cpu().numpy()
    assert np.allclose(got, want, rtol=1e-12, atol=1e-15), np.abs(got - want).max()


def test_link_scores_bad_index(bg):
    import torch

    emb = _dev(np.zeros((4, 8), np.float32))
    src = _dev(np.array([0, 9], np.int32))
    out = torch.empty(2, dtype=torch.float64, device="cuda")
    ctx = bg.get_context()
    ctx.call("bgnn_link_scores", emb.data_ptr(), 4, 8, src.data_ptr(), src.data_ptr(), 2, 0,
             None, None, None, None, None, out.data_ptr())
    with pytest.raises(bg.BGNNError, match="OUT_OF_RANGE"):
        ctx.synchronize()


def test_gat_attention_dropout_bits(bg):
    rng = np.random.default_rng(4)
    n, fin, heads, c = 800, 24, 4, 8
    ei, e = rand_graph(n, 6000, 8, hub_deg=400)
    x = rng.standard_normal((n, fin)).astype(np.float32)
    layer = bg.GATConv(inChannels=fin, outChannels=c, heads=heads, dropout=0.3)
    P = _inject(bg, layer, rng)
    ctx = bg.get_context()
    ctx.set_math(True)
    try:
        g = bg.GraphData(x=x, numNodes=n, numFeatures=fin, edgeIndex=ei, numEdges=e)
        got = layer.forward(g, seed=77).x.cpu().numpy()
    finally:
        ctx.set_math(False)
    want = orc.gat_forward(x, n, fin, ei, e, P["weight"], P["att_src"], P["att_dst"], P["bias"],
                           heads, c, dropout=0.3, seed=77).reshape(n, heads * c)
    assert_close(got, want, "GAT train dropout")
    # dropout really removed attention mass: differs from the eval output
    layer.eval()
    ev = layer.forward(g).x.cpu().numpy()
    assert not np.allclose(ev, got)


# ---- models -------------------------------------------------------------------
def _graph(bg, rng, n=400, e=2400, f=11):
    ei, e = rand_graph(n, e, int(rng.integers(1 << 30)), hub_deg=300, loops=2, dup=5)
    x = rng.standard_normal((n, f)).astype(np.float32)
    return bg.GraphData(x=x, numNodes=n, numFeatures=f, edgeIndex=ei, numEdges=e), x, ei, e


@pytest.mark.parametrize("attention", [False, True])
@pytest.mark.parametrize("residual", [True, False])
def test_student_mastery(bg, attention, residual):
    rng = np.random.default_rng(10 + attention * 2 + residual)
    g, x, ei, e = _graph(bg, rng)
    m = bg.StudentMasteryPredictor(inputFeatures=11, hiddenDim=32, useAttention=attention,
                                   numHeads=4, residual=residual).eval()
    P = _inject(bg, m, rng)
    got = m.forward(g).cpu().numpy()
    want = mz.student_mastery(x, ei, e, P, use_attention=attention, residual=residual)
    assert got.shape == (400, 1)
    assert_close(got, want, "StudentMasteryPredictor")
    res = m.predict(g)
    assert len(res["mastery"]) == 400
    assert all(p["mastered"] == (p["score"] >= 0.7) for p in res["predictions"])
    weak = m.getWeakConcepts(g, 5)
    scores = [w["score"] for w in weak]
    assert scores == sorted(scores) and scores[0] == min(res["mastery"])


@pytest.mark.parametrize("variant", ["mean", "max", "sum", "pool", "gin"])
def test_learning_path(bg, variant):
    rng = np.random.default_rng(20 + len(variant))
    g, x, ei, e = _graph(bg, rng)
    gin = variant == "gin"
    m = bg.LearningPathRecommender(inputFeatures=11, hiddenDim=32, numLayers=3,
                                   aggregator="mean" if gin else variant, useGIN=gin).eval()
    P = _inject(bg, m, rng)
    mask = [bool(v) for v in rng.random(400) < 0.1]
    for mk in (None, mask):
        got = m.forward(g, mk).cpu().numpy()
        want = mz.learning_path(x, ei, e, P, aggregator="mean" if gin else variant, use_gin=gin,
                                mask=mk)
        assert_close(got, want, f"LearningPathRecommender {variant} mask={mk is not None}")
    rec = m.recommend(g, [1, 2, 3], 4)
    assert [r["rank"] for r in rec["recommendations"]] == [1, 2, 3, 4]
    assert all(r["nodeIndex"] not in (1, 2, 3) for r in rec["recommendations"])
    path = m.getLearningPath(g, [0], [5, 6], maxSteps=3)
    assert len(path["path"]) <= 3


def test_learning_path_unnormalised(bg):
    rng = np.random.default_rng(33)
    g, x, ei, e = _graph(bg, rng)
    m = bg.LearningPathRecommender(inputFeatures=11, hiddenDim=16, normalizeScores=False).eval()
    P = _inject(bg, m, rng)
    mask = [i % 7 == 0 for i in range(400)]
    got = m.forward(g, mask).cpu().numpy()
    want = mz.learning_path(x, ei, e, P, mask=mask, normalize_scores=False)
    assert_close(got, want, "unnormalised scores")


@pytest.mark.parametrize("attention", [True, False])
@pytest.mark.parametrize("link", ["dot", "bilinear", "mlp"])
def test_concept_mapper(bg, attention, link):
    rng = np.random.default_rng(40 + attention + len(link))
    g, x, ei, e = _graph(bg, rng, n=60, e=300, f=20)
    m = bg.ConceptPrerequisiteMapper(inputFeatures=20, hiddenDim=32, useAttention=attention,
                                     linkPredictor=link).eval()
    P = _inject(bg, m, rng)
    emb = m.encode(g)
    want_emb = mz.concept_encode(x, ei, e, P, use_attention=attention)
    assert_close(emb.cpu().numpy(), want_emb, "encode")
    res = m.predictAllLinks(g)
    assert len(res["pairs"]) == 60 * 59
    src = [p["src"] for p in res["pairs"]]
    tgt = [p["tgt"] for p in res["pairs"]]
    # score the pairs from the oracle's own embeddings
    want = mz.concept_links(want_emb, np.array(src), np.array(tgt), P, link)
    assert_close(np.array(res["scores"]), want, f"link scores {link}")
    disc = m.discoverPrerequisites(g, threshold=0.0, topK=10)
    assert len(disc["newEdges"]) == 10
    assert all(f"{p['src']}->{p['tgt']}" not in disc["existingEdges"] for p in disc["newEdges"])


def test_sample_graphs_and_critical_path(bg):
    g1 = bg.StudentMasteryPredictor.createSampleGraph(10)
    assert g1.numNodes == 10 and g1.numFeatures == 11 and g1.numEdges == 2 * 9 + 2 * 3
    g2 = bg.LearningPathRecommender.createSampleCurriculum(15)
    assert g2.numNodes == 15 and g2.numFeatures == 11
    g3 = bg.ConceptPrerequisiteMapper.createSampleConceptGraph(12)
    assert g3.numNodes == 12 and g3.numFeatures == 20
    m = bg.ConceptPrerequisiteMapper(inputFeatures=20)
    cp = m.findCriticalPath(g3, 0)
    assert cp["length"] == len(cp["path"]) - 1 and cp["path"][0] == 0
    sm = bg.StudentMasteryPredictor(inputFeatures=11)
    assert len(sm.predict(g1)["mastery"]) == 10
    lp = bg.LearningPathRecommender(inputFeatures=11)
    assert len(lp.recommend(g2, [0], 3)["recommendations"]) == 3


def test_training_mode_forward_runs(bg):
    # the models default to training mode (Dropout and GAT attention dropout
    # active); the forward runs on the device generator and differs from eval
    bg.manual_seed(5)
    g = bg.ConceptPrerequisiteMapper.createSampleConceptGraph(12)
    m = bg.ConceptPrerequisiteMapper(inputFeatures=20, linkPredictor="dot")
    t1 = m.forward(g).cpu().numpy()
    bg.manual_seed(5)
    t2 = m.forward(g).cpu().numpy()
    assert_bits_equal(t1, t2, "same seed, same draws")
    ev = m.eval().forward(g).cpu().numpy()
    assert not np.allclose(ev, t1)


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("n", [47, 130, 256])
def test_linear_add_is_sage_linear_split(bg, n, exact):
    """bgnn_linear (self product) then bgnn_linear_add (neighbour product
    added to it) gives bgnn_sage_linear's bits: the fused launch (both
    products per output tile) rounds exactly like the two launches, in both
    math modes and for the 64- and 128-column tiles."""
    import torch

    rng = np.random.default_rng(n)
    m, k = 700, 100
    x = rng.standard_normal((m, k)).astype(np.float32)
    agg = rng.standard_normal((m, k)).astype(np.float32)
    ws = (rng.standard_normal((k, n)) * 0.1).astype(np.float32)
    wn = (rng.standard_normal((k, n)) * 0.1).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    d = {kk: _dev(v) for kk, v in dict(x=x, agg=agg, ws=ws, wn=wn, b=b).items()}
    ctx = bg.get_context()
    ctx.set_math(exact)
    try:
        st = torch.empty((m, n), dtype=torch.float32, device="cuda")
        out = torch.empty_like(st)
        ref = torch.empty_like(st)
        ctx.call("bgnn_linear", d["x"].data_ptr(), d["ws"].data_ptr(), m, k, n, None, 0, 0.0,
                 st.data_ptr())
        ctx.call("bgnn_linear_add", d["agg"].data_ptr(), d["wn"].data_ptr(), m, k, n,
                 st.data_ptr(), d["b"].data_ptr(), 1, 0.0, out.data_ptr())
        ctx.call("bgnn_sage_linear", d["agg"].data_ptr(), d["x"].data_ptr(), d["wn"].data_ptr(),
                 d["ws"].data_ptr(), m, k, n, d["b"].data_ptr(), 1, 0.0, ref.data_ptr())
    finally:
        ctx.set_math(False)
    assert_bits_equal(out.cpu().numpy(), ref.cpu().numpy(), "split vs fused")
    # the oracle's SAGE combine (sage.ts:171-196): f32(St + Nt), + bias, ReLU
    st_o = orc.matmul(x, ws, m, k, n).reshape(m, n)
    nt_o = orc.matmul(agg, wn, m, k, n).reshape(m, n)
    comb = (st_o.astype(np.float64) + nt_o).astype(np.float32)
    comb = (comb.astype(np.float64) + b).astype(np.float32)
    if exact:
        assert_bits_equal(out.cpu().numpy(), orc.relu(comb), "vs oracle")
    else:
        assert_close(out.cpu().numpy(), orc.relu(comb), "vs oracle")


def test_sage_linear_k0(bg):
    """No input features: both products are empty, the output is
    act(f32(0 + 0) + bias) (the fused launch is skipped for k == 0)."""
    import torch

    m, n = 300, 40
    b = np.linspace(-1, 1, n).astype(np.float32)
    db = _dev(b)
    out = torch.full((m, n), float("nan"), device="cuda")
    dummy = torch.zeros(1, device="cuda")
    ctx = bg.get_context()
    ctx.call("bgnn_sage_linear", dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(),
             dummy.data_ptr(), m, 0, n, db.data_ptr(), 1, 0.0, out.data_ptr())
    assert_bits_equal(out.cpu().numpy(), np.tile(np.maximum(b, 0), (m, 1)), "k == 0")


def test_pinned_host_graphdata_overlaps_upload(bg):
    """GraphData from pinned host tensors (edges uploaded first, features on
    a copy stream) gives the same layer output as from numpy arrays."""
    import torch

    rng = np.random.default_rng(12)
    n, f = 3000, 24
    ei, e = rand_graph(n, 20000, 6, hub_deg=800, loops=3)
    x = rng.standard_normal((n, f)).astype(np.float32)
    conv = bg.SAGEConv(inChannels=f, outChannels=16)
    _inject(bg, conv, rng)
    want = conv.forward(bg.GraphData(x=x, numNodes=n, numFeatures=f, edgeIndex=ei,
                                     numEdges=e)).x.cpu().numpy()
    xh = torch.from_numpy(x).pin_memory()
    eh = torch.from_numpy(ei.view(np.int32)).pin_memory()
    g = bg.GraphData(x=xh, numNodes=n, numFeatures=f, edgeIndex=eh, numEdges=e)
    got = conv.forward(g).x.cpu().numpy()
    assert_bits_equal(got, want, "pinned-host GraphData")
    assert g.addSelfLoops().numEdges >= e


def test_captured_forward_replays_bits(bg):
    """A GIN stack + pool captured in a CUDA graph replays the eager bits, and
    picks up new features written into the captured input buffer."""
    import torch

    rng = np.random.default_rng(21)
    n, f = 2000, 32
    ei, e = rand_graph(n, 12000, 9, hub_deg=400)
    x = rng.standard_normal((n, f)).astype(np.float32)
    batch = np.sort(rng.integers(0, 40, n)).astype(np.uint32)
    g = bg.GraphData(x=x, numNodes=n, numFeatures=f, edgeIndex=ei, numEdges=e, batch=batch)
    gd = g.withFeatures(g.x_device())
    layers = [bg.GINConv(inChannels=f, outChannels=64), bg.GINConv(inChannels=64, outChannels=64)]
    for lay in layers:
        _inject(bg, lay, rng, scale=0.2)

    def step():
        h = gd
        for i, lay in enumerate(layers):
            h = lay.forward(h, _act="relu" if i == 0 else None)
        return bg.global_sum_pool(h, 40)

    eager = step().cpu().numpy()
    cap = bg.CapturedForward(step)
    assert_bits_equal(cap().cpu().numpy(), eager, "replay")
    x2 = rng.standard_normal((n, f)).astype(np.float32)
    gd.x.copy_(torch.from_numpy(x2).cuda())
    want2 = step().cpu().numpy()
    assert_bits_equal(cap().cpu().numpy(), want2, "replay with new features")
    cap.close()
