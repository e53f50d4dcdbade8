"""Layer forwards on the cuda backend against the oracle's restatement of the
reference layers, with the reference's parameter names injected.

BGNN_MATH_EXACT reproduces the reference's bits (GCN, SAGE, GIN); GAT and
ELU call exp, whose last double ulp can differ between CUDA and the host libm,
so those are held to the 1e-5 rel / 1e-6 abs bar.  BGNN_MATH_FAST is held to
the same bar everywhere.
"""
import numpy as np
import pytest

from browsergnn_b200 import synth
from oracle import oracle as orc
from tests.helpers import assert_bits_equal, assert_close, loopless, rand_graph

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bg():
    import browsergnn_b200 as bg

    bg.init_browsergnn()
    return bg


@pytest.fixture(params=[True, False], ids=["exact", "fast"])
def mode(bg, request):
    ctx = bg.get_context()
    ctx.set_math(request.param)
    yield request.param
    ctx.set_math(False)


def weights(rng, *shape, fan=None):
    fan = fan or (shape[0], shape[-1])
    return synth.glorot(fan[0], fan[1], rng, shape=shape)


def check(got, want, exact_bits, what):
    if exact_bits:
        assert_bits_equal(got, want, what)
    else:
        assert_close(got, want, what)


def test_reference_layer_shapes(bg):
    # tests/layers.test.ts:14-30 graph, shape-only checks of the reference
    g = bg.GraphData(x=[1, 0, 0, 0, 1, 0, 0, 0, 1, 1, 1, 1], numNodes=4, numFeatures=3,
                     edgeIndex=[0, 0, 1, 1, 2, 2, 3, 3, 1, 3, 0, 2, 1, 3, 0, 2], numEdges=8)
    assert bg.GCNConv(inChannels=3, outChannels=16).numParameters() == 3 * 16 + 16
    assert bg.GCNConv(inChannels=3, outChannels=8, bias=False).numParameters() == 24
    assert tuple(bg.GCNConv(inChannels=3, outChannels=8).forward(g).x.shape) == (4, 8)
    assert tuple(bg.GCNConv(inChannels=3, outChannels=8, normalize=False).forward(g).x.shape) == (4, 8)
    with pytest.raises(ValueError):
        bg.GCNConv(inChannels=5, outChannels=8).forward(g)
    gat = bg.GATConv(inChannels=3, outChannels=8, heads=2)
    assert tuple(gat.forward(g).x.shape) == (4, 16)
    assert tuple(bg.GATConv(inChannels=3, outChannels=8, heads=2, concat=False).forward(g).x.shape) == (4, 8)
    for aggr in ("mean", "max", "sum", "pool"):
        assert tuple(bg.SAGEConv(inChannels=3, outChannels=8, aggregator=aggr).forward(g).x.shape) == (4, 8)
    assert tuple(bg.SAGEConv(inChannels=3, outChannels=8, rootWeight=False).forward(g).x.shape) == (4, 8)
    out = bg.SAGEConv(inChannels=3, outChannels=8, normalize=True).forward(g).x.cpu().numpy()
    norms = np.sqrt((out.astype(np.float64) ** 2).sum(1))  # layers.test.ts:254-275
    assert np.all((np.abs(norms - 1) < 1e-5) | (norms == 0))
    assert tuple(bg.GINConv(inChannels=3, outChannels=8).forward(g).x.shape) == (4, 8)


@pytest.mark.parametrize("case", ["loopless", "has_loops", "hub"])
def test_gcn(bg, mode, case):
    rng = np.random.default_rng(11)
    n, fin, fout = 1500, 40, 16
    if case == "loopless":
        ei, e = loopless(n, 9000, 1)
    else:
        ei, e = rand_graph(n, 9000, 2, hub_deg=2000 if case == "hub" else 0, loops=3)
    x = rng.standard_normal((n, fin)).astype(np.float32)
    w = weights(rng, fin, fout)
    b = rng.standard_normal(fout).astype(np.float32)
    layer = bg.GCNConv(inChannels=fin, outChannels=fout)
    layer.loadStateDict({"weight": w, "bias": b})
    g = bg.GraphData(x=x, numNodes=n, numFeatures=fin, edgeIndex=ei, numEdges=e)
    got = layer.forward(g).x.cpu().numpy()
    want = orc.gcn_forward(x, n, fin, ei, e, w, b, fout, True, True).reshape(n, fout)
    check(got, want, mode, f"gcn {case}")


def test_gcn_without_normalize_or_loops(bg, mode):
    rng = np.random.default_rng(12)
    n, fin, fout = 300, 9, 5
    ei, e = loopless(n, 2000, 3)
    x = rng.standard_normal((n, fin)).astype(np.float32)
    w = weights(rng, fin, fout)
    for add_loops, norm in ((False, True), (True, False), (False, False)):
        layer = bg.GCNConv(inChannels=fin, outChannels=fout, addSelfLoops=add_loops,
                           normalize=norm, bias=False)
        layer.loadStateDict({"weight": w})
        g = bg.GraphData(x=x, numNodes=n, numFeatures=fin, edgeIndex=ei, numEdges=e)
        got = layer.forward(g).x.cpu().numpy()
        want = orc.gcn_forward(x, n, fin, ei, e, w, None, fout, add_loops, norm).reshape(n, fout)
        check(got, want, mode, f"gcn loops={add_loops} norm={norm}")


@pytest.mark.parametrize("heads,c,concat", [(8, 8, True), (1, 16, True), (4, 5, False),
                                            (3, 7, True)])
@pytest.mark.parametrize("loops", ["loopless", "has_loops"])
def test_gat(bg, mode, heads, c, concat, loops):
    rng = np.random.default_rng(heads * 10 + c)
    n, fin = 1200, 30
    if loops == "loopless":
        ei, e = loopless(n, 8000, 4)
    else:
        ei, e = rand_graph(n, 8000, 5, hub_deg=700, loops=4)
    x = rng.standard_normal((n, fin)).astype(np.float32)
    w = weights(rng, fin, heads * c)
    a_s = rng.standard_normal((heads, c)).astype(np.float32) * 0.3
    a_d = rng.standard_normal((heads, c)).astype(np.float32) * 0.3
    od = heads * c if concat else c
    b = rng.standard_normal(od).astype(np.float32)
    layer = bg.GATConv(inChannels=fin, outChannels=c, heads=heads, concat=concat)
    layer.loadStateDict({"weight": w, "att_src": a_s, "att_dst": a_d, "bias": b})
    g = bg.GraphData(x=x, numNodes=n, numFeatures=fin, edgeIndex=ei, numEdges=e)
    got = layer.forward(g).x.cpu().numpy()
    want = orc.gat_forward(x, n, fin, ei, e, w, a_s, a_d, b, heads, c, 0.2, concat,
                           True).reshape(n, od)
    assert_close(got, want, f"gat h={heads} c={c} concat={concat} {loops}")


def test_gat_softmax_overflow_regime(bg):
    """The reference shifts scores by a constant 10, not the max: once a score
    exceeds ~98.7 exp overflows to inf and the weights become NaN.  The
    backend keeps that behaviour (it is the reference's output)."""
    n, fin, heads, c = 6, 2, 1, 2
    ei = np.array([0, 1, 2, 3, 4, 5, 1, 2, 3, 4, 5, 0], np.uint32)
    x = np.full((n, fin), 30.0, np.float32)
    w = np.eye(fin, heads * c, dtype=np.float32)
    a = np.full((heads, c), 1.0, np.float32)
    layer = bg.GATConv(inChannels=fin, outChannels=c, heads=heads, bias=False)
    layer.loadStateDict({"weight": w, "att_src": a, "att_dst": a})
    g = bg.GraphData(x=x, numNodes=n, numFeatures=fin, edgeIndex=ei, numEdges=6)
    got = layer.forward(g).x.cpu().numpy()
    want = orc.gat_forward(x, n, fin, ei, 6, w, a, a, None, heads, c, 0.2, True,
                           True).reshape(n, heads * c)
    assert np.isnan(want).all() and np.isnan(got).all()


@pytest.mark.parametrize("aggr", ["mean", "max", "sum", "pool"])
@pytest.mark.parametrize("root", [True, False])
@pytest.mark.parametrize("fout", [47, 130])
def test_sage(bg, mode, aggr, root, fout):
    rng = np.random.default_rng(21)
    n, fin = 2000, 24
    ei, e = rand_graph(n, 16000, 6, hub_deg=900, loops=3, dup=20)
    x = rng.standard_normal((n, fin)).astype(np.float32)
    wn = weights(rng, fin, fout)
    ws = weights(rng, fin, fout)
    b = rng.standard_normal(fout).astype(np.float32)
    sd = {"lin_neighbor": wn, "bias": b}
    if root:
        sd["lin_self"] = ws
    pw = pb = None
    if aggr == "pool":
        pw = weights(rng, fin, fin)
        pb = rng.standard_normal(fin).astype(np.float32)
        sd.update(pool_weight=pw, pool_bias=pb)
    layer = bg.SAGEConv(inChannels=fin, outChannels=fout, aggregator=aggr, rootWeight=root)
    layer.loadStateDict(sd)
    g = bg.GraphData(x=x, numNodes=n, numFeatures=fin, edgeIndex=ei, numEdges=e)
    got = layer.forward(g).x.cpu().numpy()
    want = orc.sage_forward(x, n, fin, ei, e, aggr, wn, ws if root else None, b, fout,
                            False, pw, pb).reshape(n, fout)
    check(got, want, mode, f"sage {aggr} root={root}")


def test_sage_normalize(bg, mode):
    rng = np.random.default_rng(22)
    n, fin, fout = 500, 16, 12
    ei, e = rand_graph(n, 3000, 7)
    x = rng.standard_normal((n, fin)).astype(np.float32)
    wn, ws = weights(rng, fin, fout), weights(rng, fin, fout)
    b = np.zeros(fout, np.float32)
    layer = bg.SAGEConv(inChannels=fin, outChannels=fout, normalize=True)
    layer.loadStateDict({"lin_neighbor": wn, "lin_self": ws, "bias": b})
    g = bg.GraphData(x=x, numNodes=n, numFeatures=fin, edgeIndex=ei, numEdges=e)
    got = layer.forward(g).x.cpu().numpy()
    want = orc.sage_forward(x, n, fin, ei, e, "mean", wn, ws, b, fout, True).reshape(n, fout)
    check(got, want, mode, "sage normalize")


@pytest.mark.parametrize("eps", [0.0, 0.37])
def test_gin(bg, mode, eps):
    rng = np.random.default_rng(31)
    w = synth.gin_batch(num_graphs=200)
    n, fin, hid, fout = w.num_nodes, 32, 64, 64
    w1, w2 = weights(rng, fin, hid), weights(rng, hid, fout)
    b1 = rng.standard_normal(hid).astype(np.float32)
    b2 = rng.standard_normal(fout).astype(np.float32)
    layer = bg.GINConv(inChannels=fin, outChannels=fout, hiddenChannels=hid, epsilon=eps)
    layer.loadStateDict({"epsilon": np.array([eps], np.float32), "mlp_weight1": w1,
                         "mlp_bias1": b1, "mlp_weight2": w2, "mlp_bias2": b2})
    g = bg.GraphData(x=w.x, numNodes=n, numFeatures=fin, edgeIndex=w.edge_index,
                     numEdges=w.num_edges, batch=w.extra["batch"])
    out = layer.forward(g)
    want = orc.gin_forward(w.x, n, fin, w.edge_index, w.num_edges, np.float32(eps), w1, b1, hid,
                           w2, b2, fout).reshape(n, fout)
    check(out.x.cpu().numpy(), want, mode, f"gin eps={eps}")
    pooled = bg.global_sum_pool(out, w.extra["num_graphs"]).cpu().numpy()
    wantp = orc.sum_pool(want, n, fout, w.extra["batch"], w.extra["num_graphs"])
    check(pooled, wantp.reshape(pooled.shape), mode, "sum pool")
