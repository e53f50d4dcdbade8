"""Backward kernels against the oracle's backward restatement.

The message-passing adjoint (an edge-ordered scatter of gradient messages
over the sources) and the reference's own matmul / bias / ReLU backward
(src/autograd/variable.ts) are bit-exact in both math modes where they are
additions; the k-ascending matmul backward is bit-exact in the exact mode and
within the parity bar in the fast mode."""
import numpy as np
import pytest

from oracle import oracle as orc
from tests.helpers import assert_bits_equal, assert_close, loopless, rand_graph

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bg():
    import browsergnn_b200 as bg

    bg.init_browsergnn()
    return bg


@pytest.fixture(params=[False, True], ids=["fast", "exact"])
def mode(request, bg):
    ctx = bg.get_context()
    ctx.set_math(request.param)
    yield request.param
    ctx.set_math(False)


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


@pytest.mark.parametrize("aggr", ["sum", "mean", "max"])
@pytest.mark.parametrize("f", [1, 7, 64, 130])
def test_aggregate_backward_bit_exact(bg, aggr, f):
    import torch

    from browsergnn_b200.backend import ptr

    n = 3000
    ei, e = rand_graph(n, 30000, seed=f + 3, hub_deg=2500, loops=5, dup=40)
    rng = np.random.default_rng(f)
    x = rng.standard_normal((n, f)).astype(np.float32)
    x[5, :] = -np.inf
    g = rng.standard_normal((n, f)).astype(np.float32)
    gd = bg.GraphData(x=x, numNodes=n, numFeatures=f, edgeIndex=ei, numEdges=e)
    dg = gd.device_graph()
    xd, gdv = _dev(torch, x), _dev(torch, g)
    out = torch.full((n, f), float("nan"), device="cuda")
    dg.ctx.call("bgnn_aggregate_backward", dg.h, {"sum": 0, "mean": 1, "max": 2}[aggr], ptr(xd),
                ptr(gdv), f, ptr(out))
    want = orc.aggregate_backward(ei, e, n, g, f, aggr, x=x).reshape(n, f)
    assert_bits_equal(out.cpu().numpy(), want, f"{aggr} backward f={f}")


@pytest.mark.parametrize("loops", ["appended", "present"])
@pytest.mark.parametrize("normalize", [True, False])
def test_gcn_backward_bit_exact(bg, loops, normalize):
    import torch

    from browsergnn_b200.backend import ptr

    n, f = 2500, 16
    if loops == "appended":
        ei, e = loopless(n, 20000, 3)
    else:
        ei, e = rand_graph(n, 20000, 4, hub_deg=1500, loops=6)
    g = np.random.default_rng(2).standard_normal((n, f)).astype(np.float32)
    gd = bg.GraphData(x=np.zeros((n, 1), np.float32), numNodes=n, numFeatures=1, edgeIndex=ei,
                      numEdges=e)
    dg = gd.device_graph()
    out = torch.empty((n, f), device="cuda")
    gdv = _dev(torch, g)
    dg.ctx.call("bgnn_gcn_propagate_backward", dg.h, ptr(gdv), f, 1, int(normalize), ptr(out))
    tail = loops == "appended"
    if normalize:
        want = orc.aggregate_backward(ei, e, n, g, f, "gcn", tail=tail).reshape(n, f)
    else:
        ei2, e2 = (orc.add_self_loops(ei, e, n) if tail else (ei, e))
        want = orc.aggregate_backward(ei2, e2, n, g, f, "sum").reshape(n, f)
    assert_bits_equal(out.cpu().numpy(), want, f"gcn backward {loops} normalize={normalize}")


@pytest.mark.parametrize("mkn", [(1, 1, 1), (300, 37, 16), (1500, 100, 47), (2, 256, 300)])
def test_matmul_and_bias_backward(bg, mode, mkn):
    import torch

    from browsergnn_b200.backend import ptr

    m, k, n = mkn
    rng = np.random.default_rng(m + k + n)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    g = rng.standard_normal((m, n)).astype(np.float32)
    ctx = bg.get_context()
    ad, bd, gdv = _dev(torch, a), _dev(torch, b), _dev(torch, g)
    ga = torch.empty((m, k), device="cuda")
    gb = torch.empty((k, n), device="cuda")
    ctx.call("bgnn_matmul_backward", ptr(ad), ptr(bd), ptr(gdv), m, k, n, ptr(ga), ptr(gb))
    wa, wb = orc.matmul_backward(a, b, g, m, k, n)
    bias = torch.empty(n, device="cuda")
    ctx.call("bgnn_bias_backward", ptr(gdv), m, n, ptr(bias))
    assert_bits_equal(bias.cpu().numpy(), orc.bias_backward(g, m, n), "bias backward")
    if mode:
        assert_bits_equal(ga.cpu().numpy(), wa.reshape(m, k), "grad a")
        assert_bits_equal(gb.cpu().numpy(), wb.reshape(k, n), "grad b")
    else:
        assert_close(ga.cpu().numpy(), wa.reshape(m, k), "grad a")
        assert_close(gb.cpu().numpy(), wb.reshape(k, n), "grad b")


@pytest.mark.parametrize("aggr", ["mean", "sum", "max"])
def test_sage_layer_backward(bg, mode, aggr):
    """SAGEConv.backward against the oracle's composition of the same
    adjoints (ReLU mask, bias reduction, matmul backward, message scatter)."""
    rng = np.random.default_rng(31)
    n, fin, fout = 2000, 24, 40
    ei, e = rand_graph(n, 16000, 6, hub_deg=900, loops=3, dup=20)
    x = rng.standard_normal((n, fin)).astype(np.float32)
    wn = (0.2 * rng.standard_normal((fin, fout))).astype(np.float32)
    ws = (0.2 * rng.standard_normal((fin, fout))).astype(np.float32)
    b = rng.standard_normal(fout).astype(np.float32)
    gout = rng.standard_normal((n, fout)).astype(np.float32)
    layer = bg.SAGEConv(inChannels=fin, outChannels=fout, aggregator=aggr)
    layer.loadStateDict({"lin_neighbor": wn, "lin_self": ws, "bias": b})
    gd = bg.GraphData(x=x, numNodes=n, numFeatures=fin, edgeIndex=ei, numEdges=e)
    import torch

    got = layer.backward(gd, _dev(torch, gout), _act="relu")
    # the oracle's composition
    out = orc.relu(orc.sage_forward(x, n, fin, ei, e, aggr, wn, ws, b, fout)).reshape(n, fout)
    g = np.where(out > 0, gout, 0).astype(np.float32)
    rp, so, _ = orc.dst_csr(ei, e, n)
    agg = orc.csr_aggregate(rp, so, n, x, fin, aggr, threads=1).reshape(n, fin)
    gagg, gwn = orc.matmul_backward(agg, wn, g, n, fin, fout)
    gxs, gws = orc.matmul_backward(x, ws, g, n, fin, fout)
    gmsg = orc.aggregate_backward(ei, e, n, gagg, fin, aggr, x=x)
    gx = orc.add(gxs, gmsg)
    check = assert_bits_equal if mode else assert_close
    check(got["bias"].cpu().numpy(), orc.bias_backward(g, n, fout), "bias")
    check(got["lin_neighbor"].cpu().numpy(), gwn.reshape(fin, fout), "lin_neighbor")
    check(got["lin_self"].cpu().numpy(), gws.reshape(fin, fout), "lin_self")
    check(got["x"].cpu().numpy(), gx.reshape(n, fin), "x")


def test_gcn_layer_backward(bg, mode):
    rng = np.random.default_rng(8)
    n, fin, fout = 1500, 30, 12
    ei, e = loopless(n, 10000, 5)
    x = rng.standard_normal((n, fin)).astype(np.float32)
    w = (0.2 * rng.standard_normal((fin, fout))).astype(np.float32)
    b = rng.standard_normal(fout).astype(np.float32)
    gout = rng.standard_normal((n, fout)).astype(np.float32)
    layer = bg.GCNConv(inChannels=fin, outChannels=fout)
    layer.loadStateDict({"weight": w, "bias": b})
    gd = bg.GraphData(x=x, numNodes=n, numFeatures=fin, edgeIndex=ei, numEdges=e)
    import torch

    got = layer.backward(gd, _dev(torch, gout), _act="relu")
    out = orc.relu(orc.gcn_forward(x, n, fin, ei, e, w, b, fout)).reshape(n, fout)
    g = np.where(out > 0, gout, 0).astype(np.float32)
    gh = orc.aggregate_backward(ei, e, n, g, fout, "gcn", tail=True).reshape(n, fout)
    gx, gw = orc.matmul_backward(x, w, gh, n, fin, fout)
    check = assert_bits_equal if mode else assert_close
    check(got["bias"].cpu().numpy(), orc.bias_backward(g, n, fout), "bias")
    check(got["weight"].cpu().numpy(), gw.reshape(fin, fout), "weight")
    check(got["x"].cpu().numpy(), gx.reshape(n, fin), "x")
