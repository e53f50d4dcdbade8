"""Parity of the CUDA kernels (through the C ABI) with the CPU oracle.

Integer work (CSR, degrees, indices) must match bit for bit; the aggregations
must match bit for bit as well because they follow the reference's rounding
sequence.  Everything runs on cuda:0.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as orc
from tests.helpers import assert_bits_equal, assert_close, rand_graph

pytestmark = pytest.mark.gpu

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))


@pytest.fixture(scope="module")
def bg():
    import browsergnn_b200 as bg

    bg.init_browsergnn()
    return bg


@pytest.fixture(scope="module")
def torch():
    import torch

    return torch


def dev(torch, a, dtype=None):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


# ---- the reference's KATs through the facade (host buffers) -------------------
def test_facade_kats(bg):
    cm = bg.CudaComputeManager()
    for c in GOLD["matmul"]:
        np.testing.assert_allclose(cm.matmul(c["a"], c["b"], c["m"], c["k"], c["n"]), c["expect"],
                                   atol=5e-6)
    for op, fn in (("scatter_add", cm.scatterAdd), ("scatter_mean", cm.scatterMean),
                   ("scatter_max", cm.scatterMax)):
        for c in GOLD[op]:
            got = fn(c["x"], c["index"], c["num_nodes"], c["num_features"])
            np.testing.assert_allclose(got, c["expect"], atol=5e-6)
    for c in GOLD["gather"]:
        np.testing.assert_allclose(cm.gather(c["x"], c["index"], c["num_features"]), c["expect"])
    for c in GOLD["relu"]:
        assert list(cm.relu(c["x"])) == c["expect"]
    for c in GOLD["add"]:
        assert list(cm.add(c["a"], c["b"])) == c["expect"]
    for c in GOLD["spmv"]:
        np.testing.assert_allclose(cm.spmv(c["row_ptr"], c["col"], c["val"], c["x"], c["num_rows"]),
                                   c["expect"], atol=5e-6)
    for c in GOLD["spmm"]:
        got = cm.spmm(c["row_ptr"], c["col"], c["val"], c["dense"], c["num_rows"], c["num_cols"],
                      c["num_features"])
        np.testing.assert_allclose(got, c["expect"], atol=5e-6)


def test_graph_kats(bg):
    for c in GOLD["degrees"]:
        g = bg.GraphData(x=np.zeros(c["num_nodes"]), numNodes=c["num_nodes"], numFeatures=1,
                         edgeIndex=c["edge_index"], numEdges=c["num_edges"])
        assert list(g.getInDegrees()) == c["in_degree"]
        assert list(g.getOutDegrees()) == c["out_degree"]
    for c in GOLD["self_loops"]:
        g = bg.GraphData(x=np.zeros(c["num_nodes"]), numNodes=c["num_nodes"], numFeatures=1,
                         edgeIndex=c["edge_index"], numEdges=c["num_edges"])
        assert g.hasSelfLoops() == c["has_self_loops"]
        if "after_add_num_edges" in c:
            g2 = g.addSelfLoops()
            assert g2.numEdges == c["after_add_num_edges"]
            assert g2.hasSelfLoops() == c["after_add_has_self_loops"]


# ---- CSR build, degrees, norms --------------------------------------------------
@pytest.mark.parametrize("n,e,hub", [(1, 0, 0), (5, 0, 0), (50, 400, 0), (3000, 40000, 5000),
                                     (70000, 300000, 20000)])
def test_graph_csr_bit_exact(bg, n, e, hub):
    ei, e2 = rand_graph(n, e, seed=n + e, hub_deg=hub, loops=5 if n > 5 else 0, dup=10 if e else 0)
    g = bg.GraphData(x=np.zeros(n), numNodes=n, numFeatures=1, edgeIndex=ei, numEdges=e2)
    rp, so, ed = g.device_graph().csr()
    orp, oso, oed = orc.dst_csr(ei, e2, n)
    assert np.array_equal(rp.cpu().numpy().view(np.uint32), orp)
    assert np.array_equal(so.cpu().numpy().view(np.uint32), oso)
    assert np.array_equal(ed.cpu().numpy().view(np.uint32), oed)
    assert np.array_equal(g.getInDegrees(), orc.in_degree(ei, e2, n))
    assert np.array_equal(g.getOutDegrees(), orc.out_degree(ei, e2, n))
    assert g.hasSelfLoops() == orc.has_self_loops(ei, e2)


def test_out_of_range_edge_raises(bg):
    with pytest.raises(ValueError, match="out of bounds"):
        bg.DeviceGraph(np.array([0, 5, 1, 0], np.uint32), 2, 2, 2)


@pytest.mark.parametrize("nnz,m,ncol", [(0, 3, 3), (17, 5, 4), (100000, 3000, 5000),
                                        (400000, 70000, 300), (3000000, 1100000, 16000000)])
def test_coo_to_csr_bit_exact(bg, torch, nnz, m, ncol):
    rng = np.random.default_rng(nnz + m)
    rows = rng.integers(0, m, nnz).astype(np.uint32)
    cols = rng.integers(0, ncol, nnz).astype(np.uint32)
    vals = rng.standard_normal(nnz).astype(np.float32)
    coo = bg.SparseCOO(rows, cols, vals, (m, ncol))
    csr = bg.SparseCSR.fromCOO(coo)
    orp, oci, ova = orc.coo_to_csr(rows, cols, vals, m)
    assert np.array_equal(csr.rowPtr.cpu().numpy().view(np.uint32), orp)
    assert np.array_equal(csr.colIndices.cpu().numpy().view(np.uint32), oci)
    assert_bits_equal(csr.values.cpu().numpy(), ova, "values")
    # and through the host facade
    rp, ci, va = bg.CudaComputeManager().coo_to_csr(rows, cols, vals, m, ncol)
    assert np.array_equal(rp, orp) and np.array_equal(ci, oci)


def test_sm_budget_same_bits(bg, torch):
    """An aggregation held to a few SMs (bgnn_ctx_set_sm_budget) gives the
    same bits as one on the whole GPU: only the grid shrinks."""
    from browsergnn_b200.backend import ptr

    n, f = 20000, 64
    ei, e = rand_graph(n, 300000, seed=4, hub_deg=60000, loops=3, dup=30)
    g = bg.GraphData(x=np.zeros((n, 1), np.float32), numNodes=n, numFeatures=1, edgeIndex=ei,
                     numEdges=e)
    dg = g.device_graph()
    x = torch.randn((n, f), device="cuda", generator=torch.Generator("cuda").manual_seed(2))
    full = torch.empty((n, f), device="cuda")
    few = torch.empty((n, f), device="cuda")
    dg.ctx.call("bgnn_aggregate", dg.h, 1, ptr(x), f, ptr(full))
    try:
        dg.ctx.call("bgnn_ctx_set_sm_budget", 12)
        dg.ctx.call("bgnn_aggregate", dg.h, 1, ptr(x), f, ptr(few))
    finally:
        dg.ctx.call("bgnn_ctx_set_sm_budget", 0)
    assert torch.equal(full.view(torch.int32), few.view(torch.int32))


def test_coo_to_csr_without_values(bg, torch):
    """bgnn_coo_to_csr_dev with no input values (all ones, fromEdgeIndex) and
    with no value output: the same rows and columns as the oracle."""
    from browsergnn_b200.backend import ptr

    rng = np.random.default_rng(11)
    nnz, m, ncol = 250000, 4000, 70000
    rows = rng.integers(0, m, nnz).astype(np.uint32)
    cols = rng.integers(0, ncol, nnz).astype(np.uint32)
    orp, oci, _ = orc.coo_to_csr(rows, cols, np.ones(nnz, np.float32), m)
    ctx = bg.get_context()
    r = torch.from_numpy(rows.view(np.int32)).cuda()
    c = torch.from_numpy(cols.view(np.int32)).cuda()
    for with_val_out in (True, False):
        rp = torch.empty(m + 1, dtype=torch.int32, device="cuda")
        ci = torch.empty(nnz, dtype=torch.int32, device="cuda")
        va = torch.full((nnz,), -1.0, device="cuda") if with_val_out else None
        ctx.call("bgnn_coo_to_csr_dev", ptr(r), ptr(c), None, nnz, m, ncol, ptr(rp), ptr(ci),
                 ptr(va))
        assert np.array_equal(rp.cpu().numpy().view(np.uint32), orp)
        assert np.array_equal(ci.cpu().numpy().view(np.uint32), oci)
        if with_val_out:
            assert bool((va == 1.0).all())


@pytest.mark.parametrize("loops", [False, True])
def test_gcn_norm_bit_exact(bg, loops):
    ei, e = rand_graph(2000, 30000, 3, hub_deg=3000)
    got = bg.compute_gcn_norm(ei, e, 2000, loops).cpu().numpy()
    assert_bits_equal(got, orc.gcn_norm(ei, e, 2000, loops), "gcn norm")


# ---- aggregation ----------------------------------------------------------------
FEATS = [1, 3, 4, 7, 16, 47, 64, 100, 256, 300, 1100]


@pytest.mark.parametrize("aggr", ["sum", "mean", "max"])
@pytest.mark.parametrize("f", FEATS)
def test_aggregate_bit_exact(bg, torch, aggr, f):
    n = 2500
    ei, e = rand_graph(n, 20000, seed=f, hub_deg=1500, loops=7, dup=11)
    rng = np.random.default_rng(f)
    x = rng.standard_normal((n, f)).astype(np.float32)
    x[3, :] = -np.inf if f > 1 else x[3, :]
    g = bg.GraphData(x=x, numNodes=n, numFeatures=f, edgeIndex=ei, numEdges=e)
    dg = g.device_graph()
    xd = g.x_device()
    out = torch.empty((n, f), dtype=torch.float32, device="cuda")
    dg.ctx.call("bgnn_aggregate", dg.h, {"sum": 0, "mean": 1, "max": 2}[aggr], xd.data_ptr(), f,
                out.data_ptr())
    gathered = orc.gather(x, ei[:e], f)
    want = {"sum": orc.scatter_add, "mean": orc.scatter_mean,
            "max": orc.scatter_max}[aggr](gathered, ei[e:], n, f)
    assert_bits_equal(out.cpu().numpy(), want, f"{aggr} F={f}")


@pytest.mark.parametrize("case", ["no_edges", "one_hub", "all_heavy", "long_empty_runs"])
@pytest.mark.parametrize("f", [32, 100])
def test_aggregate_schedule_edge_cases(bg, torch, case, f):
    rng = np.random.default_rng(3)
    if case == "no_edges":
        n, src, dst = 700, np.zeros(0, np.int64), np.zeros(0, np.int64)
    elif case == "one_hub":
        n = 600
        src = rng.integers(0, n, 20000)
        dst = np.full(20000, 17)
    elif case == "all_heavy":
        n = 40
        src = rng.integers(0, n, 40 * 300)
        dst = np.repeat(np.arange(n), 300)[rng.permutation(40 * 300)]
    else:
        n = 5000  # a few edges, thousands of empty rows between them
        src = rng.integers(0, n, 50)
        dst = rng.integers(0, n, 50)
    ei = np.concatenate([src, dst]).astype(np.uint32)
    e = src.size
    x = rng.standard_normal((n, f)).astype(np.float32)
    g = bg.GraphData(x=x, numNodes=n, numFeatures=f, edgeIndex=ei, numEdges=e)
    dg = g.device_graph()
    for aggr, code in (("sum", 0), ("mean", 1), ("max", 2)):
        out = torch.empty((n, f), dtype=torch.float32, device="cuda")
        dg.ctx.call("bgnn_aggregate", dg.h, code, g.x_device().data_ptr(), f, out.data_ptr())
        gathered = orc.gather(x, ei[:e], f)
        want = {"sum": orc.scatter_add, "mean": orc.scatter_mean,
                "max": orc.scatter_max}[aggr](gathered, ei[e:], n, f)
        assert_bits_equal(out.cpu().numpy(), want, f"{case} {aggr} F={f}")


@pytest.mark.parametrize("aggr", ["sum", "mean", "max"])
def test_scatter_facade_bit_exact(bg, torch, aggr):
    rng = np.random.default_rng(7)
    m, n, f = 5000, 300, 20
    idx = rng.integers(0, n, m).astype(np.uint32)
    idx[:600] = 5  # a heavy destination
    src = rng.standard_normal((m, f)).astype(np.float32)
    fn = {"sum": bg.MessagePassing.scatterAdd, "mean": bg.MessagePassing.scatterMean,
          "max": bg.MessagePassing.scatterMax}[aggr]
    got = fn(dev(torch, src), idx, n).cpu().numpy()
    want = {"sum": orc.scatter_add, "mean": orc.scatter_mean, "max": orc.scatter_max}[aggr](
        src, idx, n, f)
    assert_bits_equal(got, want, aggr)


def test_gather_and_out_of_range(bg, torch):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((50, 6)).astype(np.float32)
    idx = rng.integers(0, 50, 300).astype(np.uint32)
    got = bg.MessagePassing.gather(dev(torch, x), idx).cpu().numpy()
    assert_bits_equal(got, orc.gather(x, idx, 6).reshape(300, 6))
    with pytest.raises(bg.BGNNError):
        bg.CudaComputeManager().gather(x, np.array([0, 50], np.uint32), 6)


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("f", [5, 32, 64, 128])
def test_spmm(bg, torch, exact, f):
    ctx = bg.get_context()
    ctx.set_math(exact)
    try:
        rng = np.random.default_rng(f)
        m, ncol, nnz = 3000, 2500, 40000
        rows = rng.integers(0, m, nnz).astype(np.uint32)
        rows[:2000] = 11  # heavy row
        cols = rng.integers(0, ncol, nnz).astype(np.uint32)
        vals = rng.random(nnz).astype(np.float32)
        csr = bg.SparseCSR.fromCOO(bg.SparseCOO(rows, cols, vals, (m, ncol)))
        x = rng.standard_normal((ncol, f)).astype(np.float32)
        got = csr.matmul(dev(torch, x)).cpu().numpy()
        orp, oci, ova = orc.coo_to_csr(rows, cols, vals, m)
        want = orc.spmm(orp, oci, ova, x, m, f).reshape(m, f)
        if exact:
            assert_bits_equal(got, want, "spmm exact")
        else:
            assert_close(got, want, "spmm fast")
        # SpMV
        xv = rng.standard_normal(ncol).astype(np.float32)
        gv = csr.matvec(dev(torch, xv)).cpu().numpy()
        assert_bits_equal(gv, orc.spmv(orp, oci, ova, xv, m), "spmv")
    finally:
        ctx.set_math(False)


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("mkn", [(1, 1, 1), (37, 13, 7), (300, 1433, 16), (513, 100, 256),
                                 (257, 256, 47), (64, 0, 5)])
def test_matmul(bg, torch, exact, mkn):
    m, k, n = mkn
    ctx = bg.get_context()
    ctx.set_math(exact)
    try:
        rng = np.random.default_rng(m * 7 + k)
        a = rng.standard_normal((m, k)).astype(np.float32)
        b = rng.standard_normal((k, n)).astype(np.float32)
        got = bg.GPUTensor.matmul(dev(torch, a), dev(torch, b)).cpu().numpy()
        want = orc.matmul(a, b, m, k, n).reshape(m, n)
        if exact:
            assert_bits_equal(got, want, "matmul exact")
        else:
            assert_close(got, want, "matmul fast")
    finally:
        ctx.set_math(False)


def test_activations(bg, torch):
    x = np.array([-2, -1, -0.0, 0, 1, 2, np.nan, -np.inf, np.inf, 1e-30, -1e-30], np.float32)
    xd = dev(torch, x)
    assert_bits_equal(bg.GPUTensor.relu(xd).cpu().numpy(), orc.relu(x), "relu")
    assert_close(bg.ELU(1.0)(xd).cpu().numpy(), orc.elu(x, 1.0), "elu", rtol=0, atol=0)
    assert_bits_equal(bg.LeakyReLU(0.1)(xd).cpu().numpy(), orc.leaky_relu(x, 0.1), "leaky")
    y = np.random.default_rng(0).standard_normal(1000).astype(np.float32)
    assert_bits_equal(bg.GPUTensor.add(dev(torch, y), dev(torch, x[:1].repeat(1000))).cpu().numpy(),
                      orc.add(y, x[:1].repeat(1000)), "add")
