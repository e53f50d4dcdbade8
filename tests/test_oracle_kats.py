"""Pin the CPU oracle to the reference's own known-answer tests.

The vectors in tests/golden/reference_kats.json are transcribed from the
reference's vitest files (tests/wasm.test.ts, tests/graph.test.ts); each case
names its source lines.  These run on the CPU only.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as orc

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))


def close(got, want, case):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, case["src"]
    if case.get("exact"):
        assert np.array_equal(got, want), case["src"]
    else:
        # vitest toBeCloseTo(x, d): |got - want| < 10^-d / 2
        assert np.all(np.abs(got - want) < 10.0 ** (-case["tol_digits"]) / 2), case["src"]


@pytest.mark.parametrize("case", GOLD["matmul"], ids=lambda c: c["src"])
def test_matmul(case):
    close(orc.matmul(case["a"], case["b"], case["m"], case["k"], case["n"]), case["expect"], case)


@pytest.mark.parametrize("op", ["scatter_add", "scatter_mean", "scatter_max"])
def test_scatter(op):
    for case in GOLD[op]:
        got = getattr(orc, op)(case["x"], case["index"], case["num_nodes"], case["num_features"])
        close(got, case["expect"], case)


def test_gather():
    for case in GOLD["gather"]:
        close(orc.gather(case["x"], case["index"], case["num_features"]), case["expect"], case)


def test_relu_add():
    for case in GOLD["relu"]:
        close(orc.relu(case["x"]), case["expect"], case)
    for case in GOLD["add"]:
        close(orc.add(case["a"], case["b"]), case["expect"], case)


def test_spmv_spmm():
    for case in GOLD["spmv"]:
        close(orc.spmv(case["row_ptr"], case["col"], case["val"], case["x"], case["num_rows"]),
              case["expect"], case)
    for case in GOLD["spmm"]:
        got = orc.spmm(case["row_ptr"], case["col"], case["val"], case["dense"], case["num_rows"],
                       case["num_features"])
        close(got, case["expect"], case)


def test_degrees():
    for case in GOLD["degrees"]:
        ei = case["edge_index"]
        assert list(orc.in_degree(ei, case["num_edges"], case["num_nodes"])) == case["in_degree"]
        assert list(orc.out_degree(ei, case["num_edges"], case["num_nodes"])) == case["out_degree"]


def test_validate():
    for case in GOLD["validate"]:
        bad = orc.validate_edges(case["edge_index"], case["num_edges"], case["num_nodes"])
        assert (bad < 0) == case["valid"], case["src"]


def test_self_loops():
    for case in GOLD["self_loops"]:
        ei, e, n = case["edge_index"], case["num_edges"], case["num_nodes"]
        assert orc.has_self_loops(ei, e) == case["has_self_loops"]
        if "after_add_num_edges" in case:
            new_ei, ne = orc.add_self_loops(ei, e, n)
            assert ne == case["after_add_num_edges"]
            assert orc.has_self_loops(new_ei, ne) == case["after_add_has_self_loops"]
            # original edges first, loops appended in node order (graph.ts:246-258)
            assert list(new_ei[:e]) == ei[:e] and list(new_ei[ne:ne + e]) == ei[e:]
            assert list(new_ei[e:ne]) == list(range(n)) == list(new_ei[ne + e:])


def test_gcn_norm_hand_case():
    # Unpinned by the reference's tests; checked by hand: path 0->1->2 plus
    # self-loop counts (deg = [1, 2, 2] with addSelfLoops=True).
    ei = [0, 1, 1, 2]
    w = orc.gcn_norm(ei, 2, 3, True)
    want = np.array([1 / np.sqrt(1) * 1 / np.sqrt(2), 1 / np.sqrt(2) * 1 / np.sqrt(2)])
    assert np.allclose(w, want.astype(np.float32), rtol=0, atol=1e-7)


def test_coo_to_csr_stable_sort():
    # fromCOO sorts by (row, col) and keeps ties (duplicate edges) in input order.
    rows = [2, 0, 2, 0, 1, 2]
    cols = [1, 3, 0, 3, 2, 1]
    vals = [10, 20, 30, 40, 50, 60]
    rp, ci, va = orc.coo_to_csr(rows, cols, vals, 4)
    assert list(rp) == [0, 2, 3, 6, 6]
    assert list(ci) == [3, 3, 2, 0, 1, 1]
    assert list(va) == [20, 40, 50, 30, 10, 60]


def test_spmm_rows_matches_sequential_spmm():
    # The row-parallel restatement used for the full-size SpMM parity check
    # gives the sequential restatement's bits, for all rows and for a subset.
    rng = np.random.default_rng(3)
    n, nnz, f = 300, 4000, 5
    rows = rng.integers(0, n, nnz).astype(np.uint32)
    cols = rng.integers(0, n, nnz).astype(np.uint32)
    vals = rng.uniform(0, 1, nnz).astype(np.float32)
    rp, ci, va = orc.coo_to_csr(rows, cols, vals, n)
    x = rng.standard_normal((n, f)).astype(np.float32)
    want = orc.spmm(rp, ci, va, x, n, f).reshape(n, f)
    full = orc.spmm_rows(rp, ci, va, x, f, threads=4).reshape(n, f)
    assert np.array_equal(full.view(np.uint32), want.view(np.uint32))
    pick = np.array([7, 0, 299, 150], np.uint32)
    sub = orc.spmm_rows(rp, ci, va, x, f, rows=pick, threads=2).reshape(-1, f)
    assert np.array_equal(sub.view(np.uint32), want[pick].view(np.uint32))


def test_backward_restatement_is_gather_then_edge_ordered_scatter():
    # The message-passing adjoint equals wasmGather of the gradient rows by
    # destination, a per-edge message, then wasmScatterAdd over the sources
    # (both pinned by the reference's KATs above).
    rng = np.random.default_rng(5)
    n, e, f = 40, 300, 3
    src = rng.integers(0, n, e).astype(np.uint32)
    dst = rng.integers(0, n, e).astype(np.uint32)
    ei = np.concatenate([src, dst])
    g = rng.standard_normal((n, f)).astype(np.float32)
    x = rng.standard_normal((n, f)).astype(np.float32)
    gathered = orc.gather(g, dst, f).reshape(e, f)
    want = orc.scatter_add(gathered, src, n, f)
    got = orc.aggregate_backward(ei, e, n, g, f, "sum")
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    cnt = np.bincount(dst, minlength=n).astype(np.float64)
    msgs = (gathered.astype(np.float64) * (1.0 / cnt[dst])[:, None]).astype(np.float32)
    want = orc.scatter_add(msgs, src, n, f)
    got = orc.aggregate_backward(ei, e, n, g, f, "mean")
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    w = orc.gcn_norm(ei, e, n, False).astype(np.float64)
    msgs = (gathered.astype(np.float64) * w[:, None]).astype(np.float32)
    want = orc.scatter_add(msgs, src, n, f)
    got = orc.aggregate_backward(ei, e, n, g, f, "gcn")
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # max: each (dst, feature) routes its gradient to the edge that last
    # raised the running maximum (x > acc in COO order)
    arg = -np.ones((n, f), np.int64)
    acc = np.full((n, f), -np.inf, np.float32)
    for q in range(e):
        up = x[src[q]] > acc[dst[q]]
        acc[dst[q]][up] = x[src[q]][up]
        arg[dst[q]][up] = q
    msgs = np.where(arg[dst] == np.arange(e)[:, None], gathered, 0.0).astype(np.float32)
    want = orc.scatter_add(msgs, src, n, f)
    got = orc.aggregate_backward(ei, e, n, g, f, "max", x=x)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_matmul_backward_restatement():
    # variable.ts:213-235: grad @ B^T and A^T @ grad through Tensor.transpose
    rng = np.random.default_rng(6)
    m, k, n = 7, 5, 4
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    g = rng.standard_normal((m, n)).astype(np.float32)
    ga, gb = orc.matmul_backward(a, b, g, m, k, n)
    assert np.array_equal(ga, orc.matmul(g, np.ascontiguousarray(b.T), m, n, k))
    assert np.array_equal(gb, orc.matmul(np.ascontiguousarray(a.T), g, k, m, n))
    bias = orc.bias_backward(g, m, n)
    want = np.zeros(n, np.float32)
    for i in range(m):
        want = (want.astype(np.float64) + g[i]).astype(np.float32)
    assert np.array_equal(bias, want)
