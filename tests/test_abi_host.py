"""CPU-only checks: the C-ABI library loads and exports every declared symbol,
the host-side graph logic follows the reference, and the generators are
deterministic.  No kernel is launched here."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = []
    inc = os.path.join(ROOT, "include")
    for fn in sorted(os.listdir(inc)):
        if fn.endswith(".h"):
            txt = open(os.path.join(inc, fn)).read()
            names += re.findall(r"^BGNN_API\s+[\w\s\*]+?\b(bgnn_\w+)\s*\(", txt, re.M)
    return names


@pytest.fixture(scope="module")
def lib():
    from browsergnn_b200 import _lib
    from browsergnn_b200.build import LIB, build

    if not os.path.exists(LIB):
        build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = declared_symbols()
    assert len(names) >= 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    from browsergnn_b200 import _lib

    # and the ctypes table covers the whole header
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)
    assert lib.bgnn_abi_version() == 1


def test_null_context_is_rejected_without_a_gpu(lib):
    assert lib.bgnn_ctx_destroy(None) == 0
    assert lib.bgnn_ctx_set_math(None, 0) == 1  # BGNN_ERR_INVALID_ARG
    out = ctypes.c_void_p()
    rc = lib.bgnn_ctx_create(-1, ctypes.byref(out))
    assert rc != 0 and not out.value


def test_graphdata_validation_messages():
    from browsergnn_b200 import GraphData

    # graph.test.ts:25-47
    with pytest.raises(ValueError, match="doesn't match numNodes"):
        GraphData(x=[1, 2, 3], numNodes=2, numFeatures=3, edgeIndex=[0, 1], numEdges=1)
    with pytest.raises(ValueError, match="Edge index 5 out of bounds for 2 nodes"):
        GraphData(x=[1, 2], numNodes=2, numFeatures=1, edgeIndex=[0, 5, 1, 0], numEdges=2)
    with pytest.raises(ValueError, match="Edge index length"):
        GraphData(x=[1, 2], numNodes=2, numFeatures=1, edgeIndex=[0, 1, 1], numEdges=2)
    g = GraphData(x=[1, 2, 3, 4], numNodes=4, numFeatures=1, edgeIndex=[0, 1, 2, 1, 2, 3],
                  numEdges=3)
    assert list(g.sourceNodes) == [0, 1, 2] and list(g.targetNodes) == [1, 2, 3]
    assert g.getEdge(1) == [1, 2]


def test_add_remove_self_loops_host():
    from browsergnn_b200 import GraphData

    g = GraphData(x=[1, 2, 3], numNodes=3, numFeatures=1, edgeIndex=[0, 1, 1, 2], numEdges=2)
    g2 = g.addSelfLoops()
    assert g2.numEdges == 5
    assert list(g2.edgeIndex) == [0, 1, 0, 1, 2, 1, 2, 0, 1, 2]
    g3 = GraphData(x=[1, 2], numNodes=2, numFeatures=1, edgeIndex=[0, 0, 1, 0, 1, 1], numEdges=3)
    assert g3.removeSelfLoops().numEdges == 1


def test_batch_graphs_kat():
    from browsergnn_b200 import GraphData, batchGraphs

    # graph.test.ts:238-263
    g1 = GraphData(x=[1, 2, 3, 4], numNodes=2, numFeatures=2, edgeIndex=[0, 1, 1, 0], numEdges=2)
    g2 = GraphData(x=[5, 6, 7, 8, 9, 10], numNodes=3, numFeatures=2, edgeIndex=[0, 1, 1, 2],
                   numEdges=2)
    b = batchGraphs([g1, g2])
    assert b.numNodes == 5 and b.numEdges == 4
    assert b.batch[0] == 0 and b.batch[2] == 1
    assert list(b.edgeIndex) == [0, 1, 2, 3, 1, 0, 3, 4]
    with pytest.raises(ValueError):
        batchGraphs([])


def test_rmat_generator_deterministic_and_bounded():
    from browsergnn_b200 import synth

    a = synth.rmat_edges(12, 3000, 20000, 99)
    b = synth.rmat_edges(12, 3000, 20000, 99)
    assert np.array_equal(a, b)
    assert a.size == 40000 and a.max() < 3000
    # R-MAT skew: the most popular destination is far above the mean
    deg = np.bincount(a[20000:], minlength=3000)
    assert deg.max() > 20 * deg.mean()
    p = synth.permute_ids(np.arange(3000), 3000, 5)
    assert np.array_equal(np.sort(p), np.arange(3000))


def test_workload_shapes():
    from browsergnn_b200 import synth

    w = synth.gcn_cora_like()
    assert w.num_nodes == 2708 and w.num_edges == 10556 and w.x.shape == (2708, 1433)
    ei = w.edge_index
    assert not np.any(ei[:w.num_edges] == ei[w.num_edges:])  # BA has no self-loops
    pairs = set(zip(ei[:5278].tolist(), ei[5278:10556].tolist()))
    assert len(pairs) == 5278
    gi = synth.gin_batch(num_graphs=32)
    assert gi.extra["batch"].size == gi.num_nodes
