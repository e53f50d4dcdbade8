"""The allocation-free GAT entry point (bgnn_gat_noalloc).

Some callers cannot let the library allocate device memory while they run: a
server that reserves its whole budget at start-up, or an embedding host (a
Node-API addon inside a JavaScript runtime, say) that owns the device memory.
bgnn_gat_noalloc serves them with a fixed device array as its scratch.  Its
output is checked against the allocating entry point (bgnn_gat) and against
the oracle's GATConv forward, on two calls in a row.  This file is collected
last so that a failure here leaves every other test run.
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc
from tests.helpers import assert_close, loopless, rand_graph

pytestmark = pytest.mark.gpu


def _call(ctx, name, *args):
    return getattr(ctx.lib, name)(ctx.h, *args)


def _graph(kind):
    """(edge_index, num_edges, num_nodes): 'appended' has no self-loop, so
    the layer appends one per node (gat.ts:116-118); 'has_loops' already has
    some, so nothing is appended; 'no_edges' has only the appended loops."""
    if kind == "appended":
        n = 3000
        ei, e = loopless(n, 20000, 9)
        # a hub row long enough for the heavy-row kernel
        hub = np.arange(1, 801, dtype=np.uint32)
        ei = np.concatenate([ei[:e], hub, ei[e:], np.zeros(800, np.uint32)])
        return ei, e + 800, n
    if kind == "has_loops":
        n = 3000
        ei, e = rand_graph(n, 20000, 9, hub_deg=600, loops=5)
        return ei, e, n
    return np.zeros(0, np.uint32), 0, 50


@pytest.mark.parametrize("concat", [1, 0])
@pytest.mark.parametrize("kind", ["appended", "has_loops", "no_edges"])
def test_gat_noalloc_matches_allocating_entry_point_and_oracle(concat, kind):
    import torch

    import browsergnn_b200 as bg
    from browsergnn_b200.backend import ptr

    bg.init_browsergnn()
    ctx = bg.get_context()
    rng = np.random.default_rng(5 + concat)
    heads, c = 8, 8
    ei, e, n = _graph(kind)
    hc = heads * c
    od = hc if concat else c
    g = bg.GraphData(x=np.zeros(n, np.float32), numNodes=n, numFeatures=1, edgeIndex=ei,
                     numEdges=e)
    dg = g.device_graph()
    h_np = rng.standard_normal((n, hc)).astype(np.float32)
    as_np = (0.3 * rng.standard_normal((heads, c))).astype(np.float32)
    ad_np = (0.3 * rng.standard_normal((heads, c))).astype(np.float32)
    b_np = rng.standard_normal(od).astype(np.float32)
    h = torch.from_numpy(h_np).cuda()
    a_s = torch.from_numpy(as_np).cuda()
    a_d = torch.from_numpy(ad_np).cuda()
    bias = torch.from_numpy(b_np).cuda()
    # ELU after the layer (act 3, alpha 1), as the GAT workload's first layer
    args = (dg.h, ptr(h), heads, c, ptr(a_s), ptr(a_d), 0.2, concat, 1, ptr(bias), 3, 1.0)

    ctx.bind()
    # the allocation-free calls come first, on a graph that has never run a
    # GAT, so they cannot lean on anything the allocating entry point builds
    gots = []
    for _ in range(2):  # two calls in a row share (and reuse) the fixed scratch
        got = torch.full((n, od), float("nan"), device="cuda")
        rc = _call(ctx, "bgnn_gat_noalloc", *args, ptr(got))
        assert rc == 0, ctx.lib.bgnn_last_error(ctx.h)
        assert ctx.lib.bgnn_ctx_synchronize(ctx.h) == 0
        gots.append(got.cpu().numpy())
    want_dev = torch.empty((n, od), device="cuda")
    assert _call(ctx, "bgnn_gat", *args, ptr(want_dev)) == 0
    torch.cuda.synchronize()
    # the oracle's GATConv forward with an identity weight: X * I reproduces
    # h exactly (each output adds one product x*1 and otherwise x*0 = +-0)
    want = orc.elu(orc.gat_forward(h_np, n, hc, ei, e, np.eye(hc, dtype=np.float32), as_np,
                                   ad_np, b_np, heads, c, 0.2, bool(concat), True)).reshape(n, od)
    for got in gots:
        assert_close(got, want_dev.cpu().numpy(), f"gat_noalloc vs bgnn_gat ({kind})")
        assert_close(got, want, f"gat_noalloc vs oracle ({kind})")


def test_gat_noalloc_zero_nodes():
    """A graph with no nodes returns at once and writes nothing."""
    import browsergnn_b200 as bg

    bg.init_browsergnn()
    ctx = bg.get_context()
    ctx.bind()
    gh = ctypes.c_void_p()
    assert ctx.lib.bgnn_graph_create(ctx.h, None, 0, 0, 0, 0, ctypes.byref(gh)) == 0
    try:
        rc = _call(ctx, "bgnn_gat_noalloc", gh, ctypes.c_void_p(16), 2, 4, ctypes.c_void_p(16),
                   ctypes.c_void_p(16), 0.2, 1, 1, None, 0, 0.0, ctypes.c_void_p(16))
        assert rc == 0, ctx.lib.bgnn_last_error(ctx.h)
        assert ctx.lib.bgnn_ctx_synchronize(ctx.h) == 0
    finally:
        ctx.lib.bgnn_graph_destroy(gh)


def test_gat_noalloc_rejects_graphs_beyond_its_scratch():
    import torch

    import browsergnn_b200 as bg
    from browsergnn_b200.backend import ptr

    bg.init_browsergnn()
    ctx = bg.get_context()
    n, heads, c = 1000, 32, 1
    ei, e = rand_graph(n, 140000, 3)  # (140000 + 1000 loops) * 32 > 4,194,304 floats
    g = bg.GraphData(x=np.zeros(n, np.float32), numNodes=n, numFeatures=1, edgeIndex=ei,
                     numEdges=e)
    dg = g.device_graph()
    h = torch.zeros((n, heads * c), device="cuda")
    att = torch.zeros((heads, c), device="cuda")
    out = torch.zeros((n, heads * c), device="cuda")
    ctx.bind()
    rc = _call(ctx, "bgnn_gat_noalloc", dg.h, ptr(h), heads, c, ptr(att), ptr(att), 0.2, 1, 1,
               None, 0, 0.0, ptr(out))
    assert rc == 1  # BGNN_ERR_INVALID_ARG
    assert b"limit" in ctx.lib.bgnn_last_error(ctx.h)
