"""The allocation-free GAT entry point (bgnn_gat_noalloc) against bgnn_gat.

Some callers cannot let the library allocate device memory while they run: a
server that reserves its whole budget at start-up, or an embedding host (a
Node-API addon inside a JavaScript runtime, say) that owns the device memory.
bgnn_gat_noalloc serves them with a fixed device array as its scratch.  This
file is collected last so that a failure here leaves every other test run.
"""
import ctypes

import numpy as np
import pytest

from tests.helpers import assert_close, rand_graph

pytestmark = pytest.mark.gpu


def _call(ctx, name, *args):
    return getattr(ctx.lib, name)(ctx.h, *args)


def test_gat_noalloc_matches_allocating_entry_point():
    import torch

    import browsergnn_b200 as bg
    from browsergnn_b200.backend import ptr

    bg.init_browsergnn()
    ctx = bg.get_context()
    rng = np.random.default_rng(5)
    n, heads, c = 3000, 8, 8
    ei, e = rand_graph(n, 20000, 9, hub_deg=600)
    g = bg.GraphData(x=np.zeros(n, np.float32), numNodes=n, numFeatures=1, edgeIndex=ei,
                     numEdges=e)
    dg = g.device_graph()
    h = torch.from_numpy(rng.standard_normal((n, heads * c)).astype(np.float32)).cuda()
    a_s = torch.from_numpy((0.3 * rng.standard_normal((heads, c))).astype(np.float32)).cuda()
    a_d = torch.from_numpy((0.3 * rng.standard_normal((heads, c))).astype(np.float32)).cuda()
    bias = torch.from_numpy(rng.standard_normal(heads * c).astype(np.float32)).cuda()
    args = (dg.h, ptr(h), heads, c, ptr(a_s), ptr(a_d), 0.2, 1, 1, ptr(bias), 3, 1.0)

    ctx.bind()
    # the allocation-free calls come first, on a graph that has never run a
    # GAT, so they cannot lean on anything the allocating entry point builds
    gots = []
    for _ in range(2):  # two calls in a row share (and reuse) the fixed scratch
        got = torch.full((n, heads * c), float("nan"), device="cuda")
        rc = _call(ctx, "bgnn_gat_noalloc", *args, ptr(got))
        assert rc == 0, ctx.lib.bgnn_last_error(ctx.h)
        assert ctx.lib.bgnn_ctx_synchronize(ctx.h) == 0
        gots.append(got.cpu().numpy())
    want = torch.empty((n, heads * c), device="cuda")
    assert _call(ctx, "bgnn_gat", *args, ptr(want)) == 0
    torch.cuda.synchronize()
    for got in gots:
        assert_close(got, want.cpu().numpy(), "gat_noalloc")


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
