"""The library's host <-> device copies (bgnn_memcpy_h2d / bgnn_memcpy_d2h):
pageable arrays staged through its pinned chunks, page-locked arrays copied
directly, sizes that span several chunks and end mid-chunk, and two copies
from two host threads at once."""
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bg():
    import browsergnn_b200 as bg

    bg.init_browsergnn()
    return bg


@pytest.mark.parametrize("nbytes", [4, 1 << 20, (100 << 20) + 12])
def test_round_trip_pageable_and_pinned(bg, nbytes):
    import torch

    ctx = bg.get_context()
    rng = np.random.default_rng(nbytes)
    host = rng.integers(0, 2 ** 32, nbytes // 4, dtype=np.uint64).astype(np.uint32)
    dev = torch.empty(host.size, dtype=torch.int32, device="cuda")
    ctx.call("bgnn_memcpy_h2d", dev.data_ptr(), host.ctypes.data, host.nbytes)
    assert np.array_equal(dev.cpu().numpy().view(np.uint32), host)
    back = np.zeros_like(host)
    ctx.call("bgnn_memcpy_d2h", back.ctypes.data, dev.data_ptr(), back.nbytes)
    assert np.array_equal(back, host)
    pinned = torch.empty(host.size, dtype=torch.int32, pin_memory=True)
    ctx.call("bgnn_memcpy_d2h", pinned.data_ptr(), dev.data_ptr(), host.nbytes)
    assert np.array_equal(pinned.numpy().view(np.uint32), host)
    dev2 = torch.empty_like(dev)
    ctx.call("bgnn_memcpy_h2d", dev2.data_ptr(), pinned.data_ptr(), host.nbytes)
    assert torch.equal(dev, dev2)


def test_two_threads_at_once(bg):
    import torch

    ctx = bg.get_context()
    a = np.arange(30 << 20, dtype=np.float32)
    b = -np.arange(21 << 20, dtype=np.float32)
    da = torch.empty(a.size, device="cuda")
    db = torch.empty(b.size, device="cuda")
    rc = [None, None]

    def up(i, d, h):
        rc[i] = ctx.lib.bgnn_memcpy_h2d(ctx.h, d.data_ptr(), h.ctypes.data, h.nbytes)

    ts = [threading.Thread(target=up, args=(0, da, a)), threading.Thread(target=up, args=(1, db, b))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert rc == [0, 0]
    assert np.array_equal(da.cpu().numpy(), a) and np.array_equal(db.cpu().numpy(), b)


def test_graphdata_from_pageable_arrays(bg):
    """GraphData from host arrays: x uploads beside the CSR build and the
    layer's output reads back through the staging; the same numbers as the
    ordinary path."""
    from tests.helpers import rand_graph

    n, f = 5000, 40
    ei, e = rand_graph(n, 60000, 7, hub_deg=2000)
    x = np.random.default_rng(3).standard_normal((n, f)).astype(np.float32)
    layer = bg.SAGEConv(inChannels=f, outChannels=24)
    g = bg.GraphData(x=x, numNodes=n, numFeatures=f, edgeIndex=ei, numEdges=e)
    out = layer.forward(g).x_host()
    g2 = bg.GraphData(x=x, numNodes=n, numFeatures=f, edgeIndex=ei, numEdges=e)
    want = layer.forward(g2.withFeatures(g2.x_device())).x.cpu().numpy()
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


def test_large_edge_list_checked_on_the_device(bg):
    """Above the host-check size an out-of-range index is caught by the
    device CSR build, with the reference's message."""
    n = 1000
    e = (1 << 20) + 5
    ei = np.zeros(2 * e, np.uint32)
    ei[e + 17] = n + 3
    g = bg.GraphData(x=np.zeros((n, 1), np.float32), numNodes=n, numFeatures=1, edgeIndex=ei,
                     numEdges=e)
    with pytest.raises(ValueError, match="out of bounds"):
        g.device_graph()
