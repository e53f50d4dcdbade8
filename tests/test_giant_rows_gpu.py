"""Hub rows long enough to get their own launch (the giant-slice kernel: the
row cut into feature slices, one CTA per slice alone on its SM), at slice
widths that divide the features and with a narrow last slice, and hub rows
that stay in the main launch as slices; every output bit for bit against the
oracle's edge-ordered aggregation."""
import numpy as np
import pytest

from oracle import oracle as orc
from tests.helpers import assert_bits_equal

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bg():
    import browsergnn_b200 as bg

    bg.init_browsergnn()
    return bg


def _hub_graph(n, e, hubs, seed):
    """Random edges plus hub rows (dst = 2, 5, ...) of the given degrees,
    shuffled together so each hub's edges are spread over the COO order."""
    rng = np.random.default_rng(seed)
    s = [rng.integers(0, n, e)]
    d = [rng.integers(0, n, e)]
    for i, deg in enumerate(hubs):
        s.append(rng.integers(0, n, deg))
        d.append(np.full(deg, 2 + 3 * i))
    s, d = np.concatenate(s), np.concatenate(d)
    perm = rng.permutation(s.size)
    return np.concatenate([s[perm], d[perm]]).astype(np.uint32), int(s.size)


@pytest.mark.parametrize("f", [4, 32, 36, 100, 128, 256])
@pytest.mark.parametrize("aggr", ["sum", "mean", "max"])
def test_giant_rows_bit_exact(bg, f, aggr):
    import torch

    from browsergnn_b200.backend import ptr

    n = 40000
    ei, e = _hub_graph(n, 200000, [150000, 40000, 9000], seed=f)
    rng = np.random.default_rng(f + 1)
    x = rng.standard_normal((n, f)).astype(np.float32)
    g = bg.GraphData(x=x, numNodes=n, numFeatures=f, edgeIndex=ei, numEdges=e)
    dg = g.device_graph()
    xd = torch.from_numpy(x).cuda()
    out = torch.full((n, f), float("nan"), device="cuda")
    code = {"sum": 0, "mean": 1, "max": 2}[aggr]
    dg.ctx.call("bgnn_aggregate", dg.h, code, ptr(xd), f, ptr(out))
    rp, so, _ = orc.dst_csr(ei, e, n)
    want = orc.csr_aggregate(rp, so, n, x, f, aggr).reshape(n, f)
    got = out.cpu().numpy()
    for hub in (2, 5, 8):
        assert_bits_equal(got[hub], want[hub], f"hub row {hub} F={f} {aggr}")
    assert_bits_equal(got, want, f"all rows F={f} {aggr}")


@pytest.mark.parametrize("f", [32, 100])
def test_giant_rows_spmm_bit_exact(bg, f):
    """The same hubs through the CSR SpMM (per-entry values), in the exact
    mode (each step the reference's f64 product and f32 store)."""
    import torch

    n = 40000
    ei, e = _hub_graph(n, 200000, [150000, 40000], seed=3 + f)
    rows, cols = ei[e:], ei[:e]
    vals = np.random.default_rng(f).uniform(0, 1, e).astype(np.float32)
    ctx = bg.get_context()
    ctx.set_math(True)
    try:
        csr = bg.SparseCSR.fromCOO(bg.SparseCOO(rows, cols, vals, (n, n)))
        x = np.random.default_rng(f + 7).standard_normal((n, f)).astype(np.float32)
        out = csr.matmul(torch.from_numpy(x).cuda()).cpu().numpy()
    finally:
        ctx.set_math(False)
    rp = csr.rowPtr.cpu().numpy().view(np.uint32)
    ci = csr.colIndices.cpu().numpy().view(np.uint32)
    cv = csr.values.cpu().numpy()
    want = orc.spmm_rows(rp, ci, cv, x, f).reshape(n, f)
    assert_bits_equal(out, want, f"SpMM F={f}")


def test_giant_row_reads_each_source_once(bg):
    """A 150,000-edge hub row summed over indicator features (feature c of
    node i is 1 when i mod 32 == c): every column must count exactly the hub's
    sources congruent to c.  A source-id slot overwritten before its stage was
    copied shows up here as a row counted in the wrong column."""
    import torch

    from browsergnn_b200.backend import ptr

    n, f, deg = 40000, 32, 150000
    rng = np.random.default_rng(11)
    src = rng.integers(0, n, deg).astype(np.uint32)
    bs = rng.integers(0, n, 200000).astype(np.uint32)
    bd = rng.integers(1, n, 200000).astype(np.uint32)
    ei = np.concatenate([src, bs, np.zeros(deg, np.uint32), bd])
    g = bg.GraphData(x=np.zeros((n, 1), np.float32), numNodes=n, numFeatures=1, edgeIndex=ei,
                     numEdges=deg + 200000)
    dg = g.device_graph()
    idx = torch.arange(n, device="cuda")
    xm = torch.zeros((n, f), device="cuda")
    xm[idx, idx % f] = 1.0
    out = torch.empty((n, f), device="cuda")
    for _ in range(3):
        dg.ctx.call("bgnn_aggregate", dg.h, 0, ptr(xm), f, ptr(out))
        got = out[0].cpu().numpy()
        want = np.bincount(src % f, minlength=f).astype(np.float32)
        assert np.array_equal(got, want), (got - want)
