"""X*W on the tcgen05 tensor cores (BGNN_MATH_TENSOR, 3xTF32 split).

This mode is not the reference's summation order, so its bar is numerical,
against the exact product computed in float64: every output within
(2^-19 + 3 K 2^-24) * sum_k |a_k b_k| (the split's dropped terms plus one f32
rounding per accumulated product), and the median error below
2^-20 * sum_k |a_k b_k| (a dropped lo term would be 2^-11).  The count of elements
outside the reference parity bar (1e-6 + 1e-5 |ref| against the oracle) is
recorded, not required to be zero.  Shapes cover one and several n tiles,
widths that are not a multiple of 16, partial m tiles, both operand
segments (the SAGE pair), an addend, bias and activations, and the FP32
fallback for rows whose length is not a multiple of 4."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bg():
    import browsergnn_b200 as bg

    bg.init_browsergnn()
    ctx = bg.get_context()
    ctx.set_math("tensor")
    yield bg
    ctx.set_math("fast")


def _t(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _check(got, a_list, b_list, addend=None, bias=None, what=""):
    exact = sum(a.astype(np.float64) @ b.astype(np.float64) for a, b in zip(a_list, b_list))
    mag = sum(np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
              for a, b in zip(a_list, b_list))
    ref = exact.copy()
    if addend is not None:
        ref = ref + addend
        mag = mag + np.abs(addend)
    if bias is not None:
        ref = ref + bias
        mag = mag + np.abs(bias)
    ktot = sum(a.shape[1] for a in a_list)
    err = np.abs(got.astype(np.float64) - ref)
    bound = (2.0 ** -19 + 3 * ktot * 2.0 ** -24) * mag + 2.0 ** -23 * np.abs(ref) + 1e-30
    bad = err > bound
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} beyond the 3xTF32 bound; "
                           f"worst ratio {float((err / bound).max()):.3g}")
    rel = err / (mag + 1e-30)
    assert float(np.median(rel)) < 2.0 ** -20, (what, float(np.median(rel)))


@pytest.mark.parametrize("mkn", [(1, 32, 16), (300, 256, 256), (1000, 100, 47), (513, 32, 16),
                                 (4100, 256, 256), (700, 64, 300), (129, 48, 64), (257, 96, 128)])
def test_tensor_matmul_within_tf32x3_bound(bg, mkn):
    import torch

    m, k, n = mkn
    rng = np.random.default_rng(m + k + n)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = (rng.standard_normal((k, n)) * 0.1).astype(np.float32)
    got = bg.GPUTensor.matmul(_t(torch, a), _t(torch, b)).cpu().numpy()
    _check(got, [a], [b], what=f"matmul {mkn}")


def test_tensor_sage_pair_and_linear_add(bg):
    import torch

    from browsergnn_b200.backend import ptr

    ctx = bg.get_context()
    rng = np.random.default_rng(9)
    m, k, n = 3000, 256, 256
    x = rng.standard_normal((m, k)).astype(np.float32)
    agg = rng.standard_normal((m, k)).astype(np.float32)
    ws = (0.1 * rng.standard_normal((k, n))).astype(np.float32)
    wn = (0.1 * rng.standard_normal((k, n))).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    # device copies held for the whole call (a temporary dropped after ptr()
    # could hand its memory to the next operand)
    d_x, d_agg, d_ws, d_wn, d_b = (_t(torch, v) for v in (x, agg, ws, wn, bias))
    out = torch.empty((m, n), device="cuda")
    ctx.call("bgnn_sage_linear", ptr(d_agg), ptr(d_x), ptr(d_wn), ptr(d_ws), m, k, n, ptr(d_b), 0,
             0.0, ptr(out))
    _check(out.cpu().numpy(), [x, agg], [ws, wn], bias=bias, what="sage pair")
    addend = rng.standard_normal((m, n)).astype(np.float32)
    d_add = _t(torch, addend)
    out2 = torch.empty((m, n), device="cuda")
    ctx.call("bgnn_linear_add", ptr(d_agg), ptr(d_wn), m, k, n, ptr(d_add), ptr(d_b), 0, 0.0,
             ptr(out2))
    _check(out2.cpu().numpy(), [agg], [wn], addend=addend, bias=bias, what="linear_add")
    # ReLU epilogue: the activation applied to the same values
    out3 = torch.empty((m, n), device="cuda")
    ctx.call("bgnn_linear_add", ptr(d_agg), ptr(d_wn), m, k, n, ptr(d_add), ptr(d_b), 1, 0.0,
             ptr(out3))
    assert torch.equal(out3, torch.relu(out2))
    # the addend may be the output itself (in place)
    ctx.call("bgnn_linear_add", ptr(d_agg), ptr(d_wn), m, k, n, ptr(d_add), ptr(d_b), 0, 0.0,
             ptr(d_add))
    assert torch.equal(d_add, out2)


def test_tensor_mode_falls_back_for_unaligned_rows(bg):
    """k % 4 != 0: TMA cannot stream the rows, the FP32 kernel runs (and
    gives the FAST-mode result in the reference's order)."""
    import torch

    m, k, n = 200, 13, 40
    rng = np.random.default_rng(1)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    got = bg.GPUTensor.matmul(_t(torch, a), _t(torch, b)).cpu().numpy()
    want = orc.matmul(a, b, m, k, n).reshape(m, n)
    from tests.helpers import assert_close

    assert_close(got, want, "fallback")


def test_tensor_mode_sage_layer_against_oracle(bg):
    """A SAGE layer in tensor mode against the oracle: every element within
    the 3xTF32 error of the products; elements outside the reference parity
    bar are counted (the reference's own f32 rounding sequence differs)."""
    from tests.helpers import rand_graph

    rng = np.random.default_rng(21)
    n, fin, fout = 4000, 256, 256
    ei, e = rand_graph(n, 40000, 6, hub_deg=900)
    x = rng.standard_normal((n, fin)).astype(np.float32)
    wn = (0.06 * rng.standard_normal((fin, fout))).astype(np.float32)
    ws = (0.06 * rng.standard_normal((fin, fout))).astype(np.float32)
    b = rng.standard_normal(fout).astype(np.float32)
    layer = bg.SAGEConv(inChannels=fin, outChannels=fout)
    layer.loadStateDict({"lin_neighbor": wn, "lin_self": ws, "bias": b})
    g = bg.GraphData(x=x, numNodes=n, numFeatures=fin, edgeIndex=ei, numEdges=e)
    got = layer.forward(g).x.cpu().numpy().astype(np.float64)
    want = orc.sage_forward(x, n, fin, ei, e, "mean", wn, ws, b, fout).reshape(n, fout)
    # the oracle's aggregation (bit-exact on the GPU in every mode) as the A operand
    rp, so, _ = orc.dst_csr(ei, e, n)
    agg = orc.csr_aggregate(rp, so, n, x, fin, "mean", threads=0).reshape(n, fin)
    _check(got.astype(np.float32), [x, agg], [ws, wn], bias=b, what="sage layer")
    outside = np.abs(got - want) > 1e-6 + 1e-5 * np.abs(want)
    # The reference rounds after every k step; the tensor core accumulates
    # its own way, so a few per cent of the elements land outside the
    # element-wise parity bar (that is why this mode is not the default).
    # The rate is printed for the record and only checked for sanity.
    print(f"tensor mode: {int(outside.sum())} of {outside.size} elements outside the parity bar")
    assert outside.mean() < 0.2
