"""The row partition on the device (bgnn_part_*), checked on one GPU: every
rank's plan is derived without communication, so all ranks of a partition
can be built here and compared with the host restatement
(browsergnn_b200.partition.plan_rows).  The halo exchange is then played on
one GPU (each rank's halo rows copied from the full feature matrix), and the
local aggregations / SpMM must equal the whole graph's rows bit for bit, for
whole rows and for column slices (the pipelined exchange aggregates a layer
chunk by chunk)."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc
from tests.helpers import rand_graph

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bg():
    import browsergnn_b200 as bg

    bg.init_browsergnn()
    return bg


def _local_csr(ctx, pg):
    import torch

    from browsergnn_b200.backend import ptr

    rp = torch.empty(pg.n_own + 1, dtype=torch.int32, device="cuda")
    col = torch.empty(max(pg.num_local_edges, 1), dtype=torch.int32, device="cuda")
    ctx.call("bgnn_graph_csr", pg.graph, ptr(rp), ptr(col), None)
    return (rp.cpu().numpy().view(np.uint32).astype(np.int64),
            col[: pg.num_local_edges].cpu().numpy().view(np.uint32).astype(np.int64))


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_device_plan_matches_host_plan(bg, world):
    from browsergnn_b200 import partition
    from browsergnn_b200.distributed import PartitionedGraph

    n = 5000
    ei, e = rand_graph(n, 60000, seed=world, hub_deg=4000, loops=9, dup=40)
    rp, so = partition.dst_csr(ei, e, n)
    ctx = bg.get_context()
    for rank in range(world):
        want = partition.plan_rows(rp, so, world, rank)
        pg = PartitionedGraph.from_edge_index(ei, e, n, world, rank)
        assert pg.bounds == want.bounds
        assert (pg.lo, pg.hi, pg.n_halo, pg.entry_lo) == (want.lo, want.hi, want.n_halo,
                                                         want.entry_lo)
        assert pg.send_counts == want.send_counts and pg.recv_counts == want.recv_counts
        hid, srow = pg.lists()
        assert np.array_equal(hid.cpu().numpy(), want.halo_ids)
        assert np.array_equal(srow.cpu().numpy(), want.send_rows)
        lrp, lcol = _local_csr(ctx, pg)
        assert np.array_equal(lrp, want.row_ptr) and np.array_equal(lcol, want.col)
        for blocks in (1, 3, 4, 8):
            sf, rf = pg.row_blocks(blocks)
            wsf, wrf = partition.row_blocks(want, blocks)
            assert np.array_equal(sf.astype(np.int64), wsf), (rank, blocks)
            assert np.array_equal(rf.astype(np.int64), wrf), (rank, blocks)
        pg.close()


@pytest.mark.parametrize("world", [2, 5])
@pytest.mark.parametrize("aggr", ["sum", "mean", "max"])
def test_partitioned_aggregation_bit_exact(bg, world, aggr):
    import torch

    from browsergnn_b200.backend import ptr
    from browsergnn_b200.distributed import PartitionedGraph

    n, f = 4000, 100
    ei, e = rand_graph(n, 50000, seed=7, hub_deg=5000, loops=5, dup=30)
    x = torch.randn((n, f), device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    g = bg.GraphData(x=x, numNodes=n, numFeatures=f, edgeIndex=ei, numEdges=e)
    dg = g.device_graph()
    code = {"sum": 0, "mean": 1, "max": 2}[aggr]
    full = torch.empty((n, f), device="cuda")
    dg.ctx.call("bgnn_aggregate", dg.h, code, ptr(x), f, ptr(full))
    ctx = dg.ctx
    for rank in range(world):
        pg = PartitionedGraph.from_edge_index(ei, e, n, world, rank)
        hid, srow = pg.lists()
        ext = pg.ext_buffer(f)
        ext[: pg.n_own] = x[pg.lo:pg.hi]
        # the exchange played on one GPU: the owners' rows, packed as the
        # owners would pack them, unpacked into the halo rows
        halo = x.index_select(0, hid)
        ctx.call("bgnn_part_unpack", pg.h, ptr(halo.contiguous()), f, ptr(ext), f, 0)
        assert torch.equal(ext[pg.n_own:], halo)
        out = torch.full((pg.n_own, f), float("nan"), device="cuda")
        ctx.call("bgnn_aggregate_strided", pg.graph, code, None, ptr(ext), f, f, ptr(out), f)
        assert torch.equal(out.view(torch.int32), full[pg.lo:pg.hi].view(torch.int32))
        # column chunks of 36 / 36 / 28 (16-byte aligned starts), as the pipeline runs them
        out2 = torch.full((pg.n_own, f), float("nan"), device="cuda")
        for c0, w in ((0, 36), (36, 36), (72, 28)):
            ctx.call("bgnn_aggregate_strided", pg.graph, code, None, ptr(ext[:, c0:]), f, w,
                     ptr(out2[:, c0:]), f)
        assert torch.equal(out2.view(torch.int32), full[pg.lo:pg.hi].view(torch.int32))
        # what this rank packs for its peers: its owned rows in send order
        send = torch.empty((pg.n_send, 40), device="cuda")
        ctx.call("bgnn_part_pack", pg.h, ptr(ext), f, 8, 40, ptr(send))
        assert torch.equal(send, ext[srow][:, 8:48])
        pg.close()


def test_partitioned_spmm_bit_exact(bg):
    import torch

    from browsergnn_b200.backend import ptr
    from browsergnn_b200.distributed import PartitionedGraph

    n, nnz, f = 6000, 90000, 64
    rng = np.random.default_rng(3)
    rows = np.concatenate([rng.integers(0, n, nnz), np.full(3000, 11)]).astype(np.uint32)
    cols = rng.integers(0, n, rows.size).astype(np.uint32)
    vals = rng.uniform(0, 1, rows.size).astype(np.float32)
    csr = bg.SparseCSR.fromCOO(bg.SparseCOO(rows, cols, vals, (n, n)))
    x = torch.randn((n, f), device="cuda", generator=torch.Generator("cuda").manual_seed(2))
    full = csr.matmul(x)
    want = orc.spmm(csr.rowPtr.cpu().numpy().view(np.uint32),
                    csr.colIndices.cpu().numpy().view(np.uint32), csr.values.cpu().numpy(),
                    x.cpu().numpy(), n, f).reshape(n, f)
    from tests.helpers import assert_close

    assert_close(full.cpu().numpy(), want, "spmm")
    ctx = bg.get_context()
    world = 4
    for rank in range(world):
        pg = PartitionedGraph.from_csr(csr, world, rank)
        hid, _ = pg.lists()
        ext = pg.ext_buffer(f)
        ext[: pg.n_own] = x[pg.lo:pg.hi]
        ext[pg.n_own:] = x.index_select(0, hid)
        local = csr.values[pg.entry_lo:pg.entry_lo + pg.num_local_edges]
        out = torch.empty((pg.n_own, f), device="cuda")
        ctx.call("bgnn_aggregate_strided", pg.graph, 3, ptr(local), ptr(ext), f, f, ptr(out), f)
        assert torch.equal(out.view(torch.int32), full[pg.lo:pg.hi].view(torch.int32))
        pg.close()


def test_partition_rejects_bad_input(bg):
    import torch

    from browsergnn_b200.backend import ptr

    ctx = bg.get_context()
    h = ctypes.c_void_p()
    rp = torch.tensor([0, 2, 1, 3], dtype=torch.int32, device="cuda")  # decreases at row 1
    col = torch.zeros(3, dtype=torch.int32, device="cuda")
    with pytest.raises(bg.BGNNError):
        ctx.call("bgnn_part_create_csr", ptr(rp), ptr(col), 3, 2, 0, ctypes.byref(h))
    rp = torch.tensor([0, 1, 2, 3], dtype=torch.int32, device="cuda")
    col = torch.tensor([0, 7, 1], dtype=torch.int32, device="cuda")  # column 7 >= 3
    with pytest.raises(bg.BGNNError):
        ctx.call("bgnn_part_create_csr", ptr(rp), ptr(col), 3, 1, 0, ctypes.byref(h))
    with pytest.raises(bg.BGNNError):
        ctx.call("bgnn_part_create_csr", ptr(rp), ptr(col), 3, 2, 2, ctypes.byref(h))


def test_single_rank_dist_sage_matches_layer(bg):
    """A world of one through the NCCL path (communicator of one rank, no
    exchange): the partitioned SAGEConv equals the ordinary forward."""
    import torch

    from browsergnn_b200 import distributed
    from tests.helpers import assert_close

    n, fin, fout = 3000, 48, 40
    ei, e = rand_graph(n, 30000, seed=4, hub_deg=2000, loops=3)
    rng = np.random.default_rng(4)
    x = rng.standard_normal((n, fin)).astype(np.float32)
    layer = bg.SAGEConv(inChannels=fin, outChannels=fout)
    layer.loadStateDict({"lin_neighbor": (0.1 * rng.standard_normal((fin, fout))).astype(np.float32),
                         "lin_self": (0.1 * rng.standard_normal((fin, fout))).astype(np.float32),
                         "bias": rng.standard_normal(fout).astype(np.float32)})
    g = bg.GraphData(x=x, numNodes=n, numFeatures=fin, edgeIndex=ei, numEdges=e)
    want = layer.forward(g, _act="relu").x
    d = distributed.DistContext(0, 1, unique_id=distributed.DistContext.make_unique_id(),
                                timeout_ms=30000)
    try:
        pgd = distributed.partition(g, d)
        got = layer.forward(pgd, _act="relu").x
        d.synchronize()
        assert torch.equal(got.view(torch.int32), want.view(torch.int32))
        assert_close(got.cpu().numpy(), orc.relu(orc.sage_forward(
            x, n, fin, ei, e, "mean", layer.p("lin_neighbor").cpu().numpy(),
            layer.p("lin_self").cpu().numpy(), layer.p("bias").cpu().numpy(),
            fout)).reshape(n, fout), "dist sage")
        assert d.allreduce_max([1.5, -2.0]) == [1.5, -2.0]
    finally:
        d.close()
