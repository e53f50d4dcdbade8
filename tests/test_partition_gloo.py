"""The N > 1 path on CPU: gloo ranks each derive the row-partition plan
(browsergnn_b200.partition.plan_rows, the host restatement of the device
plan), exchange halo rows with the plan's counts, and aggregate their rows
with the oracle over the local CSR.  Every rank's rows must equal the
single-process result bit for bit (each row keeps its COO edge order), and
the plans must agree across ranks without any exchange of requests."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from tests.helpers import rand_graph


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, n, f, ei, e, x, want, q):
    import torch
    import torch.distributed as dist

    from browsergnn_b200 import partition
    from oracle import oracle as orc

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rp, so = partition.dst_csr(ei, e, n)
        plan = partition.plan_rows(rp, so, world, rank)
        # every rank derived the same bounds, and what p receives from r is
        # what r sends to p, in the same (sorted id) order
        plans = [None] * world
        dist.all_gather_object(plans, (plan.bounds, plan.send_counts, plan.recv_counts,
                                       (plan.send_rows + plan.lo).tolist(),
                                       plan.halo_ids.tolist()))
        ok_plan = all(p[0] == plan.bounds for p in plans)
        for p in range(world):
            if p == rank:
                continue
            bounds, sc_p, rc_p, send_p, halo_p = plans[p]
            mine_from_p = [h for h in plan.halo_ids.tolist()
                           if bounds[p] <= h < bounds[p + 1]]
            off = sum(sc_p[:rank])
            ok_plan = ok_plan and rc_p[rank] == plan.send_counts[p]
            ok_plan = ok_plan and send_p[off:off + sc_p[rank]] == mine_from_p
        ext = torch.full((plan.n_own + plan.n_halo, f), float("nan"))
        ext[: plan.n_own] = torch.from_numpy(x[plan.lo:plan.hi])
        partition.exchange(plan, ext)
        need = np.concatenate([np.arange(plan.lo, plan.hi), plan.halo_ids]).astype(np.int64)
        ok_ext = np.array_equal(ext.numpy(), x[need])
        # the early sends' order: row block by row block, same halo
        for blocks in (1, 3, 4):
            ext_b = torch.full((plan.n_own + plan.n_halo, f), float("nan"))
            ext_b[: plan.n_own] = torch.from_numpy(x[plan.lo:plan.hi])
            partition.exchange_blocks(plan, ext_b, blocks)
            ok_ext = ok_ext and np.array_equal(ext_b.numpy(), x[need])
        res = {}
        for op in ("sum", "mean", "max"):
            got = orc.csr_aggregate(plan.row_ptr.astype(np.uint32), plan.col.astype(np.uint32),
                                    plan.n_own, ext.numpy(), f, op, threads=1).reshape(-1, f)
            res[op] = np.array_equal(got.view(np.uint32),
                                     want[op][plan.lo:plan.hi].view(np.uint32))
        q.put((rank, ok_plan, ok_ext, res, plan.n_own, int(plan.col.size)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_halo_partition_matches_single_process(world):
    from oracle import oracle as orc

    n, f = 3000, 5
    ei, e = rand_graph(n, 40000, seed=world, hub_deg=3000, loops=10, dup=50)
    x = np.random.default_rng(world).standard_normal((n, f)).astype(np.float32)
    rp, so, _ = orc.dst_csr(ei, e, n)
    want = {op: orc.csr_aggregate(rp, so, n, x, f, op, threads=1).reshape(n, f)
            for op in ("sum", "mean", "max")}
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, n, f, ei, e, x, want, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = [q.get() for _ in range(world)]
    total_rows = total_edges = 0
    for rank, ok_plan, ok_ext, res, n_own, ne in results:
        assert ok_plan, f"rank {rank}: plans disagree across ranks"
        assert ok_ext, f"rank {rank}: halo rows differ"
        assert all(res.values()), (rank, res)
        total_rows += n_own
        total_edges += ne
    assert total_rows == n and total_edges == e


def test_plan_edge_cases():
    """No edges (rows still balance), more ranks than rows, a hub row."""
    from browsergnn_b200 import partition

    rp = np.zeros(11, np.int64)
    b = partition.row_bounds(rp, 3)
    assert b[0] == 0 and b[-1] == 10 and all(b[i] <= b[i + 1] for i in range(3))
    assert max(b[i + 1] - b[i] for i in range(3)) <= 4
    rp2 = np.array([0, 1, 2], np.int64)
    plans = [partition.plan_rows(rp2, np.array([1, 0]), 4, r) for r in range(4)]
    assert sum(p.n_own for p in plans) == 2
    for p in plans:
        assert sum(p.recv_counts) == p.n_halo
    # one hub row holding most edges gets a rank of its own
    deg = np.array([5, 5, 1000, 5, 5, 5])
    rp3 = np.concatenate([[0], np.cumsum(deg)])
    col = np.random.default_rng(0).integers(0, 6, rp3[-1])
    plans = [partition.plan_rows(rp3, col, 3, r) for r in range(3)]
    owner = [r for r, p in enumerate(plans) if p.lo <= 2 < p.hi][0]
    assert plans[owner].n_own <= 3
