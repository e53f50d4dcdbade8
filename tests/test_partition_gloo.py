"""The N > 1 path on CPU: two gloo ranks build the row partition and halo plan
(browsergnn_b200.partition.HaloPlan), exchange halo rows, and aggregate their
rows with the oracle over the local CSR.  Every rank's rows must equal the
single-process result bit for bit (each row keeps its COO edge order)."""
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

    from browsergnn_b200.partition import HaloPlan
    from oracle import oracle as orc

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        t = torch.from_numpy(ei.view(np.int32).copy())
        plan = HaloPlan(t[:e], t[e:], n, rank, world)
        xl = torch.from_numpy(x[plan.lo:plan.hi].copy())

        def pack(h, rows, out):  # CPU stand-in for bgnn_pack_rows
            out.copy_(h.index_select(0, rows.long()))

        ext = plan.exchange(xl, pack).numpy()
        need = np.concatenate([np.arange(plan.lo, plan.hi), plan.halo.numpy()]).astype(np.int64)
        ok_ext = np.array_equal(ext, x[need])
        # in-place variant: owned rows already in the buffer, only halo rows move
        buf = torch.full((plan.n_own + plan.n_halo, f), float("nan"))
        buf[: plan.n_own].copy_(xl)
        plan.exchange_into(buf, pack)
        ok_ext = ok_ext and np.array_equal(buf.numpy(), x[need])
        lei = plan.edge_index.numpy().view(np.uint32)
        rp, so, _ = orc.dst_csr(np.concatenate([lei[:plan.num_edges], lei[plan.num_edges:]]),
                                plan.num_edges, plan.n_own)
        res = {}
        for op in ("sum", "mean", "max"):
            got = orc.csr_aggregate(rp, so, plan.n_own, ext, f, op, threads=1).reshape(-1, f)
            res[op] = np.array_equal(got.view(np.uint32),
                                     want[op][plan.lo:plan.hi].view(np.uint32))
        # remote-store map: applying every rank's (peer, row) destinations to
        # its owned rows must reproduce each rank's halo rows exactly
        row_ptr, dst, peer_rows = plan.remote_map()
        maps = [None] * world
        dist.all_gather_object(maps, (plan.lo, plan.n_own, row_ptr.tolist(), dst.tolist(),
                                      peer_rows))
        buf = np.full((plan.n_own + plan.n_halo, f), np.nan, np.float32)
        buf[: plan.n_own] = x[plan.lo:plan.hi]
        ok_map = peer_rows[rank] == plan.n_own + plan.n_halo
        for lo_p, n_own_p, rp_p, dst_p, _ in maps:
            for i in range(n_own_p):
                for d in dst_p[rp_p[i]:rp_p[i + 1]]:
                    if (d >> 32) == rank:
                        ok_map = ok_map and (d & 0xffffffff) >= plan.n_own
                        buf[d & 0xffffffff] = x[lo_p + i]
        ok_map = ok_map and np.array_equal(buf, x[need])
        q.put((rank, ok_ext and ok_map, res, plan.n_own, plan.n_halo, plan.num_edges))
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
    for rank, ok_ext, res, n_own, n_halo, ne in results:
        assert ok_ext, f"rank {rank}: halo rows differ"
        assert all(res.values()), (rank, res)
        total_rows += n_own
        total_edges += ne
    assert total_rows == n and total_edges == e
