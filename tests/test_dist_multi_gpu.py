"""The NCCL path on 2-4 GPUs (one spawned process per GPU; skipped with fewer
than two): partitioned SAGEConv layers and the row-partitioned SpMM must give
every rank's rows bit for bit as a single-GPU run does, and a peer that
never joins an exchange must turn into a TIMEOUT error, not a hang.

Failures are made on the host only (a rank that skips a call); NVLS is off
in every rank and the exchange uses plain NCCL point-to-point transfers."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gpus():
    try:
        import torch

        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


needs2 = pytest.mark.skipif(_gpus() < 2, reason="needs at least two GPUs")


def _spawn(target, world, *args):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    ids = ctx.SimpleQueue()
    go = [ctx.SimpleQueue() for _ in range(world)]
    procs = [ctx.Process(target=target, args=(r, world, q, ids, go) + args) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get() for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return sorted(res, key=lambda r: r[0])


def _share_id(rank, world, ids):
    from browsergnn_b200.distributed import DistContext

    if rank == 0:
        uid = DistContext.make_unique_id()
        for _ in range(world - 1):
            ids.put(uid)
        return uid
    return ids.get()


def _layers_main(rank, world, q, ids, go, chunks, blocks):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    import browsergnn_b200 as bg
    from browsergnn_b200 import distributed
    from tests.helpers import rand_graph

    torch.cuda.set_device(rank)
    bg.init_browsergnn({"device": rank})
    try:
        n = 6000
        ei, e = rand_graph(n, 80000, seed=11, hub_deg=6000, loops=4, dup=20)
        rng = np.random.default_rng(5)
        x = rng.standard_normal((n, 100)).astype(np.float32)
        widths = [100, 256, 47]
        layers = []
        for fin, fout in zip(widths[:-1], widths[1:]):
            lay = bg.SAGEConv(inChannels=fin, outChannels=fout)
            lay.loadStateDict({"lin_neighbor": (0.1 * rng.standard_normal((fin, fout))).astype(np.float32),
                               "lin_self": (0.1 * rng.standard_normal((fin, fout))).astype(np.float32),
                               "bias": rng.standard_normal(fout).astype(np.float32)})
            layers.append(lay)
        g = bg.GraphData(x=x, numNodes=n, numFeatures=100, edgeIndex=ei, numEdges=e)
        h = g
        for i, lay in enumerate(layers):
            h = lay.forward(h, _act="relu" if i == 0 else None)
        want = h.x
        d = distributed.DistContext(rank, world, unique_id=_share_id(rank, world, ids),
                                    timeout_ms=60000)
        d.set_pipeline(chunks, 16)
        if blocks:
            d.set_row_blocks(blocks)
        pgd = distributed.partition(g, d)
        for _ in range(2):  # twice: the staging buffers are reused
            h = pgd
            for i, lay in enumerate(layers):
                last = i == len(layers) - 1
                h = lay.forward(h, _act=None if last else "relu",
                                _send_next=bool(blocks) and not last)
        d.synchronize()
        lo, hi = pgd.pg.lo, pgd.pg.hi
        ok = bool(torch.equal(h.x.view(torch.int32), want[lo:hi].view(torch.int32)))
        # the row-partitioned SpMM
        rows = np.concatenate([rng.integers(0, n, 70000), np.full(2500, 3)]).astype(np.uint32)
        cols = rng.integers(0, n, rows.size).astype(np.uint32)
        vals = rng.uniform(0, 1, rows.size).astype(np.float32)
        csr = bg.SparseCSR.fromCOO(bg.SparseCOO(rows, cols, vals, (n, n), device=rank))
        xs = torch.from_numpy(rng.standard_normal((n, 64)).astype(np.float32)).cuda()
        full = csr.matmul(xs)
        pg = distributed.PartitionedGraph.from_csr(csr, world, rank)
        ext = pg.ext_buffer(64)
        ext[: pg.n_own] = xs[pg.lo:pg.hi]
        out = pg.spmm(d, csr.values, ext)
        d.synchronize()
        ok_spmm = bool(torch.equal(out.view(torch.int32), full[pg.lo:pg.hi].view(torch.int32)))
        mx = d.allreduce_max([float(rank)])
        q.put((rank, ok, ok_spmm, hi - lo, mx[0]))
        pg.close()
        pgd.pg.close()
        d.close()
    except Exception as exc:  # noqa: BLE001 - report, do not hang the parent
        q.put((rank, False, False, 0, repr(exc)))
        raise


@needs2
@pytest.mark.parametrize("chunks,blocks", [(1, 0), (4, 0), (1, 4), (1, 1), (2, 8)])
def test_partitioned_layers_and_spmm_match_one_gpu(chunks, blocks):
    """blocks > 0: each layer's output halo is sent early, row block by row
    block, while the layer's last product runs."""
    world = min(_gpus(), 4)
    res = _spawn(_layers_main, world, chunks, blocks)
    assert sum(r[3] for r in res) == 6000
    for rank, ok, ok_spmm, _, mx in res:
        assert ok, f"rank {rank}: SAGE rows differ from the single-GPU forward ({mx})"
        assert ok_spmm, f"rank {rank}: SpMM rows differ"
        assert mx == world - 1


def _timeout_main(rank, world, q, ids, go):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import time

    import torch

    import browsergnn_b200 as bg
    from browsergnn_b200 import distributed
    from tests.helpers import rand_graph

    torch.cuda.set_device(rank)
    bg.init_browsergnn({"device": rank})
    n = 2000
    ei, e = rand_graph(n, 20000, seed=2)
    g = bg.GraphData(x=np.ones((n, 16), np.float32), numNodes=n, numFeatures=16, edgeIndex=ei,
                     numEdges=e)
    d = distributed.DistContext(rank, world, unique_id=_share_id(rank, world, ids),
                                timeout_ms=2000)
    pgd = distributed.partition(g, d)
    status, took = None, 0.0
    if rank == 0:
        # rank 1 never posts its side of this exchange
        t0 = time.time()
        try:
            pgd.pg.aggregate(d, pgd.x_ext, "sum")
            d.synchronize()
            status = "ok"
        except bg.BGNNError as exc:
            status = exc.status
        took = time.time() - t0
        for r in range(1, world):
            go[r].put("done")
    else:
        go[rank].get()  # idle (no collective in flight) until rank 0 has its answer
        d.abort()  # learned on the host that the job is over
    q.put((rank, status, took))
    pgd.pg.close()
    d.close()


@needs2
def test_missing_peer_times_out():
    from browsergnn_b200._lib import ERR_TIMEOUT

    res = _spawn(_timeout_main, 2)
    rank0 = res[0]
    assert rank0[1] == ERR_TIMEOUT, rank0
    assert rank0[2] < 30.0
