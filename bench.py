"""Benchmark: aggregated edges/s per layer forward on B200.

Workload (one step): a full-graph forward of the 3-layer GraphSAGE-mean stack
(100 -> 256 -> 256 -> 47, root weight, ReLU between layers) over a seeded
R-MAT graph with 2,450,000 nodes and 62,000,000 directed edges (a=0.57,
b=c=0.19, ids permuted) and N(0,1) features.  Metric = edges aggregated per
second per layer forward = 3 * E / step time.  Inputs are resident in HBM
(features 0.98-2.5 GB per layer, far larger than the 126 MB L2, so no L2
flush is needed between steps).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N > 1 (torchrun, one rank per GPU): the graph's destination rows are
partitioned by edge count across ranks; each layer exchanges the halo rows
with NCCL all-to-all before the local aggregation (strong scaling).

Extra keys: roofline of the dominant kernel (the F=256 aggregation), the CPU
baseline (the oracle on a 1/64 sample of the workload, all host threads),
e2e through the public API with host buffers, clocks during the timed region,
and at N=1 the standalone SpMM sweep (scale-24 R-MAT, 2^28 edges).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "aggregated edges/s per layer forward"
UNIT = "edges/s"
WIDTHS = [100, 256, 256, 47]
FALLBACK_HBM_GBS = 6650.0


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        try:
            d = json.load(open(p))
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(name):
    """(dram bytes per launch, where the figure comes from) from a committed
    ncu summary (profiles/<name>.md, lines 'dram_bytes_per_launch: <int>' and
    'captured: <what>'), or (None, None)."""
    p = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(p):
        return None, None
    val, what = None, None
    for line in open(p):
        t = line.strip()
        if t.startswith("dram_bytes_per_launch:"):
            try:
                val = int(t.split(":", 1)[1].strip().split()[0])
            except ValueError:
                val = None
        elif t.startswith("captured:"):
            what = t.split(":", 1)[1].strip()
    src = f"profiles/{name}.md" + (f" ({what})" if what else "")
    return val, src


def max_over_ranks(v):
    """Element-wise maximum over the ranks of a float or a list of floats."""
    import torch
    import torch.distributed as dist

    scalar = not isinstance(v, (list, tuple))
    t = torch.tensor([v] if scalar else list(v), dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    out = t.tolist()
    return out[0] if scalar else out


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        os.unlink(self.path)
        loaded = [s for s in sm if smax and s > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": smax,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# the SAGE stack on libbgnn_cuda
# ---------------------------------------------------------------------------
def make_weights(seed):
    from browsergnn_b200 import synth

    rng = np.random.default_rng(seed)
    layers = []
    for fin, fout in zip(WIDTHS[:-1], WIDTHS[1:]):
        layers.append({"lin_neighbor": synth.glorot(fin, fout, rng),
                       "lin_self": synth.glorot(fin, fout, rng),
                       "bias": rng.uniform(-0.1, 0.1, fout).astype(np.float32)})
    return layers


def build_layers(weights, device):
    import browsergnn_b200 as bg

    layers = []
    for (fin, fout), w in zip(zip(WIDTHS[:-1], WIDTHS[1:]), weights):
        lay = bg.SAGEConv(inChannels=fin, outChannels=fout, aggregator="mean")
        lay.loadStateDict(w)
        lay.to_device(device)
        layers.append(lay)
    return layers


def sage_forward(layers, dg, x, timers=None):
    """Three SAGEConv layers on one GPU (aggregate -> fused dual GEMM + bias +
    ReLU).  `timers` collects CUDA events around each phase (aggregate,
    linear)."""
    import torch

    from browsergnn_b200.backend import ptr

    ctx = dg.ctx
    n_own = dg.num_dst
    h = x

    def mark():
        if timers is None:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return ev

    for li, lay in enumerate(layers):
        fin, fout = lay.inChannels, lay.outChannels
        e0 = mark()
        agg = torch.empty((n_own, fin), dtype=torch.float32, device=h.device)
        e1 = mark()
        ctx.call("bgnn_aggregate", dg.h, 1, ptr(h), fin, ptr(agg))
        e2 = mark()
        out = torch.empty((n_own, fout), dtype=torch.float32, device=h.device)
        act = 1 if li < len(layers) - 1 else 0  # ReLU between layers (wasmRelu)
        ctx.call("bgnn_sage_linear", ptr(agg), ptr(h), ptr(lay.p("lin_neighbor")),
                 ptr(lay.p("lin_self")), n_own, fin, fout, ptr(lay.p("bias")), act, 0.0,
                 ptr(out))
        e3 = mark()
        if timers is not None:
            timers.append((li, fin, e1, e2, e0, e3))
        h = out
    return h


def dist_forward(layers, pgd, timers=None, early=True):
    """The same three layers on one rank of the row partition
    (browsergnn_b200.distributed): each SAGEConv.forward on the
    PartitionedGraphData runs x * W_self on a side stream while its input's
    halo rows arrive over NCCL, aggregates, and writes its output into the
    owned rows of the next layer's [owned | halo] buffer; with `early` the
    next layer's halo rows are sent block by block while that last product
    runs.  `timers` collects CUDA events around each layer."""
    import torch

    h = pgd
    for li, lay in enumerate(layers):
        a = b = None
        if timers is not None:
            a = torch.cuda.Event(enable_timing=True)
            a.record()
        last = li == len(layers) - 1
        h = lay.forward(h, _act=None if last else "relu", _send_next=early and not last)
        if timers is not None:
            b = torch.cuda.Event(enable_timing=True)
            b.record()
            timers.append((li, lay.inChannels, None, None, a, b))
    return h.x


def exchange_times(pg, dctx, reps):
    """The halo exchange alone (bgnn_dist_exchange, whole width in one NCCL
    group) per layer input width: ms, mean over reps, max over ranks."""
    import torch
    import torch.distributed as dist

    from browsergnn_b200.backend import ptr

    res = {}
    for f in sorted(set(WIDTHS[:-1])):
        ext = pg.ext_buffer(f)
        ext.normal_()
        for _ in range(2):
            pg.ctx.call_on("bgnn_dist_exchange", dctx.h, pg.h, ptr(ext), f)
        torch.cuda.synchronize()
        dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            pg.ctx.call_on("bgnn_dist_exchange", dctx.h, pg.h, ptr(ext), f)
        b.record()
        dctx.synchronize()
        ms = max_over_ranks(a.elapsed_time(b) / reps)
        recv = max_over_ranks(float(pg.n_halo * f * 4))
        res[f"F{f}"] = {"ms": round(ms, 3), "max_recv_bytes": int(recv),
                        "recv_GBps_at_max": round(recv / (ms * 1e-3) / 1e9, 1)}
        del ext
    return res


def layer_parts(layers, pg, dctx, reps):
    """The pieces of a partitioned layer run one at a time on this rank's
    share (ms, mean over reps, max over ranks): the aggregation over the
    full width and over four column chunks, x * W_self and the fused
    neighbour product.  Shows what the pipelined layer overlaps."""
    import torch
    import torch.distributed as dist

    from browsergnn_b200.backend import ptr

    ctx = pg.ctx
    m = pg.n_own

    def timed(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    out = {}
    for li, lay in enumerate(layers):
        k, n = lay.inChannels, lay.outChannels
        ext = pg.ext_buffer(k)
        ext.normal_()
        agg = torch.empty((m, k), device="cuda")
        st = torch.empty((m, n), device="cuda")
        res = torch.empty((m, n), device="cuda")
        step = (k + 3) // 4
        step = (step + 3) & ~3
        chunks = [(c0, min(step, k - c0)) for c0 in range(0, k, step)]

        def agg_full():
            ctx.call("bgnn_aggregate_strided", pg.graph, 1, None, ptr(ext), k, k, ptr(agg), k)

        def agg_chunks():
            for c0, w in chunks:
                ctx.call("bgnn_aggregate_strided", pg.graph, 1, None, ptr(ext[:, c0:]), k, w,
                         ptr(agg[:, c0:]), k)

        def self_mm():
            ctx.call("bgnn_linear", ptr(ext), ptr(lay.p("lin_self")), m, k, n, None, 0, 0.0,
                     ptr(st))

        def neigh_mm():
            ctx.call("bgnn_linear_add", ptr(agg), ptr(lay.p("lin_neighbor")), m, k, n, ptr(st),
                     ptr(lay.p("bias")), 1, 0.0, ptr(res))

        v = [timed(agg_full), timed(agg_chunks), timed(self_mm), timed(neigh_mm)]
        v = max_over_ranks(v)
        out[f"L{li + 1}"] = {"aggregate_full_width": round(v[0], 3),
                             f"aggregate_{len(chunks)}_chunks": round(v[1], 3),
                             "x_w_self": round(v[2], 3), "agg_w_neigh_add": round(v[3], 3)}
        del ext, agg, st, res
    return out


def e2e_single(layers, ei, x, n, e, warmup, steps):
    """The public API from ordinary (pageable) host arrays, as a Node-API
    caller hands over typed arrays: GraphData from the host edge list and
    features (the edge list staged to the device and the CSR built and
    validated there while the features upload on a second host thread,
    both through the library's pinned staging), 3 layers, the result read
    back into a host array through the same staging."""
    import browsergnn_b200 as bg

    ei_host = np.ascontiguousarray(ei.cpu().numpy().view(np.uint32))
    x_host = np.ascontiguousarray(x.cpu().numpy())
    res = np.empty((n, WIDTHS[-1]), np.float32)
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        g = bg.GraphData(x=x_host, numNodes=n, numFeatures=WIDTHS[0], edgeIndex=ei_host,
                         numEdges=e)
        out = g
        for li, lay in enumerate(layers):
            out = lay.forward(out, _act="relu" if li < 2 else None)
        bg.to_host(out.x, res)
        t1 = time.perf_counter()
        out.device_graph().close()
        if i >= warmup:
            times.append(t1 - t0)
    s = statistics.mean(times)
    # one more, untimed, step with the phases separated (each one synchronised)
    import torch

    ph = {}
    t0 = time.perf_counter()
    g = bg.GraphData(x=x_host, numNodes=n, numFeatures=WIDTHS[0], edgeIndex=ei_host, numEdges=e)
    g.device_graph()
    torch.cuda.synchronize()
    ph["edge_upload_and_csr_build"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    g.x_device()
    ph["feature_upload_left_after_the_build"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    out = g
    for li, lay in enumerate(layers):
        out = lay.forward(out, _act="relu" if li < 2 else None)
    torch.cuda.synchronize()
    ph["three_layers"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    bg.to_host(out.x, res)
    ph["result_readback"] = time.perf_counter() - t0
    out.device_graph().close()
    return {"value": 3 * e / s, "unit": UNIT,
            "h2d_bytes_per_step": int(x_host.nbytes + ei_host.nbytes),
            "d2h_bytes_per_step": int(res.nbytes), "ms_per_step": round(1000 * s, 3),
            "includes": "pageable host arrays in (staged by the library), device CSR build and "
                        "validation, 3 layers, the result read back into a pageable array",
            "phases_ms_one_step": {k: round(1000 * v, 2) for k, v in ph.items()}}


def e2e_partitioned(layers, ei, x_own, pg0, n, e, dctx, rank, world, warmup, steps):
    """The public API on every rank from pinned host buffers: the full edge
    list in (each rank derives the partition plan from it on its device: CSR
    build, bounds, halo and send lists), this rank's feature rows in, 3
    partitioned layers, this rank's output rows out.  Host wall time per
    step, max over ranks."""
    import torch
    import torch.distributed as dist

    from browsergnn_b200 import distributed

    ei_host = ei.cpu().pin_memory()
    # every rank holds the whole feature matrix on the host, as a user would
    x_host = torch.empty((n, WIDTHS[0]), dtype=torch.float32, pin_memory=True)
    x_host[pg0.lo:pg0.hi].copy_(x_own)
    res = torch.empty((pg0.n_own, WIDTHS[-1]), dtype=torch.float32, pin_memory=True)
    times = []
    h2d = d2h = 0
    for i in range(warmup + steps):
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        pg = distributed.PartitionedGraph.from_edge_index(ei_host, e, n, world, rank)
        ext = pg.ext_buffer(WIDTHS[0])
        ext[: pg.n_own].copy_(x_host[pg.lo:pg.hi], non_blocking=True)
        h = distributed.PartitionedGraphData(pg, dctx, ext, WIDTHS[0])
        for li, lay in enumerate(layers):
            h = lay.forward(h, _act="relu" if li < 2 else None)
        res[: pg.n_own].copy_(h.x)
        t1 = time.perf_counter()
        h2d = ei_host.numel() * 4 + pg.n_own * WIDTHS[0] * 4
        d2h = pg.n_own * WIDTHS[-1] * 4
        h = None
        pg.close()
        if i >= warmup:
            times.append(t1 - t0)
    s = max_over_ranks(statistics.mean(times))
    return {"value": 3 * e / s, "unit": UNIT, "h2d_bytes_per_step": int(max_over_ranks(h2d)),
            "d2h_bytes_per_step": int(max_over_ranks(d2h)), "ms_per_step": round(1000 * s, 3),
            "includes": "per rank: H2D of the full edge list and the rank's feature rows "
                        "(pinned), device CSR build and partition plan, 3 layers with NCCL halo "
                        "exchange, D2H of the rank's rows; host wall time, max over ranks"}


# ---------------------------------------------------------------------------
# SpMM sweep (standalone CSR SpMM, scale-24 R-MAT, 2^28 edges)
# ---------------------------------------------------------------------------
def spmm_sweep(steps, warmup, hbm_peak, parity=True, dctx=None, rank=0, world=1):
    """The standalone CSR SpMM (SparseCSR.matmul) of the scale-24 R-MAT
    matrix with 2^28 entries at F = 32/64/128/256.  N>1: rows partitioned
    across the ranks (browsergnn_b200.distributed.PartitionedGraph.from_csr),
    the halo rows of X exchanged with NCCL (grouped send/recv) before the
    local SpMM; time = max over ranks."""
    import torch

    import browsergnn_b200 as bg
    from browsergnn_b200 import synth
    from browsergnn_b200.backend import ptr

    dev = torch.cuda.current_device()
    n, e, scale = 1 << synth.SPMM_SCALE, synth.SPMM_E, synth.SPMM_SCALE
    seed = synth.seed_for(5)
    ei = synth.rmat_edges_gpu(scale, n, e, seed, device=dev)
    ctx = bg.get_context(dev)
    # values f32(u * dinv[src] * dinv[dst]) with u ~ U(0,1] and dinv from the in-degree
    dinv = bg.compute_gcn_norm(ei, e, n, False)  # dinv[s]*dinv[t] per edge
    u = 1.0 - torch.rand(e, device="cuda", generator=torch.Generator("cuda").manual_seed(seed))
    vals = (u.float() * dinv).contiguous()
    del dinv
    rows = ei[:e]
    cols = ei[e:]
    coo = bg.SparseCOO(rows, cols, vals, (n, n), device=dev)
    for rep in range(2):  # the first build also grows the memory pool
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        csr = bg.SparseCSR.fromCOO(coo)
        t1.record()
        torch.cuda.synchronize()
        build_ms = t0.elapsed_time(t1)
        if rep == 0:
            first_ms = build_ms
            del csr
    del ei, rows, cols, vals, u, coo
    g = csr.graph()
    res = {"workload": f"spmm-rmat-s{scale}-{n}n-{e}e", "csr_build_ms": round(build_ms, 3),
           "csr_build_first_ms": round(first_ms, 3),
           "csr_build": "SparseCSR.fromCOO of 2^28 entries on the device (stable (row, col) "
                        "radix sort), second call; the first also grows the memory pool"}
    pg = None
    if world > 1:
        from browsergnn_b200 import distributed

        t0 = time.perf_counter()
        pg = distributed.PartitionedGraph.from_csr(csr, world, rank)
        torch.cuda.synchronize()
        res["partition_plan_s"] = round(max_over_ranks(time.perf_counter() - t0), 3)
        lrp = torch.empty(pg.n_own + 1, dtype=torch.int32, device="cuda")
        ctx.call("bgnn_graph_csr", pg.graph, ptr(lrp), None, None)
        deg = (lrp[1:] - lrp[:-1]).max().item() if pg.n_own else 0
        res["max_row_entries_over_ranks"] = int(max_over_ranks(float(deg)))
        del lrp
        res["parallelism"] = f"row-partition x{world}"
        res["scaling"] = "strong"
    per_f = {}
    gen = torch.Generator("cuda").manual_seed(seed + 1)
    host_csr = None
    if parity and world == 1:
        host_csr = (csr.rowPtr.cpu().numpy().view(np.uint32),
                    csr.colIndices.cpu().numpy().view(np.uint32), csr.values.cpu().numpy())
    for f in (32, 64, 128, 256):
        x = torch.randn((n, f), device="cuda", generator=gen)
        if pg is None:
            out = torch.empty((n, f), device="cuda")

            def run():
                ctx.call("bgnn_graph_spmm", g.h, ptr(csr.values), ptr(x), f, ptr(out))
        else:
            ext = pg.ext_buffer(f)
            ext[: pg.n_own].copy_(x[pg.lo:pg.hi])
            out = torch.empty((pg.n_own, f), device="cuda")

            def run():
                pg.spmm(dctx, csr.values, ext, out)
        for _ in range(warmup):
            run()
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            run()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        if world > 1:
            ms = max_over_ranks(ms)
        bytes_alg = 4 * (n + 1) + 8 * e + 4 * f * e + 4 * f * n  # rowPtr, col, val, gathers, out
        gbs = bytes_alg / (ms * 1e-3) / 1e9
        per_f[str(f)] = {"ms": round(ms, 3), "edges_per_s": e / (ms * 1e-3),
                         "gather_model_GBps": round(gbs, 1),
                         "hbm_frac_gather_model": round(gbs / hbm_peak / world, 3),
                         "compulsory_GBps": round((4 * (n + 1) + 8 * e + 8 * f * n)
                                                  / (ms * 1e-3) / 1e9, 1)}
        if host_csr is not None and f in (32, 256):
            per_f[str(f)]["parity"] = spmm_parity(host_csr, x, out, f, seed)
        if pg is not None:
            # where the time goes: the exchange alone and the local SpMM alone
            local_vals = csr.values[pg.entry_lo:pg.entry_lo + pg.num_local_edges]

            def parts(fn):
                for _ in range(2):
                    fn()
                torch.cuda.synchronize()
                import torch.distributed as dist

                dist.barrier()
                a0 = torch.cuda.Event(enable_timing=True)
                a1 = torch.cuda.Event(enable_timing=True)
                a0.record()
                for _ in range(steps):
                    fn()
                a1.record()
                dctx.synchronize()
                return round(max_over_ranks(a0.elapsed_time(a1) / steps), 3)

            per_f[str(f)]["exchange_ms"] = parts(
                lambda: ctx.call_on("bgnn_dist_exchange", dctx.h, pg.h, ptr(ext), f))
            per_f[str(f)]["local_spmm_ms"] = parts(
                lambda: ctx.call("bgnn_graph_spmm", pg.graph, ptr(local_vals), ptr(ext), f,
                                 ptr(out)))
            per_f[str(f)]["max_halo_rows"] = int(max_over_ranks(float(pg.n_halo)))
        if pg is not None and parity and f in (32, 256):
            # each rank's rows against a single-GPU SpMM of the whole matrix
            full = torch.empty((n, f), device="cuda")
            ctx.call("bgnn_graph_spmm", g.h, ptr(csr.values), ptr(x), f, ptr(full))
            mine = full[pg.lo:pg.hi]
            bad = int((mine.view(torch.int32) != out.view(torch.int32)).sum().item())
            tot = max_over_ranks([float(bad)])
            per_f[str(f)]["bit_identical_to_1gpu"] = tot[0] == 0
            del full, mine
        del x, out
    res["per_feature_width"] = per_f
    if pg is not None:
        pg.close()
    g.close()
    return res


def partition_bit_identity(ei, n, e, seed, layers, part, got, device):
    """Each rank's rows of the partitioned forward against the same rows of a
    single-GPU forward of the whole graph on that rank's GPU: every row is
    reduced in the same order on one GPU either way, so the bits must agree.
    Returns the mismatch count summed over ranks."""
    import torch
    import torch.distributed as dist

    from browsergnn_b200.graph import DeviceGraph

    gen = torch.Generator("cuda").manual_seed(seed)
    x_full = torch.randn((n, WIDTHS[0]), device="cuda", generator=gen)
    dg = DeviceGraph(ei, e, n, n, device=device)
    ref = sage_forward(layers, dg, x_full)
    mine = ref[part.lo:part.hi]
    bad = (mine.view(torch.int32) != got.view(torch.int32)) & ~(torch.isnan(mine) & torch.isnan(got))
    counts = torch.tensor([int(bad.sum().item()), int(got.numel())], device="cuda",
                          dtype=torch.int64)
    dist.all_reduce(counts)
    del ref, mine, x_full
    dg.close()
    return {"bit_identical_to_1gpu": bool(counts[0].item() == 0),
            "differing_elements": int(counts[0].item()), "elements": int(counts[1].item()),
            "checked": "every rank's rows against a single-GPU forward of the whole graph"}


def spmm_parity(host_csr, x, out, f, seed):
    """The SpMM output against the oracle's row-parallel wasmSpmm restatement
    (same per-row order and roundings): every row at F = 32; at wider F every
    heavy row (>= 256 entries, the hub and giant-row paths) plus 2,000,000
    seeded random rows."""
    from oracle import oracle as orc

    rp, col, val = host_csr
    n = rp.size - 1
    t0 = time.perf_counter()
    x_h = x.cpu().numpy()
    if f <= 32:
        rows = None
        got = out.cpu().numpy()
        what = f"all {n} rows"
    else:
        import torch

        deg = np.diff(rp.astype(np.int64))
        heavy = np.flatnonzero(deg >= 256).astype(np.uint32)
        rnd = np.random.default_rng(seed).integers(0, n, 2_000_000).astype(np.uint32)
        rows = np.unique(np.concatenate([heavy, rnd]))
        idx = torch.from_numpy(rows.astype(np.int64)).to(out.device)
        got = out.index_select(0, idx).cpu().numpy()
        what = (f"{rows.size} rows: all {heavy.size} rows with >= 256 entries "
                f"({int(deg[heavy].sum())} entries) + 2,000,000 random rows")
    want = orc.spmm_rows(rp, col, val, x_h, f, rows=rows, num_rows=n, threads=0)
    res = _parity(got, want.reshape(got.shape))
    res["checked"] = what
    res["oracle_seconds"] = round(time.perf_counter() - t0, 1)
    return res


def sage_oracle_parity(ei, n, e, x, weights, got_dev):
    """The full 3-layer SAGE output (every row, every feature) against the
    oracle's row-parallel restatement on all host threads."""
    from oracle import oracle as orc

    t0 = time.perf_counter()
    got = got_dev.cpu().numpy()
    ei_h = ei.cpu().numpy().view(np.uint32)
    rp, so, _ = orc.dst_csr(ei_h, e, n)
    del ei_h
    h = x.cpu().numpy()
    for li, (fin, fout) in enumerate(zip(WIDTHS[:-1], WIDTHS[1:])):
        lw = weights[li]
        h = orc.sage_forward_csr(rp, so, n, h, fin, "mean", lw["lin_neighbor"], lw["lin_self"],
                                 lw["bias"], fout, relu=li < 2, threads=0)
    want = h.reshape(got.shape)
    res = _parity(got, want)
    res["checked"] = f"full output [{n}, {WIDTHS[-1]}] of the 3-layer forward"
    res["oracle_seconds"] = round(time.perf_counter() - t0, 1)
    return res, want


def tensor_mode_line(ctx, step, steps, warmup, e, want):
    """The same step with X*W on the tcgen05 tensor cores (3xTF32): time and
    the count of output elements outside the parity bar against the same
    oracle output.  Reported beside the headline, which keeps the parity
    mode."""
    import torch

    ctx.set_math("tensor")
    try:
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            step()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        got = step().cpu().numpy()
    finally:
        ctx.set_math("fast")
    return {"ms_per_step": round(ms, 3), "value": 3 * e / (ms * 1e-3), "unit": UNIT,
            "math": "X*W on tcgen05 (kind::tf32, 3xTF32 split, k-block partials promoted to "
                    "f32 registers); aggregation unchanged",
            "parity": _parity(got, want)}


# ---------------------------------------------------------------------------
# the three small workloads (GCN, GAT, batched GIN): timed on the device,
# checked against the oracle at full size, with the oracle's single-thread
# time (the reference's one JS thread) beside them
# ---------------------------------------------------------------------------
def _time_device(fn, steps, warmup):
    """(ms per call of the CUDA-graph replay, its output, ms per eager call):
    the small workloads are launch-bound, so the forward is captured once
    (browsergnn_b200.CapturedForward) and replayed; the eager time is kept
    for reference."""
    import torch

    import browsergnn_b200 as bg

    def timed(f):
        for _ in range(warmup):
            f()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            out = f()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / steps, out

    eager_ms, _ = timed(fn)
    cap = bg.CapturedForward(fn)
    ms, out = timed(cap)
    out = out.clone()
    cap.close()
    return ms, out, eager_ms


def _parity(got, want):
    g = got.astype(np.float64).ravel()
    w = want.astype(np.float64).ravel()
    err = np.abs(g - w)
    bad = ~((err <= 1e-6 + 1e-5 * np.abs(w)) | (np.isnan(g) & np.isnan(w)))
    return {"max_abs_err": float(np.nanmax(err)) if err.size else 0.0,
            "outside_tolerance": int(bad.sum()), "elements": int(g.size),
            "tolerance": "|gpu-ref| <= 1e-6 + 1e-5|ref|"}


def small_workloads(steps, warmup):
    import browsergnn_b200 as bg
    from browsergnn_b200 import synth
    from oracle import oracle as orc

    res = {}
    rng = np.random.default_rng(7)

    # 1. 2-layer GCN 1433 -> 16 (ReLU) -> 7 on a BA graph, self-loops added
    w = synth.gcn_cora_like()
    n, e = w.num_nodes, w.num_edges
    w1, b1 = synth.glorot(1433, 16, rng), rng.uniform(-0.1, 0.1, 16).astype(np.float32)
    w2, b2 = synth.glorot(16, 7, rng), rng.uniform(-0.1, 0.1, 7).astype(np.float32)
    l1 = bg.GCNConv(inChannels=1433, outChannels=16)
    l1.loadStateDict({"weight": w1, "bias": b1})
    l2 = bg.GCNConv(inChannels=16, outChannels=7)
    l2.loadStateDict({"weight": w2, "bias": b2})
    g = bg.GraphData(x=w.x, numNodes=n, numFeatures=1433, edgeIndex=w.edge_index, numEdges=e)
    gd = g.withFeatures(g.x_device())
    ms, outg, eager_ms = _time_device(lambda: l2.forward(l1.forward(gd, _act="relu")).x, steps,
                                      warmup)
    t0 = time.perf_counter()
    h = orc.relu(orc.gcn_forward(w.x, n, 1433, w.edge_index, e, w1, b1, 16))
    want = orc.gcn_forward(h, n, 16, w.edge_index, e, w2, b2, 7)
    cpu_s = time.perf_counter() - t0
    e_layer = e + (0 if g.hasSelfLoops() else n)
    res["gcn"] = {"workload": w.name, "edges_per_layer": e_layer, "layers": 2, "ms_per_step": ms,
                  "value": 2 * e_layer / (ms * 1e-3), "unit": UNIT,
                  "cpu_oracle_1thread": {"value": 2 * e_layer / cpu_s, "seconds": cpu_s},
                  "eager_ms_per_step": eager_ms, "timing": "CUDA-graph replay of the forward",
                  "parity": _parity(outg.cpu().numpy(), want)}

    # 2. 2-layer GAT 500 -> 8 heads x 8 (ELU) -> 1 x 16 on R-MAT
    w = synth.gat_rmat()
    n, e = w.num_nodes, w.num_edges
    p1 = {"weight": synth.glorot(500, 64, rng),
          "att_src": (0.3 * rng.standard_normal((8, 8))).astype(np.float32),
          "att_dst": (0.3 * rng.standard_normal((8, 8))).astype(np.float32),
          "bias": rng.uniform(-0.1, 0.1, 64).astype(np.float32)}
    p2 = {"weight": synth.glorot(64, 16, rng),
          "att_src": (0.3 * rng.standard_normal((1, 16))).astype(np.float32),
          "att_dst": (0.3 * rng.standard_normal((1, 16))).astype(np.float32),
          "bias": rng.uniform(-0.1, 0.1, 16).astype(np.float32)}
    l1 = bg.GATConv(inChannels=500, outChannels=8, heads=8)
    l1.loadStateDict(p1)
    l2 = bg.GATConv(inChannels=64, outChannels=16, heads=1)
    l2.loadStateDict(p2)
    g = bg.GraphData(x=w.x, numNodes=n, numFeatures=500, edgeIndex=w.edge_index, numEdges=e)
    gd = g.withFeatures(g.x_device())
    ms, outg, eager_ms = _time_device(lambda: l2.forward(l1.forward(gd, _act="elu")).x, steps,
                                      warmup)
    t0 = time.perf_counter()
    h = orc.elu(orc.gat_forward(w.x, n, 500, w.edge_index, e, p1["weight"], p1["att_src"],
                                p1["att_dst"], p1["bias"], 8, 8))
    want = orc.gat_forward(h, n, 64, w.edge_index, e, p2["weight"], p2["att_src"], p2["att_dst"],
                           p2["bias"], 1, 16)
    cpu_s = time.perf_counter() - t0
    e_layer = e + (0 if g.hasSelfLoops() else n)
    res["gat"] = {"workload": w.name, "edges_per_layer": e_layer, "layers": 2, "ms_per_step": ms,
                  "value": 2 * e_layer / (ms * 1e-3), "unit": UNIT,
                  "cpu_oracle_1thread": {"value": 2 * e_layer / cpu_s, "seconds": cpu_s},
                  "eager_ms_per_step": eager_ms, "timing": "CUDA-graph replay of the forward",
                  "parity": _parity(outg.cpu().numpy(), want)}

    # 3. batched GIN: 5 layers (32 -> 64, then 64 -> 64), MLP width 64, eps 0,
    #    ReLU between layers, global sum pool
    w = synth.gin_batch()
    n, e = w.num_nodes, w.num_edges
    widths = [32, 64, 64, 64, 64, 64]
    params, layers = [], []
    for fin, fout in zip(widths[:-1], widths[1:]):
        p = {"epsilon": np.zeros(1, np.float32), "mlp_weight1": synth.glorot(fin, 64, rng),
             "mlp_bias1": rng.uniform(-0.1, 0.1, 64).astype(np.float32),
             "mlp_weight2": synth.glorot(64, fout, rng),
             "mlp_bias2": rng.uniform(-0.1, 0.1, fout).astype(np.float32)}
        lay = bg.GINConv(inChannels=fin, outChannels=fout, hiddenChannels=64)
        lay.loadStateDict(p)
        params.append(p)
        layers.append(lay)
    g = bg.GraphData(x=w.x, numNodes=n, numFeatures=32, edgeIndex=w.edge_index, numEdges=e,
                     batch=w.extra["batch"])
    gd = g.withFeatures(g.x_device())
    ng = w.extra["num_graphs"]

    def gin_step():
        h = gd
        for i, lay in enumerate(layers):
            h = lay.forward(h, _act="relu" if i < len(layers) - 1 else None)
        return bg.global_sum_pool(h, ng)

    ms, pooled, eager_ms = _time_device(gin_step, steps, warmup)
    t0 = time.perf_counter()
    h = w.x
    for i, (p, (fin, fout)) in enumerate(zip(params, zip(widths[:-1], widths[1:]))):
        h = orc.gin_forward(h, n, fin, w.edge_index, e, 0.0, p["mlp_weight1"], p["mlp_bias1"], 64,
                            p["mlp_weight2"], p["mlp_bias2"], fout)
        if i < len(layers) - 1:
            h = orc.relu(h)
    want = orc.sum_pool(h, n, 64, w.extra["batch"], ng)
    cpu_s = time.perf_counter() - t0
    res["gin"] = {"workload": w.name, "edges_per_layer": e, "layers": 5, "ms_per_step": ms,
                  "value": 5 * e / (ms * 1e-3), "unit": UNIT,
                  "cpu_oracle_1thread": {"value": 5 * e / cpu_s, "seconds": cpu_s},
                  "eager_ms_per_step": eager_ms, "timing": "CUDA-graph replay of the forward",
                  "parity": _parity(pooled.cpu().numpy(), want)}
    return res


# ---------------------------------------------------------------------------
# CPU legs: the oracle restatement of the reference CPU path
# ---------------------------------------------------------------------------
def cpu_sample_forward(threads, frac=64, repeats=1):
    """3-layer SAGE forward of the oracle on a 1/frac sample of the workload
    (same degree distribution, widths and weights).  Returns (edges/s, desc)."""
    sys.path.insert(0, ROOT)
    from browsergnn_b200 import synth
    from oracle import oracle as orc

    w = synth.sage_rmat_small(frac)
    weights = make_weights(synth.seed_for(4))
    rp, so, _ = orc.dst_csr(w.edge_index, w.num_edges, w.num_nodes)
    times = []
    for _ in range(repeats):
        h = w.x
        t0 = time.perf_counter()
        for li, (fin, fout) in enumerate(zip(WIDTHS[:-1], WIDTHS[1:])):
            lw = weights[li]
            h = orc.sage_forward_csr(rp, so, w.num_nodes, h, fin, "mean", lw["lin_neighbor"],
                                     lw["lin_self"], lw["bias"], fout, relu=li < 2,
                                     threads=threads)
        times.append(time.perf_counter() - t0)
    t = min(times)
    desc = (f"3-layer SAGE-mean forward of the CPU restatement on a 1/{frac} sample of the "
            f"workload: R-MAT {w.num_nodes} nodes / {w.num_edges} edges, same widths")
    return 3 * w.num_edges / t, desc, w.num_edges, t


def profile_case(kind, math="fast"):
    """Small, self-contained launches for ncu (profiles/ cites these):
    small    : R-MAT 1,000,000 nodes / 25,000,000 edges, F=256: one mean
               aggregation, then one SAGE linear 256 -> 256 (two SGEMM launches)
    full-agg : the benchmark graph (2,450,000 / 62,000,000), F=256 mean
               aggregation twice (capture the second)
    csr      : SparseCSR.fromCOO of the SpMM workload (2^28 entries), twice
    csr-small: SparseCSR.fromCOO of 2^25 entries (scale-21 R-MAT), twice
    linear   : the SAGE pair 256 -> 256 on 1,000,000 rows, three times (pass
               --math tensor for the tcgen05 kernel)
    gat      : the 2-layer GAT workload (20,000 nodes / 200,000 edges), three
               forwards
    spmm-small: the SpMM on a scale-21 R-MAT matrix (2^25 entries) at F = 32,
               64, 128, 256
    giant    : R-MAT scale 20 plus one 1,048,576-edge hub row, F=256 mean
               aggregation twice (the hub row takes k_agg_giant)."""
    import torch

    import browsergnn_b200 as bg
    from browsergnn_b200 import synth
    from browsergnn_b200.backend import ptr
    from browsergnn_b200.graph import DeviceGraph

    bg.init_browsergnn()
    ctx = bg.get_context()
    ctx.set_math(math)
    if kind == "linear":
        # the SAGE pair 256 -> 256 on 1,000,000 rows (2 x 131 GFLOP), three times
        m, k, nn = 1_000_000, 256, 256
        gen = torch.Generator("cuda").manual_seed(3)
        x = torch.randn((m, k), device="cuda", generator=gen)
        agg = torch.randn((m, k), device="cuda", generator=gen)
        ws = torch.randn((k, nn), device="cuda", generator=gen) * 0.06
        wn = torch.randn((k, nn), device="cuda", generator=gen) * 0.06
        b = torch.randn(nn, device="cuda", generator=gen)
        out = torch.empty((m, nn), device="cuda")
        for _ in range(3):
            a0 = torch.cuda.Event(enable_timing=True)
            a1 = torch.cuda.Event(enable_timing=True)
            a0.record()
            ctx.call("bgnn_sage_linear", ptr(agg), ptr(x), ptr(wn), ptr(ws), m, k, nn, ptr(b), 1,
                     0.0, ptr(out))
            a1.record()
            torch.cuda.synchronize()
            ms = a0.elapsed_time(a1)
            print(f"sage_linear ({math}) {m}x{k} -> {nn}: {ms:.3f} ms, "
                  f"{4 * m * k * nn / (ms * 1e-3) / 1e12:.1f} TFLOP/s of the f32 products")
        return
    if kind == "gat":
        # the 2-layer GAT workload (20,000 nodes, 200,000 edges, 500 -> 8x8 ->
        # 16), three forwards
        w = synth.gat_rmat()
        rng = np.random.default_rng(7)
        l1 = bg.GATConv(inChannels=500, outChannels=8, heads=8)
        l1.loadStateDict({"weight": synth.glorot(500, 64, rng),
                          "att_src": (0.3 * rng.standard_normal((8, 8))).astype(np.float32),
                          "att_dst": (0.3 * rng.standard_normal((8, 8))).astype(np.float32),
                          "bias": rng.uniform(-0.1, 0.1, 64).astype(np.float32)})
        l2 = bg.GATConv(inChannels=64, outChannels=16, heads=1)
        l2.loadStateDict({"weight": synth.glorot(64, 16, rng),
                          "att_src": (0.3 * rng.standard_normal((1, 16))).astype(np.float32),
                          "att_dst": (0.3 * rng.standard_normal((1, 16))).astype(np.float32),
                          "bias": rng.uniform(-0.1, 0.1, 16).astype(np.float32)})
        g = bg.GraphData(x=w.x, numNodes=w.num_nodes, numFeatures=500, edgeIndex=w.edge_index,
                         numEdges=w.num_edges)
        for _ in range(3):
            out = l2.forward(l1.forward(g, _act="elu")).x
        torch.cuda.synchronize()
        print(f"GAT forward done, output {tuple(out.shape)}")
        return
    if kind == "giant":
        # R-MAT scale 20 (1,048,576 nodes, 16,777,216 edges) plus one hub row
        # of 1,048,576 edges, F = 256 mean aggregation, twice: the hub row
        # takes the giant-row launch (k_agg_giant)
        scale, n, e0, hub = 20, 1 << 20, 1 << 24, 1 << 20
        ei = synth.rmat_edges_gpu(scale, n, e0, synth.seed_for(4))
        gen = torch.Generator("cuda").manual_seed(5)
        hub_src = torch.randint(0, n, (hub,), device="cuda", generator=gen, dtype=torch.int32)
        src = torch.cat([ei[:e0], hub_src])
        dst = torch.cat([ei[e0:], torch.full((hub,), 7, device="cuda", dtype=torch.int32)])
        e = e0 + hub
        dg = DeviceGraph(torch.cat([src, dst]), e, n, n)
        x = torch.randn((n, 256), device="cuda", generator=gen)
        agg = torch.empty((n, 256), device="cuda")
        for _ in range(2):
            a0 = torch.cuda.Event(enable_timing=True)
            a1 = torch.cuda.Event(enable_timing=True)
            a0.record()
            ctx.call("bgnn_aggregate", dg.h, 1, ptr(x), 256, ptr(agg))
            a1.record()
            torch.cuda.synchronize()
            print(f"aggregate mean F=256, {e} edges with a {hub}-edge hub: "
                  f"{a0.elapsed_time(a1):.3f} ms")
        return
    if kind == "spmm-small":
        # the SpMM sweep on a scale-21 R-MAT matrix (2,097,152 rows, 2^25
        # entries): one launch per width F = 32 / 64 / 128 / 256
        scale = 21
        n, e = 1 << scale, 1 << 25
        ei = synth.rmat_edges_gpu(scale, n, e, synth.seed_for(5))
        vals = torch.rand(e, device="cuda", generator=torch.Generator("cuda").manual_seed(2))
        csr = bg.SparseCSR.fromCOO(bg.SparseCOO(ei[:e], ei[e:], vals, (n, n)))
        del ei
        gen = torch.Generator("cuda").manual_seed(3)
        for f in (32, 64, 128, 256):
            x = torch.randn((n, f), device="cuda", generator=gen)
            a0 = torch.cuda.Event(enable_timing=True)
            a1 = torch.cuda.Event(enable_timing=True)
            a0.record()
            csr.matmul(x)
            a1.record()
            torch.cuda.synchronize()
            print(f"spmm F={f}: {a0.elapsed_time(a1):.3f} ms")
        return
    if kind == "csr-small":
        # SparseCSR.fromCOO of 2^25 entries (scale-21 R-MAT), twice
        scale = 21
        n, e = 1 << scale, 1 << 25
        ei = synth.rmat_edges_gpu(scale, n, e, synth.seed_for(5))
        vals = torch.ones(e, device="cuda")
        for _ in range(2):
            a0 = torch.cuda.Event(enable_timing=True)
            a1 = torch.cuda.Event(enable_timing=True)
            a0.record()
            csr = bg.SparseCSR.fromCOO(bg.SparseCOO(ei[:e], ei[e:], vals, (n, n)))
            a1.record()
            torch.cuda.synchronize()
            print(f"fromCOO {e} entries: {a0.elapsed_time(a1):.3f} ms")
            del csr
        return
    if kind == "csr":
        # SparseCSR.fromCOO of the SpMM workload's 2^28 entries, twice
        n, e = 1 << synth.SPMM_SCALE, synth.SPMM_E
        ei = synth.rmat_edges_gpu(synth.SPMM_SCALE, n, e, synth.seed_for(5))
        vals = torch.ones(e, device="cuda")
        for _ in range(2):
            a0 = torch.cuda.Event(enable_timing=True)
            a1 = torch.cuda.Event(enable_timing=True)
            a0.record()
            csr = bg.SparseCSR.fromCOO(bg.SparseCOO(ei[:e], ei[e:], vals, (n, n)))
            a1.record()
            torch.cuda.synchronize()
            print(f"fromCOO {e} entries: {a0.elapsed_time(a1):.3f} ms")
            del csr
        return
    if kind == "small":
        scale, n, e = 20, 1_000_000, 25_000_000
    else:
        scale, n, e = synth.SAGE_SCALE, synth.SAGE_N, synth.SAGE_E
    f = 256
    ei = synth.rmat_edges_gpu(scale, n, e, synth.seed_for(4))
    dg = DeviceGraph(ei, e, n, n)
    gen = torch.Generator("cuda").manual_seed(1)
    x = torch.randn((n, f), device="cuda", generator=gen)
    agg = torch.empty((n, f), device="cuda")
    reps = 1 if kind == "small" else 2
    for _ in range(reps):
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record()
        ctx.call("bgnn_aggregate", dg.h, 1, ptr(x), f, ptr(agg))
        a1.record()
        torch.cuda.synchronize()
        print(f"aggregate mean F={f} on {n} nodes / {e} edges: {a0.elapsed_time(a1):.3f} ms")
    if kind == "small":
        w1 = torch.randn((f, f), device="cuda", generator=gen) * 0.05
        w2 = torch.randn((f, f), device="cuda", generator=gen) * 0.05
        b = torch.randn(f, device="cuda", generator=gen)
        out = torch.empty((n, f), device="cuda")
        a0.record()
        ctx.call("bgnn_sage_linear", ptr(agg), ptr(x), ptr(w1), ptr(w2), n, f, f, ptr(b), 1, 0.0,
                 ptr(out))
        a1.record()
        torch.cuda.synchronize()
        print(f"sage_linear {n}x{f} -> {f}: {a0.elapsed_time(a1):.3f} ms")


def run_reference(args, rank, world):
    if rank != 0:
        return
    from oracle import oracle as orc

    orc.lib()
    threads = os.cpu_count() or 1
    # each step: the sample forward on all host threads
    for _ in range(args.warmup):
        cpu_sample_forward(threads, repeats=1)
    vals, secs = [], []
    for _ in range(args.steps):
        v, desc, e_s, t = cpu_sample_forward(threads, repeats=3)
        vals.append(v)
        secs.append(t)
    value = statistics.mean(vals)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * statistics.mean(secs), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "sage-mean-3layer-rmat-2450000n-62000000e",
                   "sample": "1/64 of the workload", "threads": threads},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("the reference is TypeScript and no JS runtime exists on this image; the "
                 "reference arm times the C restatement of its CPU path (oracle/)"),
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-spmm", action="store_true")
    ap.add_argument("--no-small", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the full-size output checks (oracle at N=1, N=1 bits at N>1)")
    ap.add_argument("--math", choices=["fast", "tensor"], default="fast",
                    help="fast: X*W on the FP32 pipe in the reference's order (the parity mode); "
                         "tensor: X*W on the tcgen05 tensor cores (3xTF32), with the count of "
                         "elements outside the parity bar reported")
    ap.add_argument("--chunks", type=int, default=None,
                    help="N>1: column chunks of the halo exchange, each aggregated as it lands "
                         "(default 1)")
    ap.add_argument("--row-blocks", type=int, default=-1,
                    help="N>1: row blocks of each layer's last product whose rows are sent to "
                         "the peers as they are written (0: no early sends; default: 4 from 4 "
                         "GPUs up, where the exchange outlasts x*W_self, else none)")
    ap.add_argument("--reserve-sms", type=int, default=16,
                    help="N>1: SMs the aggregation leaves to NCCL while chunks are in flight")
    ap.add_argument("--profile", choices=["small", "full-agg", "csr", "csr-small", "linear", "gat",
                                          "spmm-small", "giant"], default=None,
                    help="run one profiling case for ncu and exit")
    args = ap.parse_args()
    if args.profile:
        profile_case(args.profile, args.math)
        return
    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local = env_int("LOCAL_RANK", 0)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    import browsergnn_b200 as bg
    from browsergnn_b200 import synth
    from browsergnn_b200.backend import ptr

    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        opts = None
        try:  # NCCL kernels on a high-priority stream: the halo exchange runs
            # next to the side-stream GEMM instead of queueing behind its CTAs
            opts = dist.ProcessGroupNCCL.Options()
            opts.is_high_priority_stream = True
        except Exception:  # noqa: BLE001 - older builds: default stream priority
            opts = None
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local}"), pg_options=opts)
    bg.init_browsergnn({"device": local})
    ctx = bg.get_context(local)
    ctx.set_math(args.math)
    hbm_peak, peak_kind = peaks()

    n, e, scale = synth.SAGE_N, synth.SAGE_E, synth.SAGE_SCALE
    seed = synth.seed_for(4)
    ei = synth.rmat_edges_gpu(scale, n, e, seed, device=local)
    gen = torch.Generator("cuda").manual_seed(seed)
    x_full = torch.randn((n, WIDTHS[0]), device="cuda", generator=gen)
    weights = make_weights(seed)
    layers = build_layers(weights, local)

    t0 = time.perf_counter()
    dctx = pgd = None
    if world > 1:
        from browsergnn_b200 import distributed

        distributed.nccl_env_defaults()
        dctx = distributed.DistContext(rank, world, device=local, timeout_ms=120_000)
        if args.chunks is not None:
            dctx.set_pipeline(args.chunks, args.reserve_sms)
        if args.row_blocks < 0:
            # at 2 GPUs x*W_self (3.4 ms at F=256) hides the 1.2 ms exchange and
            # early sends only add contention (25.6 vs 24.9 ms per step); at 8
            # the exchange (1.35 ms) outlasts it (0.9 / 0.3 ms)
            args.row_blocks = 4 if world >= 4 else 0
        if args.row_blocks:
            dctx.set_row_blocks(args.row_blocks)
        torch.cuda.synchronize()
        nccl_init_s = max_over_ranks(time.perf_counter() - t0)
        t0 = time.perf_counter()
        pg = distributed.PartitionedGraph.from_edge_index(ei, e, n, world, rank, device=local)
        ext0 = pg.ext_buffer(WIDTHS[0])
        ext0[: pg.n_own].copy_(x_full[pg.lo:pg.hi])
        pgd = distributed.PartitionedGraphData(pg, dctx, ext0, WIDTHS[0])
        x = ext0[: pg.n_own]
        dg = None
        early = args.row_blocks > 0
        step = lambda timers=None: dist_forward(layers, pgd, timers, early)  # noqa: E731
    else:
        from browsergnn_b200.graph import DeviceGraph

        dg = DeviceGraph(ei, e, n, n, device=local)
        x = x_full
        step = lambda timers=None: sage_forward(layers, dg, x, timers)  # noqa: E731
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    if world > 1:
        build_s = max_over_ranks(build_s)
    del x_full

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    timers = []
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    l0 = ctx.launches
    barrier()
    start.record()
    for _ in range(args.steps):
        step(timers)
    stop.record()
    barrier()
    clocks = sampler.stop()
    launches = (ctx.launches - l0)
    final = step()  # one more untimed forward: the output the parity check reads
    torch.cuda.synchronize()
    ms_total = start.elapsed_time(stop)
    if world > 1:
        ms_total = max_over_ranks(ms_total)
    ms_step = ms_total / args.steps
    value = 3 * e / (ms_step * 1e-3)  # whole-job: all ranks' edges / max time

    # per-layer phases (mean over steps, max over ranks)
    agg_ms = {}
    phases = {}
    for li, fin, a, b, x0, l1 in timers:
        ph = phases.setdefault(li, {})
        if a is not None:
            agg_ms.setdefault((li, fin), []).append(a.elapsed_time(b))
            ph.setdefault("aggregate", []).append(a.elapsed_time(b))
            ph.setdefault("linear", []).append(b.elapsed_time(l1))
        ph.setdefault("layer", []).append(x0.elapsed_time(l1))
    keys = [(li, k) for li in sorted(phases) for k in sorted(phases[li])]
    vec = [statistics.mean(phases[li][k]) for li, k in keys]
    if world > 1:
        vec = max_over_ranks(vec)
    phase_ms = {}
    for (li, k), v in zip(keys, vec):
        phase_ms.setdefault(f"L{li + 1}", {})[k] = round(v, 3)

    roofline = None
    if world == 1:
        # the dominant kernel: the F=256 aggregation (layers 2 and 3)
        f = 256
        bytes_alg = 4 * (n + 1) + 4 * e + 4 * f * e + 4 * f * n
        agg_avg_ms = statistics.mean([m for (li, fin), v in agg_ms.items() if fin == 256
                                      for m in v])
        achieved = bytes_alg / (agg_avg_ms * 1e-3) / 1e9
        traffic, tsrc = profile_traffic("aggregate_mean_f256_sage_rmat")
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
                    "unit": "GB/s", "frac": round(achieved / hbm_peak, 3), "traffic": traffic,
                    "traffic_source": tsrc,
                    "kernel": "aggregate mean F=256 (streaming kernel, one launch)",
                    # the gather model gives no credit for L2 hits, which R-MAT
                    # hubs get: the DRAM bytes ncu counts over the same time
                    "dram_achieved": (round(traffic / (agg_avg_ms * 1e-3) / 1e9, 1)
                                      if traffic else None),
                    "dram_frac": (round(traffic / (agg_avg_ms * 1e-3) / 1e9 / hbm_peak, 3)
                                  if traffic else None),
                    "bytes_model": "gather model: 4(N+1) + 4E + 4FE + 4FN",
                    "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                    "launch_ms": round(agg_avg_ms, 3),
                    "per_layer_aggregate_ms": {f"L{li + 1}_F{fin}": round(statistics.mean(v), 3)
                                               for (li, fin), v in sorted(agg_ms.items())}}

    exchange_only = None
    if world > 1:
        exchange_only = exchange_times(pgd.pg, dctx, max(3, args.steps // 2))
        exchange_only["parts_of_a_layer"] = layer_parts(layers, pgd.pg, dctx,
                                                        max(3, args.steps // 2))

    # e2e through the public API: host features + host edge index each step
    e2e = None
    if not args.no_e2e:
        if world == 1:
            e2e = e2e_single(layers, ei, x, n, e, args.warmup, args.steps)
        else:
            e2e = e2e_partitioned(layers, ei, x, pgd.pg, n, e, dctx, rank, world,
                                  args.warmup, args.steps)

    # parity at full size: N=1 against the oracle (every output element);
    # N>1 bit for bit against a single-GPU forward of the whole graph, which
    # every rank runs on its own GPU for its own rows
    parity = tensor = None
    if not args.no_parity:
        if world == 1:
            parity, want = sage_oracle_parity(ei, n, e, x, weights, final)
            if args.math == "fast":
                tensor = tensor_mode_line(ctx, step, args.steps, args.warmup, e, want)
            del want
        else:
            parity = partition_bit_identity(ei, n, e, seed, layers, pgd.pg, final, local)
    del final

    cpu = None
    if not args.no_cpu and rank == 0 and world == 1:
        threads = os.cpu_count() or 1
        v, desc, _, _ = cpu_sample_forward(threads, repeats=3)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": desc + " (best of 3)"}

    part_info = None
    if world > 1:
        pg = pgd.pg
        lrp = torch.empty(pg.n_own + 1, dtype=torch.int32, device="cuda")
        pg.ctx.call("bgnn_graph_csr", pg.graph, ptr(lrp), None, None)
        part_info = {"rows": pg.n_own, "halo_rows": pg.n_halo, "send_rows": pg.n_send,
                     "local_edges": pg.num_local_edges,
                     "max_row_edges": int((lrp[1:] - lrp[:-1]).max().item()) if pg.n_own else 0}
        del lrp
        allinfo = [None] * world
        dist.all_gather_object(allinfo, part_info)
        part_info = {"per_rank": allinfo,
                     "halo_exchange": "NCCL grouped send/recv of the halo rows (one chunk of "
                                      "columns by default), X*W_self on a side stream "
                                      "meanwhile (browsergnn_b200.distributed)"}
        pgd = None
        pg.close()
    spmm = None
    if not args.no_spmm:
        del dg
        torch.cuda.empty_cache()
        spmm = spmm_sweep(max(3, args.steps // 2), 3, hbm_peak, parity=not args.no_parity,
                          dctx=dctx, rank=rank, world=world)
    small = None
    if not args.no_small and world == 1:
        small = small_workloads(max(3, args.steps), 3)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": "sage-mean-3layer-rmat-2450000n-62000000e",
                       "widths": WIDTHS, "edges_per_layer": e, "layers": 3,
                       "parallelism": f"row-partition x{world}" if world > 1 else "single",
                       "early_send_row_blocks": (args.row_blocks if world > 1 else None),
                       "l2": "inputs larger than L2 (no flush)",
                       "math": ("fast (f32 fma in the reference's order)" if args.math == "fast"
                                else "tensor (X*W on tcgen05, 3xTF32)"),
                       "graph_build_s": round(build_s, 3)},
            "nccl_init_s": round(nccl_init_s, 3) if world > 1 else None,
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "clocks": clocks, "gpu_launches": launches,
            "phase_ms_max_over_ranks": phase_ms,
            "parity": parity,
        }
        if tensor is not None:
            line["tensor_mode"] = tensor
        if part_info is not None:
            line["partition"] = part_info
            line["exchange_only_ms_max_over_ranks"] = exchange_only
        if spmm is not None:
            line["spmm_sweep"] = spmm
        if small is not None:
            line["workloads"] = small
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dctx.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
