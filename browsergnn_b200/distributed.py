"""Multi-GPU message passing: one process per GPU, a row partition of the
graph per rank, NCCL halo exchange over NVLink.

The reference is single-device; this module runs its SAGEConv layer
(src/layers/sage.ts:113-217) and its CSR SpMM (SparseCSR.matmul,
src/core/sparse.ts:322-344) on the GPUs of one node with the same results,
bit for bit, as on one GPU: every row is reduced on one GPU in the
reference's edge order.

    dist = DistContext(rank, world)                 # NCCL communicator
    pg = partition(graph, dist)                     # PartitionedGraphData
    h = sage1.forward(pg, _act="relu")              # SAGEConv on the partition
    out = sage2.forward(h).x                        # this rank's rows [lo, hi)

Each rank passes the full graph; the partition plan (contiguous row ranges,
halo lists, send lists) is derived on the device with no communication
(libbgnn_cuda: bgnn_part_create).  A layer's input lives in an
[owned | halo] buffer whose halo rows the layer fills through NCCL before it
aggregates (bgnn_dist_sage_layer); its output is written straight into the
owned rows of the next layer's buffer.
"""
from __future__ import annotations

import ctypes
import os
from typing import List, Optional, Sequence

import numpy as np

from . import _lib
from .backend import get_context, ptr


def _torch():
    import torch

    return torch


class DistContext:
    """One rank's NCCL communicator (bgnn_dist) on this process's GPU.

    ``unique_id`` is the 128-byte NCCL id made by rank 0
    (``DistContext.make_unique_id()``); when omitted, an initialised
    torch.distributed process group shares it.  ``timeout_ms`` bounds every
    NCCL operation: a peer that fails or never joins turns the next call into
    a ``BGNNError`` with status TIMEOUT instead of a hang."""

    def __init__(self, rank: int, world: int, device: Optional[int] = None,
                 unique_id: Optional[bytes] = None, timeout_ms: int = 120_000,
                 max_ctas: int = 0):
        torch = _torch()
        self.rank, self.world = int(rank), int(world)
        self.ctx = get_context(device)
        self.device = self.ctx.device
        if unique_id is None:
            unique_id = self._shared_unique_id()
        if len(unique_id) != 128:
            raise ValueError("the NCCL unique id has 128 bytes")
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(unique_id)
        h = ctypes.c_void_p()
        torch.cuda.set_device(self.device)
        self.ctx.call("bgnn_dist_create", buf, self.world, self.rank, int(timeout_ms),
                      int(max_ctas), ctypes.byref(h))
        self.h = h

    @staticmethod
    def make_unique_id() -> bytes:
        buf = (ctypes.c_uint8 * 128)()
        _lib.check(_lib.load().bgnn_dist_unique_id(buf))
        return bytes(buf)

    def _shared_unique_id(self) -> bytes:
        import torch.distributed as dist

        if self.world == 1:
            return self.make_unique_id()
        if not dist.is_initialized():
            raise RuntimeError("pass unique_id, or initialise torch.distributed to share it")
        obj = [self.make_unique_id() if self.rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        return obj[0]

    def set_row_blocks(self, blocks: int = 4):
        """Row blocks of a layer's last product whose rows are sent to the
        peers as each is written (sage_forward(send_next=True))."""
        self.ctx.call_on("bgnn_dist_set_row_blocks", self.h, int(blocks))

    def set_pipeline(self, chunks: int = 0, reserve_sms: int = 16):
        """Column chunks of the halo exchange, each aggregated as it lands
        (0: the default, one chunk), and the SMs the aggregation leaves to
        NCCL while later chunks are in flight."""
        self.ctx.call_on("bgnn_dist_set_pipeline", self.h, int(chunks), int(reserve_sms))

    def allreduce_max(self, values: Sequence[float]) -> List[float]:
        arr = (ctypes.c_double * len(values))(*[float(v) for v in values])
        self.ctx.bind()
        _lib.check(self.ctx.lib.bgnn_dist_allreduce_max(self.h, arr, len(values)), self.ctx.h)
        return list(arr)

    def synchronize(self):
        self.ctx.bind()
        _lib.check(self.ctx.lib.bgnn_dist_synchronize(self.h), self.ctx.h)

    def abort(self):
        """Abort the communicator after learning on the host that a peer is
        gone: pending NCCL work ends and close() needs no peer."""
        if getattr(self, "h", None):
            self.ctx.lib.bgnn_dist_abort(self.h)

    def close(self):
        if getattr(self, "h", None):
            self.ctx.lib.bgnn_dist_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PartitionedGraph:
    """One rank's share of a row-partitioned square graph (bgnn_part): rows
    [lo, hi), the local graph over [owned | halo] columns, and the exchange
    plan.  Built from a graph's edge list (rows are destinations, each row's
    edges in COO order) or from a SparseCSR (rows keep their CSR order)."""

    def __init__(self, handle, ctx, world: int, rank: int):
        self.h = handle
        self.ctx = ctx
        self.world, self.rank = int(world), int(rank)
        lo, hi, nh = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
        elo, ne, ns = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        lib = ctx.lib
        _lib.check(lib.bgnn_part_info(handle, ctypes.byref(lo), ctypes.byref(hi), ctypes.byref(nh),
                                      ctypes.byref(elo), ctypes.byref(ne), ctypes.byref(ns)))
        self.lo, self.hi, self.n_halo = lo.value, hi.value, nh.value
        self.n_own = self.hi - self.lo
        self.entry_lo, self.num_local_edges, self.n_send = elo.value, ne.value, ns.value
        b = (ctypes.c_uint32 * (self.world + 1))()
        _lib.check(lib.bgnn_part_bounds(handle, b))
        self.bounds = list(b)
        sc, rc = (ctypes.c_uint64 * self.world)(), (ctypes.c_uint64 * self.world)()
        _lib.check(lib.bgnn_part_counts(handle, sc, rc))
        self.send_counts, self.recv_counts = list(sc), list(rc)
        g = ctypes.c_void_p()
        _lib.check(lib.bgnn_part_graph(handle, ctypes.byref(g)))
        self.graph = g  # owned by the partition

    @classmethod
    def from_edge_index(cls, edge_index, num_edges: int, num_nodes: int, world: int, rank: int,
                        device: Optional[int] = None) -> "PartitionedGraph":
        torch = _torch()
        ctx = get_context(device)
        h = ctypes.c_void_p()
        if isinstance(edge_index, torch.Tensor) and edge_index.is_cuda:
            ei = edge_index.to(torch.int32).contiguous()
            ctx.call("bgnn_part_create", ptr(ei), int(num_edges), int(num_nodes), int(world),
                     int(rank), 0, ctypes.byref(h))
        else:
            if isinstance(edge_index, torch.Tensor):  # host tensor: no copy, keep pinned memory
                ei = edge_index.contiguous().numpy().view(np.uint32)
            else:
                ei = np.ascontiguousarray(np.asarray(edge_index, dtype=np.uint32))
            ctx.call("bgnn_part_create", ei.ctypes.data if ei.size else None, int(num_edges),
                     int(num_nodes), int(world), int(rank), 1, ctypes.byref(h))
        return cls(h, ctx, world, rank)

    @classmethod
    def from_csr(cls, csr, world: int, rank: int) -> "PartitionedGraph":
        """Row partition of a square SparseCSR (values stay with the caller:
        the local entries are values[entry_lo : entry_lo + num_local_edges])."""
        if csr.shape[0] != csr.shape[1]:
            raise ValueError("row partitioning needs a square matrix")
        ctx = get_context(csr.rowPtr.device.index)
        h = ctypes.c_void_p()
        ctx.call("bgnn_part_create_csr", ptr(csr.rowPtr), ptr(csr.colIndices), csr.shape[0],
                 int(world), int(rank), ctypes.byref(h))
        return cls(h, ctx, world, rank)

    def ext_buffer(self, f: int):
        """An [n_own + n_halo, f] float32 buffer for a layer's input."""
        torch = _torch()
        return torch.empty((self.n_own + self.n_halo, int(f)), dtype=torch.float32,
                           device=f"cuda:{self.ctx.device}")

    def lists(self):
        """(halo global ids [n_halo], send rows [n_send]) as int64 CUDA tensors."""
        torch = _torch()
        dev = f"cuda:{self.ctx.device}"
        hid = torch.empty(max(self.n_halo, 1), dtype=torch.int32, device=dev)
        srow = torch.empty(max(self.n_send, 1), dtype=torch.int32, device=dev)
        self.ctx.call("bgnn_part_lists", self.h, ptr(hid), ptr(srow))
        return (hid[: self.n_halo].to(torch.int64) & 0xFFFFFFFF,
                srow[: self.n_send].to(torch.int64) & 0xFFFFFFFF)

    def row_blocks(self, blocks: int):
        """(send_first, recv_first) as [world, blocks + 1] uint64 arrays: where
        each row block starts in each peer's send list and in each owner's
        halo slots (bgnn_part_row_blocks)."""
        w = self.world
        s = (ctypes.c_uint64 * (w * (blocks + 1)))()
        r = (ctypes.c_uint64 * (w * (blocks + 1)))()
        self.ctx.call("bgnn_part_row_blocks", self.h, int(blocks), s, r)
        return (np.ctypeslib.as_array(s).reshape(w, blocks + 1).copy(),
                np.ctypeslib.as_array(r).reshape(w, blocks + 1).copy())

    def aggregate(self, dist: DistContext, x_ext, aggr: str = "mean", out=None):
        """Halo exchange + sum / mean / max aggregation of the owned rows."""
        torch = _torch()
        f = int(x_ext.shape[1])
        if out is None:
            out = torch.empty((self.n_own, f), dtype=torch.float32, device=x_ext.device)
        self.ctx.call_on("bgnn_dist_aggregate", dist.h, self.h, _lib.AGGR[aggr], ptr(x_ext), f,
                         ptr(out))
        return out

    def spmm(self, dist: DistContext, values, x_ext, out=None):
        """The row-partitioned CSR SpMM: values are the whole matrix's values
        (CSR order); the local slice starts at entry_lo."""
        torch = _torch()
        f = int(x_ext.shape[1])
        if out is None:
            out = torch.empty((self.n_own, f), dtype=torch.float32, device=x_ext.device)
        local = values[self.entry_lo:self.entry_lo + self.num_local_edges]
        self.ctx.call_on("bgnn_dist_spmm", dist.h, self.h, ptr(local), ptr(x_ext), f, ptr(out))
        return out

    def close(self):
        if getattr(self, "h", None):
            try:
                _torch().cuda.synchronize(self.ctx.device)
            except Exception:
                pass
            self.ctx.lib.bgnn_part_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PartitionedGraphData:
    """The GraphData a layer sees on one rank of a partitioned graph
    (src/core/graph.ts:43): ``x`` is this rank's rows [lo, hi) (a view of
    the owned rows of the [owned | halo] buffer ``x_ext``)."""

    def __init__(self, pg: PartitionedGraph, dist: DistContext, x_ext, num_features: int):
        self.pg, self.dist = pg, dist
        self.x_ext = x_ext
        self.numFeatures = int(num_features)
        self.numNodes = pg.n_own

    @property
    def x(self):
        return self.x_ext[: self.pg.n_own]

    def withFeatures(self, new_ext) -> "PartitionedGraphData":
        return PartitionedGraphData(self.pg, self.dist, new_ext, int(new_ext.shape[1]))


def partition(graph, dist: DistContext) -> PartitionedGraphData:
    """This rank's share of a GraphData (src/core/graph.ts:43-130): the plan
    from its edge list and its feature rows [lo, hi) in a fresh
    [owned | halo] buffer."""
    pg = PartitionedGraph.from_edge_index(graph.edgeIndex, graph.numEdges, graph.numNodes,
                                          dist.world, dist.rank, device=dist.device)
    x = graph.x_device(dist.device)
    ext = pg.ext_buffer(graph.numFeatures)
    ext[: pg.n_own].copy_(x[pg.lo:pg.hi])
    return PartitionedGraphData(pg, dist, ext, graph.numFeatures)


SEND_OUT = 1  # BGNN_DIST_SEND_OUT


def sage_forward(layer, input: PartitionedGraphData, act=None,
                 send_next: bool = False) -> PartitionedGraphData:
    """SAGEConv.forward (sage.ts:113-217) on one rank of a partitioned graph:
    halo exchange (column chunks pipelined with the aggregation when the
    context asks for them), the root product on a side stream, the fused
    linear writing the owned rows of the next layer's [owned | halo] buffer.

    send_next: another layer reads this one's output, so its halo exchange
    starts while this layer's last product runs (row blocks sent as they are
    written).  Every rank passes the same value.  Layers whose output changes
    after the product (normalize) or that aggregate a projection (pool) send
    nothing early."""
    from .layers import _act_code

    torch = _torch()
    pg, dist = input.pg, input.dist
    k, n = layer.inChannels, layer.outChannels
    if input.numFeatures != k:
        raise ValueError(f"SAGEConv: Expected {k} input channels, got {input.numFeatures}")
    layer.to_device(pg.ctx.device)
    dev = input.x_ext.device
    agg = torch.empty((pg.n_own, k), dtype=torch.float32, device=dev)
    out_ext = pg.ext_buffer(n)
    code, param = _act_code(None if layer.normalize else act)
    w_self = layer.p("lin_self") if layer.rootWeight else None
    if layer.aggregator == "pool":
        # the projection depends only on the source node: project the owned
        # rows, exchange and max-aggregate the projections, then the linear
        # over the layer's own input rows
        from .ops import pool_projection

        proj = pg.ext_buffer(k)
        proj[: pg.n_own].copy_(pool_projection(pg.ctx, input.x, layer.p("pool_weight"),
                                               layer.p("pool_bias")))
        pg.ctx.call_on("bgnn_dist_aggregate", dist.h, pg.h, _lib.AGGR["max"], ptr(proj), k,
                       ptr(agg))
        pg.ctx.call("bgnn_sage_linear", ptr(agg), ptr(input.x_ext), ptr(layer.p("lin_neighbor")),
                    ptr(w_self), pg.n_own, k, n, ptr(layer.p("bias")), code, param, ptr(out_ext))
    else:
        flags = SEND_OUT if send_next and not layer.normalize else 0
        pg.ctx.call_on("bgnn_dist_sage_layer_ex", dist.h, pg.h, _lib.AGGR[layer.aggregator],
                       ptr(input.x_ext), k, n, ptr(layer.p("lin_neighbor")), ptr(w_self),
                       ptr(layer.p("bias")), code, param, ptr(agg), ptr(out_ext), flags)
    if layer.normalize:
        pg.ctx.call("bgnn_l2_normalize_rows", ptr(out_ext), pg.n_own, n)
        if act is not None:
            c2, p2 = _act_code(act)
            pg.ctx.call("bgnn_activation_dev", c2, p2, ptr(out_ext), pg.n_own * n, ptr(out_ext))
    return input.withFeatures(out_ext)


def nccl_env_defaults():
    """NCCL settings for the exchange: NVLS (NVLink SHARP multicast) is not
    needed for point-to-point traffic, and a rank that dies while its memory
    is bound to a multicast object can fault its peers."""
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
