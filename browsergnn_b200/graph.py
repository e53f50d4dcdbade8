"""GraphData: the reference's graph container, with a device-resident CSR.

Mirrors src/core/graph.ts (GraphData, batchGraphs, fromEdgeList): the same
constructor arguments (``x, numNodes, numFeatures, edgeIndex, numEdges``,
optional ``batch``, ``y``, ``graphLabel``), the same validation errors and the
same helpers.  The difference is where the edge structure lives: the first
time a layer needs it, a ``DeviceGraph`` is built once on the GPU (stable
destination CSR, degrees, self-loop flag) and shared by every ``withFeatures``
copy, instead of the reference's O(E) revalidation per layer
(src/core/graph.ts:309-325).
"""
from __future__ import annotations

import ctypes
from typing import List, Optional

import numpy as np

from . import _lib
from .backend import as_device, get_context, ptr


def _torch():
    import torch

    return torch


class DeviceGraph:
    """Owner of a bgnn_graph handle (include/bgnn.h: bgnn_graph_create)."""

    def __init__(self, edge_index, num_edges: int, num_src: int, num_dst: int,
                 device: Optional[int] = None):
        torch = _torch()
        self.ctx = get_context(device)
        self.device = self.ctx.device
        self.num_src, self.num_dst, self.num_edges = int(num_src), int(num_dst), int(num_edges)
        h = ctypes.c_void_p()
        if isinstance(edge_index, torch.Tensor) and edge_index.is_cuda:
            ei = edge_index.to(torch.int32).contiguous()
            self.ctx.call("bgnn_graph_create", ptr(ei), self.num_edges, self.num_src,
                          self.num_dst, 0, ctypes.byref(h))
        else:
            ei = np.ascontiguousarray(np.asarray(edge_index, dtype=np.uint32))
            self.ctx.call("bgnn_graph_create", ei.ctypes.data if ei.size else None,
                          self.num_edges, self.num_src, self.num_dst, 1, ctypes.byref(h))
        self.h = h
        loops = ctypes.c_int()
        _lib.check(self.ctx.lib.bgnn_graph_info(h, None, None, None, ctypes.byref(loops)))
        self.has_self_loops = bool(loops.value)

    @classmethod
    def from_csr(cls, row_ptr, col, num_rows: int, num_cols: int, device: Optional[int] = None):
        """Graph over an existing CSR (device tensors), e.g. from SparseCSR.fromCOO."""
        self = cls.__new__(cls)
        self.ctx = get_context(device)
        self.device = self.ctx.device
        self.num_src, self.num_dst = int(num_cols), int(num_rows)
        h = ctypes.c_void_p()
        self.ctx.call("bgnn_graph_create_csr", ptr(row_ptr), ptr(col), self.num_dst, self.num_src,
                      ctypes.byref(h))
        self.h = h
        ne = ctypes.c_uint64()
        _lib.check(self.ctx.lib.bgnn_graph_info(h, None, None, ctypes.byref(ne), None))
        self.num_edges = int(ne.value)
        self.has_self_loops = False
        return self

    def csr(self):
        """(row_ptr, src_of, edge_id) as int32 CUDA tensors (uint32 bit patterns)."""
        torch = _torch()
        dev = f"cuda:{self.device}"
        rp = torch.empty(self.num_dst + 1, dtype=torch.int32, device=dev)
        so = torch.empty(max(self.num_edges, 1), dtype=torch.int32, device=dev)
        ed = torch.empty(max(self.num_edges, 1), dtype=torch.int32, device=dev)
        self.ctx.call("bgnn_graph_csr", self.h, ptr(rp), ptr(so), ptr(ed))
        return rp, so[: self.num_edges], ed[: self.num_edges]

    def degrees(self):
        torch = _torch()
        dev = f"cuda:{self.device}"
        ind = torch.empty(max(self.num_dst, 1), dtype=torch.int32, device=dev)
        outd = torch.empty(max(self.num_src, 1), dtype=torch.int32, device=dev)
        self.ctx.call("bgnn_graph_degrees", self.h, ptr(ind), ptr(outd))
        return ind[: self.num_dst], outd[: self.num_src]

    def close(self):
        h = getattr(self, "h", None)
        if h:
            try:
                torch = _torch()
                torch.cuda.synchronize(self.device)
            except Exception:
                pass
            self.ctx.lib.bgnn_graph_destroy(h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GraphData:
    """src/core/graph.ts:43-130 (constructor and validation)."""

    def __init__(self, config: Optional[dict] = None, **kw):
        cfg = dict(config or {})
        cfg.update(kw)
        torch = None
        x = cfg["x"]
        n = int(cfg["numNodes"])
        f = int(cfg["numFeatures"])
        e = int(cfg["numEdges"])
        ei = cfg["edgeIndex"]
        self._x_ready = None
        # Pinned host tensors are uploaded without blocking the host: the edge
        # list first on the current stream (the CSR build needs it), then the
        # features on a copy stream, so the copy of x overlaps the CSR build;
        # x_device() makes the consumer's stream wait for it.
        if _is_pinned_host(ei) and _is_pinned_host(x):
            torch = _torch()
            dev = torch.cuda.current_device()
            ei = ei.to(f"cuda:{dev}", non_blocking=True)
            x, self._x_ready = _upload_on_copy_stream(x, dev)
        if _is_cuda_tensor(x):
            torch = _torch()
            xlen = x.numel()
        else:
            x = np.ascontiguousarray(np.asarray(x, dtype=np.float32)).reshape(-1)
            xlen = x.size
        if xlen != n * f:
            raise ValueError(
                f"Node features length {xlen} doesn't match numNodes({n}) * numFeatures({f})")
        self.x = x.reshape(n, f)
        self._x_dev = None       # device copy of a host x (made once)
        self._x_upload = None    # (thread, tensor, status) of an upload in flight
        self.numNodes = n
        self.numFeatures = f
        if _is_cuda_tensor(ei):
            if ei.numel() != 2 * e:
                raise ValueError(f"Edge index length {ei.numel()} doesn't match numEdges({e}) * 2")
            self.edgeIndex = ei.reshape(-1)
            self.numEdges = e
            self._dgraph = cfg.get("_dgraph")
            if self._dgraph is None:
                # device-side validation (graph.ts:88-92) happens in the CSR build
                self._dgraph = DeviceGraph(self.edgeIndex, e, n, n, device=ei.device.index)
        else:
            arr = np.asarray(ei)
            if arr.dtype.kind not in "ui":
                arr = arr.astype(np.int64)
            arr = arr.reshape(-1)
            if arr.size != 2 * e:
                raise ValueError(f"Edge index length {arr.size} doesn't match numEdges({e}) * 2")
            # graph.ts:88-92: the first out-of-range entry in flat order.  Large
            # unsigned lists are checked by the device CSR build instead (the
            # same error, found in the same pass that counts the degrees).
            if arr.dtype.kind == "i" and arr.size and int(arr.min()) < 0:
                bad = np.flatnonzero(arr < 0)
                raise ValueError(f"Edge index {arr[bad[0]]} out of bounds for {n} nodes")
            if arr.size and (arr.size <= _HOST_CHECK_MAX or not _device_present()) and \
                    int(arr.max()) >= n:
                bad = np.flatnonzero(arr >= n)
                raise ValueError(f"Edge index {arr[bad[0]]} out of bounds for {n} nodes")
            self.edgeIndex = np.ascontiguousarray(arr, dtype=np.uint32)
            self.numEdges = e
            self._dgraph = cfg.get("_dgraph")
        self.batch = None if cfg.get("batch") is None else np.asarray(cfg["batch"], np.uint32)
        self.y = cfg.get("y")
        self.graphLabel = cfg.get("graphLabel")
        self.edgeAttr = cfg.get("edgeAttr")
        self.numEdgeFeatures = int(cfg.get("numEdgeFeatures") or 0)

    # ---- device structure ----
    def device_graph(self, device: Optional[int] = None) -> DeviceGraph:
        if self._dgraph is None:
            # a host x starts uploading now, beside the CSR build
            self._start_x_upload(device)
            self._dgraph = DeviceGraph(self.edgeIndex, self.numEdges, self.numNodes, self.numNodes,
                                       device=device)
        return self._dgraph

    def _start_x_upload(self, device: Optional[int]):
        """Upload a host x on a second host thread (the library's staged copy
        releases the interpreter while it runs), so that it overlaps the
        edge list's upload and the CSR build; x_device() waits for it."""
        if not isinstance(self.x, np.ndarray) or self._x_dev is not None or \
                self._x_upload is not None or self.x.size == 0:
            return
        import threading

        torch = _torch()
        ctx = get_context(device)
        arr = np.ascontiguousarray(self.x, dtype=np.float32)
        t = torch.empty(arr.shape, dtype=torch.float32, device=f"cuda:{ctx.device}")
        status = [None]
        ctx.bind()

        def run():
            status[0] = ctx.lib.bgnn_memcpy_h2d(ctx.h, ptr(t), arr.ctypes.data, arr.nbytes)

        th = threading.Thread(target=run, daemon=True)
        th.start()
        self._x_upload = (th, t, status, arr)

    def x_device(self, device: Optional[int] = None):
        torch = _torch()
        if self._x_ready is not None:
            torch.cuda.current_stream().wait_event(self._x_ready)
        if _is_cuda_tensor(self.x) and self.x.dtype == torch.float32:
            return self.x.contiguous()
        if self._x_dev is not None:
            return self._x_dev
        dev = self.device_graph(device).device  # may start the upload
        if self._x_upload is not None:
            th, t, status, _ = self._x_upload
            th.join()
            self._x_upload = None
            _lib.check(status[0], get_context(t.device.index).h)
            self._x_dev = t.reshape(self.numNodes, self.numFeatures)
        else:
            self._x_dev = as_device(self.x, torch.float32, dev).reshape(self.numNodes,
                                                                        self.numFeatures)
        return self._x_dev

    def x_host(self) -> np.ndarray:
        """x as a host float32 array (a layer's output read back through the
        library's staged copy)."""
        if isinstance(self.x, np.ndarray):
            return self.x
        from .backend import to_host

        return to_host(self.x)

    # ---- reference helpers (graph.ts:135-325) ----
    def _host_edges(self) -> np.ndarray:
        if _is_cuda_tensor(self.edgeIndex):
            return self.edgeIndex.cpu().numpy().view(np.uint32)
        return self.edgeIndex

    @property
    def sourceNodes(self) -> np.ndarray:
        return self._host_edges()[: self.numEdges]

    @property
    def targetNodes(self) -> np.ndarray:
        return self._host_edges()[self.numEdges:]

    def getEdge(self, i: int):
        ei = self._host_edges()
        return [int(ei[i]), int(ei[self.numEdges + i])]

    def getInDegrees(self) -> np.ndarray:
        """graph.ts:172-182, computed on the device from the cached CSR."""
        ind, _ = self.device_graph().degrees()
        return ind.cpu().numpy().view(np.uint32)

    def getOutDegrees(self) -> np.ndarray:
        """graph.ts:187-195."""
        _, outd = self.device_graph().degrees()
        return outd.cpu().numpy().view(np.uint32)

    def hasSelfLoops(self) -> bool:
        """graph.ts:220-227 (flag computed during the device CSR build)."""
        return self.device_graph().has_self_loops

    def _x_settled(self):
        """self.x, with any pending upload ordered before the current stream."""
        if self._x_ready is not None:
            _torch().cuda.current_stream().wait_event(self._x_ready)
        return self.x

    def addSelfLoops(self) -> "GraphData":
        """graph.ts:232-272: a loop for every node lacking one, appended after
        the original edges in node order."""
        ei = self._host_edges()
        e, n = self.numEdges, self.numNodes
        src, dst = ei[:e], ei[e:]
        has = np.zeros(n, bool)
        has[src[src == dst]] = True
        add = np.flatnonzero(~has).astype(np.uint32)
        ne = e + add.size
        new = np.concatenate([src, add, dst, add]).astype(np.uint32)
        return GraphData(x=self._x_settled(), numNodes=n, numFeatures=self.numFeatures,
                         edgeIndex=new, numEdges=ne, batch=self.batch, y=self.y,
                         graphLabel=self.graphLabel)

    def removeSelfLoops(self) -> "GraphData":
        """graph.ts:277-304."""
        ei = self._host_edges()
        e = self.numEdges
        keep = ei[:e] != ei[e:]
        new = np.concatenate([ei[:e][keep], ei[e:][keep]])
        return GraphData(x=self._x_settled(), numNodes=self.numNodes,
                         numFeatures=self.numFeatures, edgeIndex=new, numEdges=int(keep.sum()),
                         batch=self.batch, y=self.y, graphLabel=self.graphLabel)

    def withFeatures(self, new_x) -> "GraphData":
        """graph.ts:309-325, sharing the cached device CSR (no revalidation)."""
        rows = new_x.shape[0]
        if rows != self.numNodes:
            raise ValueError(f"New features must have {self.numNodes} nodes")
        g = GraphData.__new__(GraphData)
        g.__dict__.update(self.__dict__)
        g.x = new_x
        g._x_ready = None
        g._x_dev = None
        g._x_upload = None
        g.numFeatures = int(new_x.shape[1])
        return g


_HOST_CHECK_MAX = 1 << 20  # edge-list entries checked on the host when a GPU is present


def _device_present() -> bool:
    try:
        return _torch().cuda.is_available()
    except Exception:  # pragma: no cover
        return False


def _is_pinned_host(a) -> bool:
    try:
        torch = _torch()
    except Exception:  # pragma: no cover
        return False
    return isinstance(a, torch.Tensor) and not a.is_cuda and a.is_pinned()


_copy_streams: dict = {}


def _upload_on_copy_stream(t, device: int):
    """Start an asynchronous host->device copy of a pinned tensor on a side
    stream; returns the device tensor and the event that marks its arrival."""
    torch = _torch()
    s = _copy_streams.get(device)
    if s is None:
        s = torch.cuda.Stream(device=device)
        _copy_streams[device] = s
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        d = t.to(f"cuda:{device}", non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(s)
    d.record_stream(torch.cuda.current_stream(device))
    return d, ev


def _is_cuda_tensor(a) -> bool:
    try:
        import torch

        return isinstance(a, torch.Tensor) and a.is_cuda
    except Exception:  # pragma: no cover
        return False


def batch_graphs(graphs: List[GraphData]) -> GraphData:
    """batchGraphs, src/core/graph.ts:439-492: block-diagonal concatenation,
    edges offset by each graph's node offset, batch[i] = graph id."""
    if not graphs:
        raise ValueError("Cannot batch empty array of graphs")
    f = graphs[0].numFeatures
    for g in graphs:
        if g.numFeatures != f:
            raise ValueError("All graphs must have same number of features")
    xs, srcs, dsts, batch = [], [], [], []
    off = 0
    for gi, g in enumerate(graphs):
        x = g.x.cpu().numpy() if _is_cuda_tensor(g.x) else np.asarray(g.x)
        xs.append(x.reshape(-1))
        ei = g._host_edges()
        srcs.append(ei[: g.numEdges].astype(np.uint32) + np.uint32(off))
        dsts.append(ei[g.numEdges:].astype(np.uint32) + np.uint32(off))
        batch.append(np.full(g.numNodes, gi, np.uint32))
        off += g.numNodes
    e = int(sum(s.size for s in srcs))
    return GraphData(x=np.concatenate(xs), numNodes=off, numFeatures=f,
                     edgeIndex=np.concatenate(srcs + dsts), numEdges=e,
                     batch=np.concatenate(batch))


batchGraphs = batch_graphs


def from_edge_list(edges, num_nodes: Optional[int] = None, node_features=None) -> GraphData:
    """fromEdgeList, src/core/graph.ts:497-531."""
    edges = np.asarray(edges, dtype=np.int64).reshape(-1, 2)
    n = int(num_nodes) if num_nodes is not None else int(edges.max()) + 1
    e = edges.shape[0]
    ei = np.concatenate([edges[:, 0], edges[:, 1]])
    if node_features is None:
        x, f = np.ones(n, np.float32), 1
    else:
        x = np.asarray(node_features, np.float32).reshape(-1)
        f = x.size // n
    return GraphData(x=x, numNodes=n, numFeatures=f, edgeIndex=ei, numEdges=e)


fromEdgeList = from_edge_list
