"""Device-tensor mirrors of the reference's sparse core and GPU facade.

  SparseCOO / SparseCSR          src/core/sparse.ts:22-383
  MessagePassing                 src/core/sparse.ts:389-474
  computeGCNNorm                 src/core/sparse.ts:480-513
  GPUSparse / GPUTensor          src/core/gpu-sparse.ts:19-285

Tensors are CUDA float32 (features) and int32 holding uint32 bit patterns
(indices).  Every method runs on libbgnn_cuda; nothing falls back to the CPU.
"""
from __future__ import annotations

from typing import Optional, Tuple

import numpy as np

from . import _lib
from .backend import as_device, get_context, ptr


def _torch():
    import torch

    return torch


def _dev_of(t) -> int:
    return t.device.index if t.device.index is not None else 0


def _idx(a, device):
    return as_device(a, _torch().int32, device)


def _f32(a, device):
    return as_device(a, _torch().float32, device)


def pool_projection(ctx, x, w, b):
    torch = _torch()
    m, k = x.shape
    out = torch.empty((m, k), dtype=torch.float32, device=x.device)
    ctx.call("bgnn_pool_projection", ptr(x), ptr(w), ptr(b), m, k, ptr(out))
    return out


class SparseCOO:
    """src/core/sparse.ts:22-230 (device arrays)."""

    def __init__(self, rows, cols, values, shape: Tuple[int, int], device: int = 0):
        self.rows = _idx(rows, device)
        self.cols = _idx(cols, device)
        self.values = _f32(values, device)
        self.shape = (int(shape[0]), int(shape[1]))
        self.nnz = int(self.values.numel())
        if self.rows.numel() != self.nnz or self.cols.numel() != self.nnz:
            raise ValueError("Row, column, and value arrays must have same length")

    @staticmethod
    def fromEdgeIndex(edge_index, num_edges: int, num_nodes: int, values=None, device: int = 0):
        """sparse.ts:81-92: rows = sources, cols = targets, values default 1."""
        torch = _torch()
        ei = _idx(edge_index, device)
        vals = values if values is not None else torch.ones(num_edges, dtype=torch.float32,
                                                           device=ei.device)
        return SparseCOO(ei[:num_edges], ei[num_edges:], vals, (num_nodes, num_nodes), device)

    def toCSR(self) -> "SparseCSR":
        return SparseCSR.fromCOO(self)


class SparseCSR:
    """src/core/sparse.ts:236-383 (device arrays)."""

    def __init__(self, rowPtr, colIndices, values, shape: Tuple[int, int]):
        self.rowPtr = rowPtr
        self.colIndices = colIndices
        self.values = values
        self.shape = (int(shape[0]), int(shape[1]))
        self.nnz = int(values.numel())
        self._graph = None

    @staticmethod
    def fromCOO(coo: SparseCOO) -> "SparseCSR":
        """Stable sort by (row, col) on the device (bit-exact with sparse.ts:259-296)."""
        torch = _torch()
        dev = _dev_of(coo.rows)
        ctx = get_context(dev)
        m, n = coo.shape
        rp = torch.empty(m + 1, dtype=torch.int32, device=coo.rows.device)
        ci = torch.empty(max(coo.nnz, 1), dtype=torch.int32, device=coo.rows.device)
        va = torch.empty(max(coo.nnz, 1), dtype=torch.float32, device=coo.rows.device)
        ctx.call("bgnn_coo_to_csr_dev", ptr(coo.rows), ptr(coo.cols), ptr(coo.values), coo.nnz,
                 m, n, ptr(rp), ptr(ci), ptr(va))
        return SparseCSR(rp, ci[: coo.nnz], va[: coo.nnz], coo.shape)

    def graph(self):
        """Cached device graph over this CSR (heavy-row schedule computed once)."""
        if self._graph is None:
            from .graph import DeviceGraph

            self._graph = DeviceGraph.from_csr(self.rowPtr, self.colIndices, self.shape[0],
                                               self.shape[1], device=_dev_of(self.rowPtr))
        return self._graph

    def matmul(self, dense):
        """CSR SpMM (sparse.ts:322-344 / wasmSpmm index.ts:342-383)."""
        torch = _torch()
        if dense.dim() != 2 or dense.shape[0] != self.shape[1]:
            raise ValueError(f"Shape mismatch: sparse {list(self.shape)} @ dense {list(dense.shape)}")
        g = self.graph()
        f = int(dense.shape[1])
        out = torch.empty((self.shape[0], f), dtype=torch.float32, device=dense.device)
        g.ctx.call("bgnn_graph_spmm", g.h, ptr(self.values), ptr(dense.contiguous()), f, ptr(out))
        return out

    def matvec(self, x):
        """SparseCSR.matvec / wasmSpmv (f64 accumulator)."""
        torch = _torch()
        ctx = get_context(_dev_of(self.rowPtr))
        out = torch.empty(self.shape[0], dtype=torch.float32, device=x.device)
        ctx.call("bgnn_spmv_dev", ptr(self.rowPtr), ptr(self.colIndices), ptr(self.values),
                 ptr(x.contiguous()), self.shape[0], self.shape[1], ptr(out))
        return out


class MessagePassing:
    """src/core/sparse.ts:389-474 on device tensors (edge-order semantics)."""

    @staticmethod
    def _scatter(aggr, src, index, numNodes):
        torch = _torch()
        if src.dim() != 2:
            raise ValueError("Source must be 2D tensor")
        idx = _idx(index, _dev_of(src))
        if aggr != "max" and src.shape[0] != idx.numel():
            raise ValueError("Source rows must match index length")
        ctx = get_context(_dev_of(src))
        f = int(src.shape[1])
        out = torch.empty((int(numNodes), f), dtype=torch.float32, device=src.device)
        ctx.call("bgnn_scatter_dev", _lib.AGGR[aggr], ptr(src.contiguous()), ptr(idx),
                 idx.numel(), int(numNodes), f, ptr(out))
        return out

    @staticmethod
    def scatterAdd(src, index, numNodes):
        return MessagePassing._scatter("sum", src, index, numNodes)

    @staticmethod
    def scatterMean(src, index, numNodes):
        return MessagePassing._scatter("mean", src, index, numNodes)

    @staticmethod
    def scatterMax(src, index, numNodes):
        return MessagePassing._scatter("max", src, index, numNodes)

    @staticmethod
    def gather(src, index):
        torch = _torch()
        if src.dim() != 2:
            raise ValueError("Source must be 2D tensor")
        idx = _idx(index, _dev_of(src))
        ctx = get_context(_dev_of(src))
        f = int(src.shape[1])
        out = torch.empty((idx.numel(), f), dtype=torch.float32, device=src.device)
        ctx.call("bgnn_gather_dev", ptr(src.contiguous()), int(src.shape[0]), ptr(idx),
                 idx.numel(), f, ptr(out))
        return out


def compute_gcn_norm(edge_index, num_edges: int, num_nodes: int, add_self_loops: bool = True,
                     device: Optional[int] = None):
    """computeGCNNorm (sparse.ts:480-513) on the device."""
    torch = _torch()
    ctx = get_context(device)
    ei = _idx(edge_index, ctx.device)
    out = torch.empty(max(num_edges, 1), dtype=torch.float32, device=ei.device)
    ctx.call("bgnn_gcn_norm_dev", ptr(ei), num_edges, num_nodes, int(add_self_loops), ptr(out))
    return out[:num_edges]


computeGCNNorm = compute_gcn_norm


class GPUSparse:
    """src/core/gpu-sparse.ts:19-186: the same static methods, always on CUDA."""

    @staticmethod
    def matmul(sparse, dense):
        csr = sparse if isinstance(sparse, SparseCSR) else sparse.toCSR()
        return csr.matmul(dense)

    scatterAdd = staticmethod(MessagePassing.scatterAdd)
    scatterMean = staticmethod(MessagePassing.scatterMean)
    scatterMax = staticmethod(MessagePassing.scatterMax)
    gather = staticmethod(MessagePassing.gather)


class GPUTensor:
    """src/core/gpu-sparse.ts:192-278."""

    @staticmethod
    def matmul(a, b):
        torch = _torch()
        if a.dim() != 2 or b.dim() != 2:
            raise ValueError("Both tensors must be 2D")
        if a.shape[1] != b.shape[0]:
            raise ValueError(f"Shape mismatch: {list(a.shape)} @ {list(b.shape)}")
        ctx = get_context(_dev_of(a))
        m, k = a.shape
        n = b.shape[1]
        out = torch.empty((m, n), dtype=torch.float32, device=a.device)
        ctx.call("bgnn_matmul_dev", ptr(a.contiguous()), ptr(b.contiguous()), m, k, n, ptr(out))
        return out

    @staticmethod
    def relu(x):
        torch = _torch()
        ctx = get_context(_dev_of(x))
        out = torch.empty_like(x)
        ctx.call("bgnn_activation_dev", _lib.ACT["relu"], 0.0, ptr(x.contiguous()), x.numel(),
                 ptr(out))
        return out

    @staticmethod
    def add(a, b):
        torch = _torch()
        if a.numel() != b.numel():
            raise ValueError(f"Size mismatch: {a.numel()} vs {b.numel()}")
        ctx = get_context(_dev_of(a))
        out = torch.empty_like(a)
        ctx.call("bgnn_add_dev", ptr(a.contiguous()), ptr(b.contiguous()), a.numel(), ptr(out))
        return out
