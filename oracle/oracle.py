"""ctypes front end for the CPU oracle (libbgnn_oracle.so).

TEST INFRASTRUCTURE ONLY: the restatement of BrowserGNN's CPU message-passing
path that the CUDA library is checked against.  Only tests/,
``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference arm import
this module; the product package never does.

Every function takes and returns numpy arrays (float32 features, uint32
indices) and calls the C restatement in ``bgnn_oracle.c``, which cites the
reference function it follows.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libbgnn_oracle.so")
_lib = None

_F = ctypes.POINTER(ctypes.c_float)
_U = ctypes.POINTER(ctypes.c_uint32)
_I64 = ctypes.c_int64


def build() -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(L):
    v = None
    sig = {
        "orc_matmul": (v, [_F, _F, _I64, _I64, _I64, _F]),
        "orc_matmul_par": (v, [_F, _F, _I64, _I64, _I64, ctypes.c_int, _F]),
        "orc_scatter_add": (v, [_F, _U, _I64, _I64, _I64, _F]),
        "orc_scatter_mean": (v, [_F, _U, _I64, _I64, _I64, _F]),
        "orc_scatter_max": (v, [_F, _U, _I64, _I64, _I64, _F]),
        "orc_gather": (v, [_F, _U, _I64, _I64, _F]),
        "orc_relu": (v, [_F, _I64, _F]),
        "orc_add": (v, [_F, _F, _I64, _F]),
        "orc_spmv": (v, [_U, _U, _F, _F, _I64, _F]),
        "orc_spmm": (v, [_U, _U, _F, _F, _I64, _I64, _F]),
        "orc_spmm_rows": (v, [_U, _U, _F, _F, _I64, _U, _I64, ctypes.c_int, _F]),
        "orc_aggregate_backward": (v, [_U, _I64, _I64, _F, _F, _I64, ctypes.c_int, ctypes.c_int,
                                       _F]),
        "orc_matmul_backward": (v, [_F, _F, _F, _I64, _I64, _I64, _F, _F]),
        "orc_bias_backward": (v, [_F, _I64, _I64, _F]),
        "orc_coo_spmm": (v, [_U, _U, _F, _I64, _I64, _F, _I64, _F]),
        "orc_coo_to_csr": (ctypes.c_int, [_U, _U, _F, _I64, _I64, _U, _U, _F]),
        "orc_gcn_norm": (v, [_U, _I64, _I64, ctypes.c_int, _F]),
        "orc_validate_edges": (_I64, [_U, _I64, _I64]),
        "orc_in_degree": (v, [_U, _I64, _I64, _U]),
        "orc_out_degree": (v, [_U, _I64, _I64, _U]),
        "orc_has_self_loops": (ctypes.c_int, [_U, _I64]),
        "orc_add_self_loops": (_I64, [_U, _I64, _I64, _U]),
        "orc_elu": (v, [_F, _I64, ctypes.c_double, _F]),
        "orc_leaky_relu": (v, [_F, _I64, ctypes.c_double, _F]),
        "orc_relu_max": (v, [_F, _I64, _F]),
        "orc_gcn_forward": (ctypes.c_int, [_F, _I64, _I64, _U, _I64, _F, _F, _I64,
                                           ctypes.c_int, ctypes.c_int, _F]),
        "orc_gat_forward": (ctypes.c_int, [_F, _I64, _I64, _U, _I64, _F, _F, _F, _F, _I64,
                                           _I64, ctypes.c_double, ctypes.c_int, ctypes.c_int,
                                           _F]),
        "orc_sage_forward": (ctypes.c_int, [_F, _I64, _I64, _U, _I64, ctypes.c_int, _F, _F, _F,
                                            _F, _F, _I64, ctypes.c_int, _F]),
        "orc_gin_forward": (ctypes.c_int, [_F, _I64, _I64, _U, _I64, ctypes.c_float, _F, _F,
                                           _I64, _F, _F, _I64, _F]),
        "orc_sum_pool": (v, [_F, _I64, _I64, _U, _I64, _F]),
        "orc_dst_csr": (ctypes.c_int, [_U, _I64, _I64, _U, _U, _U]),
        "orc_csr_aggregate": (v, [_U, _U, _I64, _F, _I64, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, _F]),
        "orc_sage_forward_csr": (ctypes.c_int, [_U, _U, _I64, _F, _I64, ctypes.c_int, _F, _F,
                                                _F, _I64, ctypes.c_int, ctypes.c_int, _F]),
        "orc_linear": (v, [_F, _I64, _I64, _F, _F, _I64, _F]),
        "orc_gat_forward_train": (ctypes.c_int, [_F, _I64, _I64, _U, _I64, _F, _F, _F, _F, _I64,
                                                 _I64, ctypes.c_double, ctypes.c_int,
                                                 ctypes.c_int, ctypes.c_double, ctypes.c_uint64,
                                                 _F]),
        "orc_sigmoid": (v, [_F, _I64, _F]),
        "orc_tanh": (v, [_F, _I64, _F]),
        "orc_gelu": (v, [_F, _I64, _F]),
        "orc_silu": (v, [_F, _I64, _F]),
        "orc_prelu": (v, [_F, _I64, _F, _I64, _F]),
        "orc_softmax_rows": (v, [_F, _I64, _I64, ctypes.POINTER(ctypes.c_uint8), ctypes.c_float,
                                 ctypes.c_int, _F]),
        "orc_uniform": (ctypes.c_double, [ctypes.c_uint64, ctypes.c_uint64]),
        "orc_dropout": (v, [_F, _I64, ctypes.c_double, ctypes.c_uint64, _F]),
        "orc_link_scores": (v, [_F, _I64, _U, _U, _I64, ctypes.c_int, _F, _F, _F, _F, _F,
                                ctypes.POINTER(ctypes.c_double)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _f(a):
    if a is None:
        return None
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a


def _u(a):
    return np.ascontiguousarray(a, dtype=np.uint32)


def _pf(a):
    return None if a is None else a.ctypes.data_as(_F)


def _pu(a):
    return None if a is None else a.ctypes.data_as(_U)


# ---- src/backend/wasm/index.ts ---------------------------------------------
def matmul(a, b, m, k, n, threads=1):
    a, b = _f(a), _f(b)
    out = np.empty(m * n, np.float32)
    if threads == 1:
        lib().orc_matmul(_pf(a), _pf(b), m, k, n, _pf(out))
    else:
        lib().orc_matmul_par(_pf(a), _pf(b), m, k, n, threads, _pf(out))
    return out


def _scatter(name, src, index, num_nodes, nf):
    src, index = _f(src), _u(index)
    out = np.empty(num_nodes * nf, np.float32)
    getattr(lib(), name)(_pf(src), _pu(index), index.size, num_nodes, nf, _pf(out))
    return out


def scatter_add(src, index, num_nodes, nf):
    return _scatter("orc_scatter_add", src, index, num_nodes, nf)


def scatter_mean(src, index, num_nodes, nf):
    return _scatter("orc_scatter_mean", src, index, num_nodes, nf)


def scatter_max(src, index, num_nodes, nf):
    return _scatter("orc_scatter_max", src, index, num_nodes, nf)


def gather(src, index, nf):
    src, index = _f(src), _u(index)
    out = np.empty(index.size * nf, np.float32)
    lib().orc_gather(_pf(src), _pu(index), index.size, nf, _pf(out))
    return out


def relu(x):
    x = _f(x)
    out = np.empty_like(x)
    lib().orc_relu(_pf(x), x.size, _pf(out))
    return out


def relu_max(x):
    x = _f(x)
    out = np.empty_like(x)
    lib().orc_relu_max(_pf(x), x.size, _pf(out))
    return out


def elu(x, alpha=1.0):
    x = _f(x)
    out = np.empty_like(x)
    lib().orc_elu(_pf(x), x.size, alpha, _pf(out))
    return out


def leaky_relu(x, slope=0.01):
    x = _f(x)
    out = np.empty_like(x)
    lib().orc_leaky_relu(_pf(x), x.size, slope, _pf(out))
    return out


def add(a, b):
    a, b = _f(a), _f(b)
    out = np.empty_like(a)
    lib().orc_add(_pf(a), _pf(b), a.size, _pf(out))
    return out


def spmv(row_ptr, col, val, x, num_rows):
    row_ptr, col, val, x = _u(row_ptr), _u(col), _f(val), _f(x)
    out = np.empty(num_rows, np.float32)
    lib().orc_spmv(_pu(row_ptr), _pu(col), _pf(val), _pf(x), num_rows, _pf(out))
    return out


def spmm(row_ptr, col, val, dense, num_rows, nf):
    row_ptr, col, val, dense = _u(row_ptr), _u(col), _f(val), _f(dense)
    out = np.empty(num_rows * nf, np.float32)
    lib().orc_spmm(_pu(row_ptr), _pu(col), _pf(val), _pf(dense), num_rows, nf, _pf(out))
    return out


def spmm_rows(row_ptr, col, val, dense, nf, rows=None, num_rows=None, threads=0):
    """wasmSpmm for the listed rows (all rows when rows is None), row-parallel
    on `threads` host threads (0: all); [len(rows), nf] in list order."""
    row_ptr, col, val, dense = _u(row_ptr), _u(col), _f(val), _f(dense)
    if rows is None:
        nrows = int(num_rows if num_rows is not None else row_ptr.size - 1)
        rp = None
    else:
        rows = _u(rows)
        nrows = int(rows.size)
        rp = _pu(rows)
    out = np.empty(max(nrows * nf, 1), np.float32)
    lib().orc_spmm_rows(_pu(row_ptr), _pu(col), _pf(val), _pf(dense), nf, rp, nrows, threads,
                        _pf(out))
    return out[: nrows * nf]


def coo_spmm(rows, cols, vals, m, dense, k):
    rows, cols, vals, dense = _u(rows), _u(cols), _f(vals), _f(dense)
    out = np.empty(m * k, np.float32)
    lib().orc_coo_spmm(_pu(rows), _pu(cols), _pf(vals), rows.size, m, _pf(dense), k, _pf(out))
    return out


# ---- src/core/sparse.ts / graph.ts ------------------------------------------
def coo_to_csr(rows, cols, vals, num_rows):
    rows, cols = _u(rows), _u(cols)
    vals = None if vals is None else _f(vals)
    nnz = rows.size
    row_ptr = np.empty(num_rows + 1, np.uint32)
    col_out = np.empty(max(nnz, 1), np.uint32)
    val_out = np.empty(max(nnz, 1), np.float32)
    rc = lib().orc_coo_to_csr(_pu(rows), _pu(cols), _pf(vals), nnz, num_rows, _pu(row_ptr),
                              _pu(col_out), _pf(val_out))
    if rc != 0:
        raise ValueError(f"orc_coo_to_csr failed ({rc})")
    return row_ptr, col_out[:nnz], val_out[:nnz]


def gcn_norm(edge_index, num_edges, num_nodes, add_self_loops=True):
    ei = _u(edge_index)
    out = np.empty(num_edges, np.float32)
    lib().orc_gcn_norm(_pu(ei), num_edges, num_nodes, int(add_self_loops), _pf(out))
    return out


def validate_edges(edge_index, num_edges, num_nodes):
    ei = _u(edge_index)
    return int(lib().orc_validate_edges(_pu(ei), num_edges, num_nodes))


def in_degree(edge_index, num_edges, num_nodes):
    ei = _u(edge_index)
    out = np.empty(num_nodes, np.uint32)
    lib().orc_in_degree(_pu(ei), num_edges, num_nodes, _pu(out))
    return out


def out_degree(edge_index, num_edges, num_nodes):
    ei = _u(edge_index)
    out = np.empty(num_nodes, np.uint32)
    lib().orc_out_degree(_pu(ei), num_edges, num_nodes, _pu(out))
    return out


def has_self_loops(edge_index, num_edges):
    return bool(lib().orc_has_self_loops(_pu(_u(edge_index)), num_edges))


def add_self_loops(edge_index, num_edges, num_nodes):
    ei = _u(edge_index)
    out = np.empty(2 * (num_edges + num_nodes), np.uint32)
    ne = int(lib().orc_add_self_loops(_pu(ei), num_edges, num_nodes, _pu(out)))
    return out[:2 * ne], ne


# ---- layer forwards (src/layers) ---------------------------------------------
def gcn_forward(x, n, fin, edge_index, num_edges, weight, bias, fout, add_self_loops=True,
                normalize=True):
    out = np.empty(n * fout, np.float32)
    rc = lib().orc_gcn_forward(_pf(_f(x)), n, fin, _pu(_u(edge_index)), num_edges,
                               _pf(_f(weight)), _pf(_f(bias)), fout, int(add_self_loops),
                               int(normalize), _pf(out))
    assert rc == 0
    return out


def gat_forward(x, n, fin, edge_index, num_edges, weight, att_src, att_dst, bias, heads, c,
                negative_slope=0.2, concat=True, add_self_loops=True, dropout=0.0, seed=0):
    od = heads * c if concat else c
    out = np.empty(n * od, np.float32)
    rc = lib().orc_gat_forward_train(_pf(_f(x)), n, fin, _pu(_u(edge_index)), num_edges,
                                     _pf(_f(weight)), _pf(_f(att_src)), _pf(_f(att_dst)),
                                     _pf(_f(bias)), heads, c, float(negative_slope), int(concat),
                                     int(add_self_loops), float(dropout),
                                     int(seed) & (2 ** 64 - 1), _pf(out))
    assert rc == 0
    return out


SAGE_AGGR = {"mean": 0, "max": 1, "sum": 2, "pool": 3}


def sage_forward(x, n, fin, edge_index, num_edges, aggr, lin_neighbor, lin_self, bias, fout,
                 normalize=False, pool_weight=None, pool_bias=None):
    out = np.empty(n * fout, np.float32)
    rc = lib().orc_sage_forward(_pf(_f(x)), n, fin, _pu(_u(edge_index)), num_edges,
                                SAGE_AGGR[aggr], _pf(_f(lin_neighbor)), _pf(_f(lin_self)),
                                _pf(_f(bias)), _pf(_f(pool_weight)), _pf(_f(pool_bias)), fout,
                                int(normalize), _pf(out))
    assert rc == 0
    return out


def gin_forward(x, n, fin, edge_index, num_edges, eps, w1, b1, hidden, w2, b2, fout):
    out = np.empty(n * fout, np.float32)
    rc = lib().orc_gin_forward(_pf(_f(x)), n, fin, _pu(_u(edge_index)), num_edges,
                               float(eps), _pf(_f(w1)), _pf(_f(b1)), hidden, _pf(_f(w2)),
                               _pf(_f(b2)), fout, _pf(out))
    assert rc == 0
    return out


def sum_pool(x, n, f, batch, num_graphs):
    out = np.empty(num_graphs * f, np.float32)
    lib().orc_sum_pool(_pf(_f(x)), n, f, _pu(_u(batch)), num_graphs, _pf(out))
    return out


# ---- streamed / row-parallel -------------------------------------------------
def dst_csr(edge_index, num_edges, num_nodes):
    ei = _u(edge_index)
    row_ptr = np.empty(num_nodes + 1, np.uint32)
    src_of = np.empty(max(num_edges, 1), np.uint32)
    eid = np.empty(max(num_edges, 1), np.uint32)
    rc = lib().orc_dst_csr(_pu(ei), num_edges, num_nodes, _pu(row_ptr), _pu(src_of), _pu(eid))
    assert rc == 0
    return row_ptr, src_of[:num_edges], eid[:num_edges]


AGG_OPS = {"sum": 0, "mean": 1, "max": 2, "gcn": 3}


def csr_aggregate(row_ptr, src_of, num_rows, x, f, op, self_loop_tail=False, threads=0):
    out = np.empty(num_rows * f, np.float32)
    lib().orc_csr_aggregate(_pu(_u(row_ptr)), _pu(_u(src_of)), num_rows, _pf(_f(x)), f,
                            AGG_OPS[op], int(self_loop_tail), threads, _pf(out))
    return out


def sage_forward_csr(row_ptr, src_of, n, x, fin, aggr, lin_neighbor, lin_self, bias, fout,
                     relu=False, threads=0):
    out = np.empty(n * fout, np.float32)
    rc = lib().orc_sage_forward_csr(_pu(_u(row_ptr)), _pu(_u(src_of)), n, _pf(_f(x)), fin,
                                    SAGE_AGGR[aggr], _pf(_f(lin_neighbor)), _pf(_f(lin_self)),
                                    _pf(_f(bias)), fout, int(relu), threads, _pf(out))
    assert rc == 0
    return out


# ---- backward --------------------------------------------------------------
BACKWARD_OPS = {"sum": 0, "mean": 1, "max": 2, "gcn": 3}


def aggregate_backward(edge_index, num_edges, num_nodes, grad, f, op, x=None, tail=False):
    """Gradient for the source rows of sum / mean / max / gcn aggregation
    (the edge-ordered scatter of gradient messages); x is the forward input
    (needed for max)."""
    out = np.empty(num_nodes * f, np.float32)
    xx = _f(x) if x is not None else np.zeros(1, np.float32)
    lib().orc_aggregate_backward(_pu(_u(edge_index)), num_edges, num_nodes, _pf(xx),
                                 _pf(_f(grad)), f, BACKWARD_OPS[op], int(tail), _pf(out))
    return out


def matmul_backward(a, b, grad, m, k, n):
    """(grad_a [m, k], grad_b [k, n]) of Variable.matmul (variable.ts:213-235)."""
    ga = np.empty(m * k, np.float32)
    gb = np.empty(k * n, np.float32)
    lib().orc_matmul_backward(_pf(_f(a)), _pf(_f(b)), _pf(_f(grad)), m, k, n, _pf(ga), _pf(gb))
    return ga, gb


def bias_backward(grad, rows, cols):
    out = np.empty(cols, np.float32)
    lib().orc_bias_backward(_pf(_f(grad)), rows, cols, _pf(out))
    return out


# ---- model zoo: src/nn/linear.ts, src/nn/activation.ts, src/core/tensor.ts ----
def linear(x, w, b=None):
    """Linear.forward (src/nn/linear.ts:50-111); x [m, k], w [n, k]."""
    x = _f(x)
    w = _f(w)
    n, k = w.shape
    m = x.size // k
    out = np.empty((m, n), np.float32)
    lib().orc_linear(_pf(x), m, k, _pf(w), _pf(_f(b)), n, _pf(out))
    return out


def _unary(name, x):
    x = _f(x)
    out = np.empty_like(x)
    getattr(lib(), name)(_pf(x), x.size, _pf(out))
    return out


def sigmoid(x):
    return _unary("orc_sigmoid", x)


def tanh(x):
    return _unary("orc_tanh", x)


def gelu(x):
    return _unary("orc_gelu", x)


def silu(x):
    return _unary("orc_silu", x)


def prelu(x, w):
    x, w = _f(x), _f(w)
    out = np.empty_like(x)
    lib().orc_prelu(_pf(x), x.size, _pf(w), w.size, _pf(out))
    return out


def softmax_rows(x, col_mask=None, mask_value=-1e9, log=False):
    """Tensor.softmax / logSoftmax of a 2-D array (src/core/tensor.ts:435-499)."""
    x = _f(x)
    rows, cols = x.shape
    out = np.empty_like(x)
    m = None
    if col_mask is not None:
        m = np.ascontiguousarray(col_mask, dtype=np.uint8)
    lib().orc_softmax_rows(_pf(x), rows, cols,
                           None if m is None else m.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
                           float(mask_value), int(bool(log)), _pf(out))
    return out


def uniform(seed, i):
    return float(lib().orc_uniform(int(seed) & (2 ** 64 - 1), int(i)))


def dropout(x, p, seed):
    x = _f(x)
    out = np.empty_like(x)
    lib().orc_dropout(_pf(x), x.size, float(p), int(seed) & (2 ** 64 - 1), _pf(out))
    return out


LINK_MODES = {"dot": 0, "bilinear": 1, "mlp": 2}


def link_scores(emb, src, tgt, mode, w_bilinear=None, w1=None, b1=None, w2=None, b2=None):
    """ConceptPrerequisiteMapper.predictLinks (ConceptPrerequisiteMapper.ts:224-295)."""
    emb = _f(emb)
    d = emb.shape[1]
    src, tgt = _u(src), _u(tgt)
    out = np.empty(src.size, np.float64)
    lib().orc_link_scores(_pf(emb), d, _pu(src), _pu(tgt), src.size, LINK_MODES[mode],
                          _pf(_f(w_bilinear)), _pf(_f(w1)), _pf(_f(b1)), _pf(_f(w2)),
                          _pf(_f(b2)), out.ctypes.data_as(ctypes.POINTER(ctypes.c_double)))
    return out
