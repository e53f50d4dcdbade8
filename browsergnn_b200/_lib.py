"""ctypes binding of libbgnn_cuda.so (include/bgnn.h).

The library is the only compute path: if it is missing or no CUDA device is
present, every operation raises -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libbgnn_cuda.so")

# bgnn_status
OK, ERR_INVALID_ARG, ERR_OUT_OF_RANGE, ERR_CUDA, ERR_NO_MEMORY, ERR_TIMEOUT, ERR_UNSUPPORTED, \
    ERR_DEVICE = range(8)
MATH_FAST, MATH_EXACT, MATH_TENSOR = 0, 1, 2
AGGR = {"sum": 0, "add": 0, "mean": 1, "max": 2}
AGGR_SPMM = 3
ACT = {None: 0, "none": 0, "relu": 1, "relu_max": 2, "elu": 3, "leaky_relu": 4, "sigmoid": 5,
       "tanh": 6, "gelu": 7, "silu": 8}
LINK = {"dot": 0, "bilinear": 1, "mlp": 2}

STATUS_NAMES = {
    OK: "OK", ERR_INVALID_ARG: "INVALID_ARG", ERR_OUT_OF_RANGE: "OUT_OF_RANGE", ERR_CUDA: "CUDA",
    ERR_NO_MEMORY: "NO_MEMORY", ERR_TIMEOUT: "TIMEOUT", ERR_UNSUPPORTED: "UNSUPPORTED",
    ERR_DEVICE: "DEVICE",
}


class BGNNError(RuntimeError):
    """A non-OK status returned by libbgnn_cuda."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{STATUS_NAMES.get(status, status)}] {message}")
        self.status = status


class BGNNIndexError(BGNNError, ValueError):
    """An index out of range (the reference throws an Error from GraphData)."""


_P = ctypes.c_void_p
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64
_I = ctypes.c_int
_D = ctypes.c_double
_F = ctypes.c_float

# name -> argtypes (all return int unless listed in _RESTYPE)
SIGNATURES = {
    "bgnn_abi_version": [],
    "bgnn_ctx_create": [_I, ctypes.POINTER(_P)],
    "bgnn_ctx_destroy": [_P],
    "bgnn_ctx_set_stream": [_P, _P],
    "bgnn_ctx_set_sm_budget": [_P, _U32],
    "bgnn_ctx_set_math": [_P, _I],
    "bgnn_ctx_synchronize": [_P],
    "bgnn_last_error": [_P],
    "bgnn_ctx_launch_count": [_P],
    "bgnn_memcpy_h2d": [_P, _P, _P, _U64],
    "bgnn_memcpy_d2h": [_P, _P, _P, _U64],
    "bgnn_spmm_host": [_P, _P, _P, _P, _P, _U32, _U32, _U32, _P],
    "bgnn_scatter_add_host": [_P, _P, _P, _U64, _U32, _U32, _P],
    "bgnn_scatter_mean_host": [_P, _P, _P, _U64, _U32, _U32, _P],
    "bgnn_scatter_max_host": [_P, _P, _P, _U64, _U32, _U32, _P],
    "bgnn_gather_host": [_P, _P, _U32, _P, _U64, _U32, _P],
    "bgnn_matmul_host": [_P, _P, _P, _U32, _U32, _U32, _P],
    "bgnn_relu_host": [_P, _P, _U64, _P],
    "bgnn_add_host": [_P, _P, _P, _U64, _P],
    "bgnn_spmv_host": [_P, _P, _P, _P, _P, _U32, _U32, _P],
    "bgnn_spmm_dev": [_P, _P, _P, _P, _P, _U32, _U32, _U32, _P],
    "bgnn_scatter_dev": [_P, _I, _P, _P, _U64, _U32, _U32, _P],
    "bgnn_gather_dev": [_P, _P, _U32, _P, _U64, _U32, _P],
    "bgnn_matmul_dev": [_P, _P, _P, _U32, _U32, _U32, _P],
    "bgnn_activation_dev": [_P, _I, _D, _P, _U64, _P],
    "bgnn_add_dev": [_P, _P, _P, _U64, _P],
    "bgnn_spmv_dev": [_P, _P, _P, _P, _P, _U32, _U32, _P],
    "bgnn_coo_to_csr_dev": [_P, _P, _P, _P, _U64, _U32, _U32, _P, _P, _P],
    "bgnn_coo_to_csr_host": [_P, _P, _P, _P, _U64, _U32, _U32, _P, _P, _P],
    "bgnn_gcn_norm_dev": [_P, _P, _U64, _U32, _I, _P],
    "bgnn_graph_create": [_P, _P, _U64, _U32, _U32, _I, ctypes.POINTER(_P)],
    "bgnn_graph_create_csr": [_P, _P, _P, _U32, _U32, ctypes.POINTER(_P)],
    "bgnn_graph_destroy": [_P],
    "bgnn_graph_info": [_P, ctypes.POINTER(_U32), ctypes.POINTER(_U32), ctypes.POINTER(_U64),
                        ctypes.POINTER(_I)],
    "bgnn_graph_degrees": [_P, _P, _P, _P],
    "bgnn_graph_csr": [_P, _P, _P, _P, _P],
    "bgnn_aggregate": [_P, _P, _I, _P, _U32, _P],
    "bgnn_gcn_propagate": [_P, _P, _P, _U32, _I, _I, _P, _I, _D, _P],
    "bgnn_gat": [_P, _P, _P, _U32, _U32, _P, _P, _D, _I, _I, _P, _I, _D, _P],
    "bgnn_gat_noalloc": [_P, _P, _P, _U32, _U32, _P, _P, _D, _I, _I, _P, _I, _D, _P],
    "bgnn_gat_train": [_P, _P, _P, _U32, _U32, _P, _P, _D, _I, _I, _P, _I, _D, _D, _U64, _P],
    "bgnn_gin_aggregate": [_P, _P, _P, _U32, _F, _P],
    "bgnn_graph_spmm": [_P, _P, _P, _P, _U32, _P],
    "bgnn_linear": [_P, _P, _P, _U32, _U32, _U32, _P, _I, _D, _P],
    "bgnn_sage_linear": [_P, _P, _P, _P, _P, _U32, _U32, _U32, _P, _I, _D, _P],
    "bgnn_linear_add": [_P, _P, _P, _U32, _U32, _U32, _P, _P, _I, _D, _P],
    "bgnn_l2_normalize_rows": [_P, _P, _U32, _U32],
    "bgnn_sum_pool": [_P, _P, _U32, _U32, _P, _U32, _P],
    "bgnn_pack_rows": [_P, _P, _U32, _P, _U32, _U32, _P],
    "bgnn_pool_projection": [_P, _P, _P, _P, _U32, _U32, _P],
    "bgnn_synth_rmat": [_P, _U64, _I, _U32, _U64, _D, _D, _D, _I, _P],
    "bgnn_dense": [_P, _P, _P, _U32, _U32, _U32, _P, _I, _D, _P],
    "bgnn_segment_sum": [_P, _P, _U32, _P, _U32, _P],
    "bgnn_softmax_rows": [_P, _P, _U32, _U32, _P, _F, _I, _P],
    "bgnn_dropout": [_P, _P, _U64, _D, _U64, _P],
    "bgnn_prelu": [_P, _P, _U64, _P, _U32, _P],
    "bgnn_link_scores": [_P, _P, _U32, _U32, _P, _P, _U64, _I, _P, _P, _P, _P, _P, _P],
    "bgnn_aggregate_strided": [_P, _P, _I, _P, _P, _U64, _U32, _P, _U64],
    "bgnn_aggregate_backward": [_P, _P, _I, _P, _P, _U32, _P],
    "bgnn_gcn_propagate_backward": [_P, _P, _P, _U32, _I, _I, _P],
    "bgnn_matmul_backward": [_P, _P, _P, _P, _U32, _U32, _U32, _P, _P],
    "bgnn_bias_backward": [_P, _P, _U64, _U32, _P],
    "bgnn_relu_backward": [_P, _P, _P, _U64, _P],
    "bgnn_part_create": [_P, _P, _U64, _U32, _U32, _U32, _I, ctypes.POINTER(_P)],
    "bgnn_part_create_csr": [_P, _P, _P, _U32, _U32, _U32, ctypes.POINTER(_P)],
    "bgnn_part_destroy": [_P],
    "bgnn_part_info": [_P, ctypes.POINTER(_U32), ctypes.POINTER(_U32), ctypes.POINTER(_U32),
                       ctypes.POINTER(_U64), ctypes.POINTER(_U64), ctypes.POINTER(_U64)],
    "bgnn_part_bounds": [_P, ctypes.POINTER(_U32)],
    "bgnn_part_counts": [_P, ctypes.POINTER(_U64), ctypes.POINTER(_U64)],
    "bgnn_part_row_blocks": [_P, _P, _U32, ctypes.POINTER(_U64), ctypes.POINTER(_U64)],
    "bgnn_part_graph": [_P, ctypes.POINTER(_P)],
    "bgnn_part_lists": [_P, _P, _P, _P],
    "bgnn_part_pack": [_P, _P, _P, _U64, _U32, _U32, _P],
    "bgnn_part_unpack": [_P, _P, _P, _U32, _P, _U64, _U32],
    "bgnn_dist_unique_id": [_P],
    "bgnn_dist_create": [_P, _P, _U32, _U32, _U32, _U32, ctypes.POINTER(_P)],
    "bgnn_dist_destroy": [_P],
    "bgnn_dist_abort": [_P],
    "bgnn_dist_set_pipeline": [_P, _U32, _U32],
    "bgnn_dist_exchange": [_P, _P, _P, _U32],
    "bgnn_dist_aggregate": [_P, _P, _I, _P, _U32, _P],
    "bgnn_dist_spmm": [_P, _P, _P, _P, _U32, _P],
    "bgnn_dist_sage_layer": [_P, _P, _I, _P, _U32, _U32, _P, _P, _P, _I, _D, _P, _P],
    "bgnn_dist_sage_layer_ex": [_P, _P, _I, _P, _U32, _U32, _P, _P, _P, _I, _D, _P, _P, _U32],
    "bgnn_dist_set_row_blocks": [_P, _U32],
    "bgnn_dist_allreduce_max": [_P, ctypes.POINTER(_D), _U32],
    "bgnn_dist_synchronize": [_P],
}
_RESTYPE = {"bgnn_last_error": ctypes.c_char_p, "bgnn_ctx_launch_count": ctypes.c_uint64}

_lib = None
_lock = threading.Lock()


def load():
    """Load libbgnn_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m browsergnn_b200.build` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = _RESTYPE.get(name, ctypes.c_int)
            if lib.bgnn_abi_version() != 1:
                raise RuntimeError("libbgnn_cuda ABI version mismatch")
            _lib = lib
    return _lib


def check(status: int, ctx=None):
    if status == OK:
        return
    msg = ""
    if ctx is not None:
        raw = load().bgnn_last_error(ctx)
        msg = raw.decode() if raw else ""
    if status == ERR_OUT_OF_RANGE:
        raise BGNNIndexError(status, msg)
    raise BGNNError(status, msg)
