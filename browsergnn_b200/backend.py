"""The `cuda` backend: context management and the GPU facade.

Mirrors the reference's backend selection and GPU dispatch facade:
  BackendManager / initBrowserGNN / getBackend   src/backend/index.ts:102-274
  WebGPUComputeManager (host arrays in, fresh host array out)
                                                 src/backend/webgpu/compute-pipeline.ts:140-644
  GPUSparse / GPUTensor (Tensor in, Tensor out)  src/core/gpu-sparse.ts:19-285

Differences by design: there is no silent CPU fallback -- a failing CUDA call
raises, and the backend refuses to initialise without a CUDA device.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _lib

BACKEND_NAME = "cuda"


def _torch():
    import torch

    return torch


class CudaContext:
    """One libbgnn context per device, following torch's current stream."""

    def __init__(self, device: int = 0):
        torch = _torch()
        if not torch.cuda.is_available():
            raise RuntimeError("the cuda backend needs a CUDA device (there is no CPU fallback)")
        self.lib = _lib.load()
        h = ctypes.c_void_p()
        _lib.check(self.lib.bgnn_ctx_create(int(device), ctypes.byref(h)))
        self.h = h
        self.device = int(device)
        self._stream = None
        self._math = _lib.MATH_FAST

    def bind(self):
        torch = _torch()
        s = torch.cuda.current_stream(self.device).cuda_stream
        if s != self._stream:
            _lib.check(self.lib.bgnn_ctx_set_stream(self.h, s if s else None), self.h)
            self._stream = s
        return self.h

    def call(self, name: str, *args):
        h = self.bind()
        rc = getattr(self.lib, name)(h, *args)
        _lib.check(rc, self.h)

    def call_on(self, name: str, *args):
        """Call an entry point whose first argument is another handle (a
        partition, a communicator) that reports errors on this context."""
        self.bind()
        rc = getattr(self.lib, name)(*args)
        _lib.check(rc, self.h)

    def set_math(self, mode):
        """True / "exact": the reference's rounding, bit for bit; False /
        "fast": f32 fma in the reference's order (the default); "tensor":
        X*W on the tcgen05 tensor cores (3xTF32, f32-level accuracy, not
        the reference's summation order)."""
        if mode is True or mode == "exact":
            code = _lib.MATH_EXACT
        elif mode is False or mode is None or mode == "fast":
            code = _lib.MATH_FAST
        elif mode == "tensor":
            code = _lib.MATH_TENSOR
        else:
            raise ValueError(f"unknown math mode {mode!r}")
        _lib.check(self.lib.bgnn_ctx_set_math(self.h, code), self.h)
        self._math = code

    @property
    def exact(self) -> bool:
        return self._math == _lib.MATH_EXACT

    def synchronize(self):
        self.bind()
        _lib.check(self.lib.bgnn_ctx_synchronize(self.h), self.h)

    @property
    def launches(self) -> int:
        return int(self.lib.bgnn_ctx_launch_count(self.h))

    def close(self):
        if self.h:
            self.lib.bgnn_ctx_destroy(self.h)
            self.h = None


_contexts: dict = {}


def get_context(device: Optional[int] = None) -> CudaContext:
    torch = _torch()
    if device is None:
        device = torch.cuda.current_device() if torch.cuda.is_available() else 0
    ctx = _contexts.get(device)
    if ctx is None:
        ctx = CudaContext(device)
        _contexts[device] = ctx
    return ctx


def ptr(t) -> Optional[int]:
    """Device address of a torch tensor (None passes NULL)."""
    return None if t is None else t.data_ptr()


def as_device(a, dtype, device: int):
    """numpy / list / torch -> contiguous CUDA tensor of `dtype`.  Host
    arrays go through the library's staged copy (bgnn_memcpy_h2d)."""
    torch = _torch()
    if isinstance(a, torch.Tensor):
        t = a.to(device=f"cuda:{device}", dtype=dtype)
        return t.contiguous()
    npdt = {torch.float32: np.float32, torch.int32: np.uint32}[dtype]
    arr = np.ascontiguousarray(np.asarray(a, dtype=npdt))
    t = torch.empty(arr.shape, dtype=dtype, device=f"cuda:{device}")
    if arr.size:
        get_context(device).call("bgnn_memcpy_h2d", ptr(t), arr.ctypes.data, arr.nbytes)
    return t


def to_host(t, out: Optional[np.ndarray] = None) -> np.ndarray:
    """A CUDA tensor's values in a host float32 / uint32 array (a fresh one, as
    WebGPUComputeManager returns, or `out`), through the library's staged
    copy (bgnn_memcpy_d2h): no page-locked memory needed on the caller's
    side."""
    torch = _torch()
    t = t.contiguous()
    npdt = {torch.float32: np.float32, torch.int32: np.uint32}[t.dtype]
    if out is None:
        out = np.empty(tuple(t.shape), npdt)
    if out.nbytes != t.numel() * t.element_size() or not out.flags.c_contiguous:
        raise ValueError("out must be a contiguous array of the tensor's size")
    if out.size:
        get_context(t.device.index).call("bgnn_memcpy_d2h", out.ctypes.data, ptr(t), out.nbytes)
    return out


# ---- backend manager mirror ---------------------------------------------------
def init_browsergnn(config: Optional[dict] = None) -> str:
    """initBrowserGNN (src/backend/index.ts:265): brings up the cuda backend."""
    device = (config or {}).get("device", None)
    get_context(device)
    return BACKEND_NAME


initBrowserGNN = init_browsergnn


def get_backend() -> str:
    return BACKEND_NAME


getBackend = get_backend


def is_gpu_available() -> bool:
    """isGPUAvailable (src/core/gpu-sparse.ts:283-285)."""
    try:
        return _torch().cuda.is_available() and _lib.load() is not None
    except Exception:
        return False


isGPUAvailable = is_gpu_available


# ---- WebGPUComputeManager mirror: host arrays in, fresh host arrays out ------
def _f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _u32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


def _hp(a):
    return a.ctypes.data if a is not None and a.size else None


class CudaComputeManager:
    """Same method set as WebGPUComputeManager (compute-pipeline.ts:140-644).

    Each call copies its inputs to the device, runs, and returns a new float32
    numpy array, as the reference's manager returns a fresh Float32Array.
    """

    def __init__(self, device: Optional[int] = None):
        self.ctx = get_context(device)

    def _call(self, name, *args):
        # host entry points are synchronous; they run on the context stream
        self.ctx.call(name, *args)

    def spmm(self, rowPtr, colIndices, values, dense, numRows, numCols, numFeatures):
        rp, ci, va, de = _u32(rowPtr), _u32(colIndices), _f32(values), _f32(dense)
        out = np.empty(int(numRows) * int(numFeatures), np.float32)
        self._call("bgnn_spmm_host", _hp(rp), _hp(ci), _hp(va), _hp(de), numRows, numCols,
                   numFeatures, _hp(out))
        return out

    def _scatter(self, name, src, indices, numNodes, numFeatures):
        s, ix = _f32(src), _u32(indices)
        out = np.empty(int(numNodes) * int(numFeatures), np.float32)
        self._call(name, _hp(s), _hp(ix), ix.size, numNodes, numFeatures, _hp(out))
        return out

    def scatterAdd(self, src, indices, numNodes, numFeatures):
        return self._scatter("bgnn_scatter_add_host", src, indices, numNodes, numFeatures)

    def scatterMean(self, src, indices, numNodes, numFeatures):
        return self._scatter("bgnn_scatter_mean_host", src, indices, numNodes, numFeatures)

    def scatterMax(self, src, indices, numNodes, numFeatures):
        return self._scatter("bgnn_scatter_max_host", src, indices, numNodes, numFeatures)

    def gather(self, src, indices, numFeatures):
        s, ix = _f32(src), _u32(indices)
        nf = int(numFeatures)
        rows = s.size // nf if nf else 0
        out = np.empty(ix.size * nf, np.float32)
        self._call("bgnn_gather_host", _hp(s), rows, _hp(ix), ix.size, nf, _hp(out))
        return out

    def matmul(self, a, b, m, k, n):
        aa, bb = _f32(a), _f32(b)
        out = np.empty(int(m) * int(n), np.float32)
        self._call("bgnn_matmul_host", _hp(aa), _hp(bb), m, k, n, _hp(out))
        return out

    def relu(self, data):
        x = _f32(data)
        out = np.empty_like(x)
        self._call("bgnn_relu_host", _hp(x), x.size, _hp(out))
        return out

    def add(self, a, b):
        aa, bb = _f32(a), _f32(b)
        if aa.size != bb.size:
            raise ValueError(f"Size mismatch: {aa.size} vs {bb.size}")
        out = np.empty_like(aa)
        self._call("bgnn_add_host", _hp(aa), _hp(bb), aa.size, _hp(out))
        return out

    def spmv(self, rowPtr, colIndices, values, x, numRows):
        rp, ci, va, xx = _u32(rowPtr), _u32(colIndices), _f32(values), _f32(x)
        out = np.empty(int(numRows), np.float32)
        self._call("bgnn_spmv_host", _hp(rp), _hp(ci), _hp(va), _hp(xx), numRows, xx.size,
                   _hp(out))
        return out

    def coo_to_csr(self, rows, cols, values, numRows, numCols):
        r, c = _u32(rows), _u32(cols)
        v = None if values is None else _f32(values)
        rp = np.empty(int(numRows) + 1, np.uint32)
        co = np.empty(max(r.size, 1), np.uint32)
        vo = np.empty(max(r.size, 1), np.float32)
        self._call("bgnn_coo_to_csr_host", _hp(r), _hp(c), _hp(v), r.size, numRows, numCols,
                   _hp(rp), _hp(co), _hp(vo))
        return rp, co[:r.size], vo[:r.size]


def get_compute_manager() -> CudaComputeManager:
    """getComputeManager (src/backend/index.ts:293)."""
    return CudaComputeManager()


getComputeManager = get_compute_manager
