"""Neural-network modules of src/nn/ on the cuda backend.

Linear (src/nn/linear.ts), the activation modules of src/nn/activation.ts
(ReLU, LeakyReLU, ELU, Sigmoid, Tanh, Softmax, LogSoftmax, GELU, SiLU, PReLU,
Dropout) and the Module / Sequential containers of src/nn/module.ts.  Same
constructor arguments, parameter names and shapes, defaults and errors as the
reference; ``forward`` takes a CUDA tensor (or a GraphData, whose features it
transforms) and returns the same kind.

Training-mode Dropout draws from a counter-based generator (libbgnn_cuda's
bgnn_dropout) instead of Math.random(): the keep/scale rule is the
reference's, the random stream is not (the reference's is unseeded).  In eval
mode Dropout is the identity, exactly as in the reference.
"""
from __future__ import annotations

from typing import Optional

import numpy as np

from . import _lib
from .backend import get_context, ptr
from .graph import GraphData
from .layers import (ELU, LeakyReLU, Module, ReLU, Sequential, _Act, _param, _torch,
                     manual_seed, next_dropout_seed, register_fusable)

__all__ = [
    "Module", "Sequential", "Linear", "ReLU", "LeakyReLU", "ELU", "Sigmoid", "Tanh", "GELU",
    "SiLU", "PReLU", "Softmax", "LogSoftmax", "Dropout", "manual_seed",
]


def _tensor_of(input):
    return input.x_device() if isinstance(input, GraphData) else input


def _wrap(input, out):
    return input.withFeatures(out) if isinstance(input, GraphData) else out


class Linear(Module):
    """src/nn/linear.ts:19-115: y = x W^T + b with ``weight`` [out, in] and
    ``bias`` [out] (zeros); the weight is a normal draw scaled by
    sqrt(2 / (in + out)).  Each output is one double sum over the inputs,
    stored to f32, then the bias is added in f32."""

    def __init__(self, config: Optional[dict] = None, **kw):
        super().__init__()
        cfg = dict(config or {})
        cfg.update(kw)
        self.inFeatures = int(cfg["inFeatures"])
        self.outFeatures = int(cfg["outFeatures"])
        self.useBias = bool(cfg.get("bias", True))
        stdv = np.sqrt(2.0 / (self.inFeatures + self.outFeatures))
        self.registerParameter("weight", _param((self.outFeatures, self.inFeatures), stdv))
        if self.useBias:
            self.registerParameter("bias", _param((self.outFeatures,), zeros=True))

    def forward(self, input, _act=None):
        torch = _torch()
        x = _tensor_of(input)
        if not hasattr(x, "is_cuda"):
            x = torch.as_tensor(np.asarray(x, np.float32))
        if x.dim() == 1:
            if x.shape[0] != self.inFeatures:
                raise ValueError(f"Expected input size {self.inFeatures}, got {x.shape[0]}")
            rows = 1
        elif x.dim() == 2:
            if x.shape[1] != self.inFeatures:
                raise ValueError(f"Expected input size {self.inFeatures}, got {x.shape[1]}")
            rows = int(x.shape[0])
        else:
            raise ValueError(f"Linear layer expects 1D or 2D input, got {x.dim()}D")
        if not x.is_cuda:
            x = x.to("cuda")
        x = x.to(torch.float32).contiguous()
        dev = x.device.index
        self.to_device(dev)
        out = torch.empty((rows, self.outFeatures), dtype=torch.float32, device=x.device)
        code, param = (0, 0.0) if _act is None else (_lib.ACT[_act[0]], float(_act[1]))
        get_context(dev).call("bgnn_dense", ptr(x), ptr(self.p("weight")), rows, self.inFeatures,
                              self.outFeatures, ptr(self.p("bias")), code, param, ptr(out))
        if x.dim() == 1:
            out = out.reshape(self.outFeatures)
        return _wrap(input, out)

    def __repr__(self):
        return f"Linear({self.inFeatures} -> {self.outFeatures}, bias={self.useBias})"


class Sigmoid(_Act):
    """Tensor.sigmoid (src/core/tensor.ts:413-419): 1 / (1 + exp(-x)) in double."""
    act = "sigmoid"


class Tanh(_Act):
    """Tensor.tanh (src/core/tensor.ts:424-430)."""
    act = "tanh"


class GELU(_Act):
    """src/nn/activation.ts:129-147 (tanh approximation, evaluated in double)."""
    act = "gelu"


class SiLU(_Act):
    """src/nn/activation.ts:153-168: x / (1 + exp(-x))."""
    act = "silu"


class PReLU(Module):
    """src/nn/activation.ts:175-200: learnable ``weight`` [numParameters]
    filled with ``init``; slope weight[0] or weight[i % numParameters]."""

    def __init__(self, numParameters: int = 1, init: float = 0.25):
        super().__init__()
        torch = _torch()
        self.registerParameter("weight", torch.full((int(numParameters),), float(init),
                                                    dtype=torch.float32))

    def forward(self, input):
        torch = _torch()
        x = _tensor_of(input).contiguous()
        self.to_device(x.device.index)
        w = self.p("weight")
        out = torch.empty_like(x)
        get_context(x.device.index).call("bgnn_prelu", ptr(x), x.numel(), ptr(w), w.numel(),
                                         ptr(out))
        return _wrap(input, out)


class _RowSoftmax(Module):
    log = 0

    def forward(self, input):
        torch = _torch()
        x = _tensor_of(input)
        if x.dim() != 2:
            name = "Log softmax" if self.log else "Softmax"
            raise ValueError(f"{name} currently only supports 2D tensors")
        x = x.contiguous()
        out = torch.empty_like(x)
        rows, cols = x.shape
        get_context(x.device.index).call("bgnn_softmax_rows", ptr(x), rows, cols, None, 0.0,
                                         self.log, ptr(out))
        return _wrap(input, out)


class Softmax(_RowSoftmax):
    """Tensor.softmax along the last axis (src/core/tensor.ts:435-464)."""
    log = 0


class LogSoftmax(_RowSoftmax):
    """Tensor.logSoftmax along the last axis (src/core/tensor.ts:469-499)."""
    log = 1


class Dropout(Module):
    """src/nn/activation.ts:207-245.  Identity in eval mode or for p = 0;
    in training mode element i survives when u_i > p and is scaled by
    1 / (1 - p), u_i from the counter-based generator (one fresh seed per
    call)."""

    def __init__(self, p: float = 0.5):
        super().__init__()
        if p < 0 or p > 1:
            raise ValueError("Dropout probability must be between 0 and 1")
        self.p = float(p)

    def forward(self, input, seed: Optional[int] = None):
        if not self._training or self.p == 0:
            return input
        torch = _torch()
        x = _tensor_of(input).contiguous()
        out = torch.empty_like(x)
        s = next_dropout_seed() if seed is None else int(seed)
        get_context(x.device.index).call("bgnn_dropout", ptr(x), x.numel(), self.p, s, ptr(out))
        return _wrap(input, out)


register_fusable(Linear)
