"""GCNConv, GATConv, SAGEConv, GINConv on the cuda backend.

Same configuration keys, parameter names, shapes, defaults and errors as the
reference layers (src/layers/gcn.ts, gat.ts, sage.ts, gin.ts), so weights
injected through ``loadStateDict`` under the reference's names produce the
reference's outputs.  ``forward`` takes and returns a ``GraphData``; features
stay on the GPU between layers, and the graph's CSR is built once and shared.

Parameter initialisation follows the reference's scheme (a normal draw scaled
by sqrt(2/(fan_in+fan_out)), zero biases) from a seeded generator; the
reference draws from the unseeded Math.random, so parity tests inject weights.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Optional

import numpy as np

from . import _lib
from .backend import get_context, ptr
from .graph import GraphData

_rng = np.random.default_rng(0xB200)
_seed_rng = np.random.default_rng(0xB2000D)


def manual_seed(seed: int) -> None:
    """Reseed the generator that gives each training-mode dropout call
    (Dropout modules, GAT attention dropout) its own seed."""
    global _seed_rng
    _seed_rng = np.random.default_rng(int(seed))


def next_dropout_seed() -> int:
    return int(_seed_rng.integers(0, 2 ** 63, dtype=np.int64))


def _torch():
    import torch

    return torch


def _param(shape, stdv=None, zeros=False):
    torch = _torch()
    if zeros:
        arr = np.zeros(shape, np.float32)
    else:
        arr = (stdv * _rng.standard_normal(int(np.prod(shape)))).astype(np.float32).reshape(shape)
    return torch.from_numpy(arr)


class Parameter:
    """A named tensor (src/nn/module.ts Parameter): ``.tensor`` is a CUDA
    tensor once the module has been moved to a device (lazily on forward)."""

    def __init__(self, tensor):
        self.tensor = tensor

    def numel(self):
        return int(self.tensor.numel())


class Module:
    """src/nn/module.ts:23-139: parameter registry, train/eval flag
    (``_training`` defaults to True, as in the reference)."""

    def __init__(self):
        self._parameters: "OrderedDict[str, Parameter]" = OrderedDict()
        self._buffers: "OrderedDict[str, object]" = OrderedDict()
        self._modules: "OrderedDict[str, Module]" = OrderedDict()
        self._training = True
        self._device = None

    def registerParameter(self, name, tensor):
        self._parameters[name] = Parameter(tensor)

    def registerBuffer(self, name, tensor):
        self._buffers[name] = tensor

    def registerModule(self, name, module):
        self._modules[name] = module

    def namedParameters(self, prefix: str = ""):
        out = []
        for n, p in self._parameters.items():
            out.append((prefix + n, p))
        for mn, m in self._modules.items():
            out.extend(m.namedParameters(prefix + mn + "."))
        return out

    def parameters(self):
        return [p for _, p in self.namedParameters()]

    def numParameters(self) -> int:
        return sum(p.numel() for p in self.parameters())

    def train(self, mode: bool = True):
        self._training = mode
        for m in self._modules.values():
            m.train(mode)
        return self

    def eval(self):
        return self.train(False)

    @property
    def training(self) -> bool:
        return self._training

    def stateDict(self):
        return {n: p.tensor.detach().cpu().numpy().copy() for n, p in self.namedParameters()}

    def loadStateDict(self, state, strict: bool = True):
        """Weight injection by the reference's parameter names
        (src/utils/serialization.ts:58-115)."""
        torch = _torch()
        named = dict(self.namedParameters())
        for name, value in state.items():
            if name not in named:
                if strict:
                    raise KeyError(f"Unexpected parameter: {name}")
                continue
            p = named[name]
            arr = np.asarray(value.cpu().numpy() if hasattr(value, "cpu") else value,
                             dtype=np.float32)
            if arr.size != p.tensor.numel():
                raise ValueError(f"Shape mismatch for {name}: {arr.size} vs {p.tensor.numel()}")
            t = torch.from_numpy(np.ascontiguousarray(arr).reshape(tuple(p.tensor.shape)))
            p.tensor = t.to(p.tensor.device)
        if strict:
            missing = set(named) - set(state)
            if missing:
                raise KeyError(f"Missing parameters: {sorted(missing)}")

    def to_device(self, device: int):
        torch = _torch()
        if self._device != device:
            for p in self._parameters.values():
                p.tensor = p.tensor.to(device=f"cuda:{device}", dtype=torch.float32).contiguous()
            for k, b in list(self._buffers.items()):
                if hasattr(b, "to"):
                    self._buffers[k] = b.to(f"cuda:{device}")
            for m in self._modules.values():
                m.to_device(device)
            self._device = device
        return self

    def p(self, name):
        return self._parameters[name].tensor if name in self._parameters else None

    def __call__(self, *a, **kw):
        return self.forward(*a, **kw)


def _act_code(act):
    if act is None:
        return 0, 0.0
    if isinstance(act, tuple):
        return _lib.ACT[act[0]], float(act[1])
    return _lib.ACT[act], (1.0 if act == "elu" else 0.01)


def _prepare(layer: Module, graph: GraphData, in_channels: int, name: str):
    if graph.numFeatures != in_channels:
        raise ValueError(f"{name}: Expected {in_channels} input channels, got {graph.numFeatures}")
    dg = graph.device_graph()
    layer.to_device(dg.device)
    return dg, graph.x_device(dg.device)


def _linear(ctx, x, w, bias=None, act=None):
    torch = _torch()
    m, k = x.shape
    n = w.shape[1]
    out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    code, param = _act_code(act)
    ctx.call("bgnn_linear", ptr(x), ptr(w), m, k, n, ptr(bias), code, param, ptr(out))
    return out


def _pre_activation_grad(ctx, grad_out, out, act):
    """The gradient before the layer's activation (only ReLU is
    differentiated, as in src/autograd/variable.ts:358-373)."""
    torch = _torch()
    if act in (None, "none"):
        return grad_out.contiguous()
    if act != "relu":
        raise NotImplementedError(f"backward through activation {act!r}")
    g = torch.empty_like(grad_out)
    ctx.call("bgnn_relu_backward", ptr(grad_out.contiguous()), ptr(out), out.numel(), ptr(g))
    return g


def _matmul_backward(ctx, a, w, g):
    """(grad_a, grad_w) of a @ w (Variable.matmul, variable.ts:213-235)."""
    torch = _torch()
    m, k = a.shape
    n = w.shape[1]
    ga = torch.empty((m, k), dtype=torch.float32, device=a.device)
    gw = torch.empty((k, n), dtype=torch.float32, device=a.device)
    ctx.call("bgnn_matmul_backward", ptr(a), ptr(w), ptr(g), m, k, n, ptr(ga), ptr(gw))
    return ga, gw


def _bias_backward(ctx, g):
    torch = _torch()
    out = torch.empty(g.shape[1], dtype=torch.float32, device=g.device)
    ctx.call("bgnn_bias_backward", ptr(g), g.shape[0], g.shape[1], ptr(out))
    return out


class GCNConv(Module):
    """src/layers/gcn.ts:34-286."""

    def __init__(self, config: Optional[dict] = None, **kw):
        super().__init__()
        cfg = dict(config or {})
        cfg.update(kw)
        self.inChannels = int(cfg["inChannels"])
        self.outChannels = int(cfg["outChannels"])
        self.addSelfLoops = bool(cfg.get("addSelfLoops", True))
        self.normalize = bool(cfg.get("normalize", True))
        self.useBias = bool(cfg.get("bias", True))
        stdv = np.sqrt(2.0 / (self.inChannels + self.outChannels))
        self.registerParameter("weight", _param((self.inChannels, self.outChannels), stdv))
        if self.useBias:
            self.registerParameter("bias", _param((self.outChannels,), zeros=True))

    def forward(self, input: GraphData, _act=None) -> GraphData:
        torch = _torch()
        dg, x = _prepare(self, input, self.inChannels, "GCNConv")
        ctx = dg.ctx
        h = _linear(ctx, x, self.p("weight"))  # X @ W  (gcn.ts:98)
        out = torch.empty((input.numNodes, self.outChannels), dtype=torch.float32, device=x.device)
        code, param = _act_code(_act)
        ctx.call("bgnn_gcn_propagate", dg.h, ptr(h), self.outChannels, int(self.addSelfLoops),
                 int(self.normalize), ptr(self.p("bias")), code, param, ptr(out))
        return input.withFeatures(out)

    forwardAsync = forward

    def backward(self, input: GraphData, grad_out, _act=None, output=None) -> dict:
        """Gradients of forward(input, _act) for an upstream gradient
        grad_out [N, out]: {"x", "weight", "bias"}.  The reference never
        differentiates a layer; this is the adjoint of each forward step
        (bgnn_gcn_propagate_backward for the propagation, Variable.matmul's
        backward for X @ W, the broadcast reduction for the bias, ReLU's
        mask).  `output` is the forward's output (recomputed when omitted)."""
        dg, x = _prepare(self, input, self.inChannels, "GCNConv")
        ctx = dg.ctx
        torch = _torch()
        if _act not in (None, "none") and output is None:
            output = self.forward(input, _act=_act).x
        g = _pre_activation_grad(ctx, grad_out, output, _act)
        grads = {}
        if self.useBias:
            grads["bias"] = _bias_backward(ctx, g)
        gh = torch.empty_like(g)
        ctx.call("bgnn_gcn_propagate_backward", dg.h, ptr(g), self.outChannels,
                 int(self.addSelfLoops), int(self.normalize), ptr(gh))
        grads["x"], grads["weight"] = _matmul_backward(ctx, x, self.p("weight"), gh)
        return grads

    def __repr__(self):
        return (f"GCNConv({self.inChannels} -> {self.outChannels}, bias={self.useBias}, "
                f"normalize={self.normalize})")


class GATConv(Module):
    """src/layers/gat.ts:36-454."""

    def __init__(self, config: Optional[dict] = None, **kw):
        super().__init__()
        cfg = dict(config or {})
        cfg.update(kw)
        self.inChannels = int(cfg["inChannels"])
        self.outChannels = int(cfg["outChannels"])
        self.heads = int(cfg.get("heads", 1))
        self.concat = bool(cfg.get("concat", True))
        self.negativeSlope = float(cfg.get("negativeSlope", 0.2))
        self.dropout = float(cfg.get("dropout", 0.0))
        self.addSelfLoops = bool(cfg.get("addSelfLoops", True))
        self.useBias = bool(cfg.get("bias", True))
        stdv = np.sqrt(2.0 / (self.inChannels + self.outChannels))
        hc = self.heads * self.outChannels
        self.registerParameter("weight", _param((self.inChannels, hc), stdv))
        att_stdv = np.sqrt(2.0 / (2 * self.outChannels))
        self.registerParameter("att_src", _param((self.heads, self.outChannels), att_stdv))
        self.registerParameter("att_dst", _param((self.heads, self.outChannels), att_stdv))
        if self.useBias:
            self.registerParameter("bias", _param((hc if self.concat else self.outChannels,),
                                                  zeros=True))

    @property
    def outputDim(self) -> int:
        return self.heads * self.outChannels if self.concat else self.outChannels

    def forward(self, input: GraphData, _act=None, seed: Optional[int] = None) -> GraphData:
        torch = _torch()
        dg, x = _prepare(self, input, self.inChannels, "GATConv")
        ctx = dg.ctx
        h = _linear(ctx, x, self.p("weight"))  # H = X @ W  (gat.ts:130)
        out = torch.empty((input.numNodes, self.outputDim), dtype=torch.float32, device=x.device)
        code, param = _act_code(_act)
        args = (dg.h, ptr(h), self.heads, self.outChannels, ptr(self.p("att_src")),
                ptr(self.p("att_dst")), self.negativeSlope, int(self.concat),
                int(self.addSelfLoops), ptr(self.p("bias")), code, param)
        if self._training and self.dropout > 0:
            # gat.ts:194-203: attention dropout while training, one draw per
            # (edge, head) from the counter-based generator
            s = next_dropout_seed() if seed is None else int(seed)
            ctx.call("bgnn_gat_train", *args, self.dropout, s, ptr(out))
        else:
            ctx.call("bgnn_gat", *args, ptr(out))
        return input.withFeatures(out)

    forwardAsync = forward


class SAGEConv(Module):
    """src/layers/sage.ts:43-373 (aggregators mean / max / sum / pool)."""

    def __init__(self, config: Optional[dict] = None, **kw):
        super().__init__()
        cfg = dict(config or {})
        cfg.update(kw)
        self.inChannels = int(cfg["inChannels"])
        self.outChannels = int(cfg["outChannels"])
        self.aggregator = cfg.get("aggregator", "mean")
        if self.aggregator not in ("mean", "max", "sum", "pool"):
            raise ValueError(f"Unknown aggregator: {self.aggregator}")
        self.normalize = bool(cfg.get("normalize", False))
        self.rootWeight = bool(cfg.get("rootWeight", True))
        self.useBias = bool(cfg.get("bias", True))
        stdv = np.sqrt(2.0 / (self.inChannels + self.outChannels))
        self.registerParameter("lin_neighbor", _param((self.inChannels, self.outChannels), stdv))
        if self.rootWeight:
            self.registerParameter("lin_self", _param((self.inChannels, self.outChannels), stdv))
        if self.useBias:
            self.registerParameter("bias", _param((self.outChannels,), zeros=True))
        if self.aggregator == "pool":
            pstdv = np.sqrt(2.0 / (2 * self.inChannels))
            self.registerParameter("pool_weight", _param((self.inChannels, self.inChannels), pstdv))
            self.registerParameter("pool_bias", _param((self.inChannels,), zeros=True))

    def aggregate(self, dg, x):
        """Step 1-2 (sage.ts:124-168): fused gather + scatter{Mean,Max,Add}."""
        torch = _torch()
        ctx = dg.ctx
        src = x
        aggr = self.aggregator
        if aggr == "pool":
            # the projection of an edge's message depends only on its source
            # node, so project each node once and max-aggregate the projections
            from .ops import pool_projection

            src = pool_projection(ctx, x, self.p("pool_weight"), self.p("pool_bias"))
            aggr = "max"
        agg = torch.empty((dg.num_dst, self.inChannels), dtype=torch.float32, device=x.device)
        ctx.call("bgnn_aggregate", dg.h, _lib.AGGR[aggr], ptr(src), self.inChannels, ptr(agg))
        return agg

    def forward(self, input: GraphData, _act=None, _send_next: bool = False) -> GraphData:
        if getattr(input, "pg", None) is not None:
            # one rank's share of a row-partitioned graph (distributed.partition);
            # _send_next: another layer reads the output (its halo exchange
            # starts while this layer's last product runs)
            from .distributed import sage_forward

            return sage_forward(self, input, _act, send_next=_send_next)
        torch = _torch()
        dg, x = _prepare(self, input, self.inChannels, "SAGEConv")
        ctx = dg.ctx
        agg = self.aggregate(dg, x)
        out = torch.empty((input.numNodes, self.outChannels), dtype=torch.float32, device=x.device)
        act = None if self.normalize else _act
        code, param = _act_code(act)
        ctx.call("bgnn_sage_linear", ptr(agg), ptr(x), ptr(self.p("lin_neighbor")),
                 ptr(self.p("lin_self")), input.numNodes, self.inChannels, self.outChannels,
                 ptr(self.p("bias")), code, param, ptr(out))
        if self.normalize:
            ctx.call("bgnn_l2_normalize_rows", ptr(out), input.numNodes, self.outChannels)
            if _act is not None:
                code, param = _act_code(_act)
                ctx.call("bgnn_activation_dev", code, param, ptr(out), out.numel(), ptr(out))
        return input.withFeatures(out)

    forwardAsync = forward

    def backward(self, input: GraphData, grad_out, _act=None, output=None) -> dict:
        """Gradients of forward(input, _act) for an upstream gradient
        grad_out [N, out]: {"x", "lin_neighbor", "lin_self", "bias"} (sum,
        mean and max aggregators, no L2 normalisation).  Each forward step's
        adjoint: ReLU's mask, the broadcast bias reduction, Variable.matmul's
        backward for both products (variable.ts:213-235), and the message
        passing's edge-ordered scatter over the sources
        (bgnn_aggregate_backward); grad x = f32(x-path + message-path)."""
        if self.aggregator == "pool" or self.normalize:
            raise NotImplementedError("backward of the pool aggregator / L2 normalisation")
        torch = _torch()
        dg, x = _prepare(self, input, self.inChannels, "SAGEConv")
        ctx = dg.ctx
        if _act not in (None, "none") and output is None:
            output = self.forward(input, _act=_act).x
        g = _pre_activation_grad(ctx, grad_out, output, _act)
        agg = self.aggregate(dg, x)
        grads = {}
        if self.useBias:
            grads["bias"] = _bias_backward(ctx, g)
        gagg, grads["lin_neighbor"] = _matmul_backward(ctx, agg, self.p("lin_neighbor"), g)
        gx = torch.empty_like(x)
        ctx.call("bgnn_aggregate_backward", dg.h, _lib.AGGR[self.aggregator], ptr(x), ptr(gagg),
                 self.inChannels, ptr(gx))
        if self.rootWeight:
            gself, grads["lin_self"] = _matmul_backward(ctx, x, self.p("lin_self"), g)
            ctx.call("bgnn_add_dev", ptr(gself), ptr(gx), gx.numel(), ptr(gx))
        grads["x"] = gx
        return grads


class GINConv(Module):
    """src/layers/gin.ts:41-319 (2-layer MLP)."""

    def __init__(self, config: Optional[dict] = None, **kw):
        super().__init__()
        cfg = dict(config or {})
        cfg.update(kw)
        self.inChannels = int(cfg["inChannels"])
        self.outChannels = int(cfg["outChannels"])
        self.hiddenChannels = int(cfg.get("hiddenChannels", self.outChannels))
        self.trainEpsilon = bool(cfg.get("trainEpsilon", True))
        self.useBias = bool(cfg.get("bias", True))
        self.numLayers = int(cfg.get("numLayers", 2))
        eps = _torch().tensor([float(cfg.get("epsilon", 0.0))], dtype=_torch().float32)
        if self.trainEpsilon:
            self.registerParameter("epsilon", eps)
        else:
            self.registerBuffer("epsilon", eps)
        s1 = np.sqrt(2.0 / (self.inChannels + self.hiddenChannels))
        self.registerParameter("mlp_weight1", _param((self.inChannels, self.hiddenChannels), s1))
        if self.useBias:
            self.registerParameter("mlp_bias1", _param((self.hiddenChannels,), zeros=True))
        s2 = np.sqrt(2.0 / (self.hiddenChannels + self.outChannels))
        self.registerParameter("mlp_weight2", _param((self.hiddenChannels, self.outChannels), s2))
        if self.useBias:
            self.registerParameter("mlp_bias2", _param((self.outChannels,), zeros=True))

    def _eps(self) -> float:
        # read back once per parameter tensor (a host read inside a forward
        # would also stall the stream and break CUDA-graph capture)
        t = self.p("epsilon") if self.trainEpsilon else self._buffers["epsilon"]
        cached = getattr(self, "_eps_cache", None)
        if cached is not None and cached[0] is t:
            return cached[1]
        v = float(np.float32(t.detach().cpu().numpy().reshape(-1)[0]))
        self._eps_cache = (t, v)
        return v

    def forward(self, input: GraphData, _act=None) -> GraphData:
        torch = _torch()
        dg, x = _prepare(self, input, self.inChannels, "GINConv")
        ctx = dg.ctx
        comb = torch.empty((input.numNodes, self.inChannels), dtype=torch.float32, device=x.device)
        ctx.call("bgnn_gin_aggregate", dg.h, ptr(x), self.inChannels, self._eps(), ptr(comb))
        hid = _linear(ctx, comb, self.p("mlp_weight1"), self.p("mlp_bias1"), act="relu_max")
        out = _linear(ctx, hid, self.p("mlp_weight2"), self.p("mlp_bias2"), act=_act)
        return input.withFeatures(out)

    forwardAsync = forward


# ---- activations and containers (src/nn/activation.ts, module.ts) ----------
class _Act(Module):
    act = None
    param = 0.0

    def forward(self, input):
        torch = _torch()
        x = input.x_device() if isinstance(input, GraphData) else input
        ctx = get_context(x.device.index)
        out = torch.empty_like(x)
        ctx.call("bgnn_activation_dev", _lib.ACT[self.act], self.param, ptr(x), x.numel(), ptr(out))
        return input.withFeatures(out) if isinstance(input, GraphData) else out


class ReLU(_Act):
    """ReLU module -> Tensor.relu -> wasmRelu (x > 0 ? x : 0)."""
    act = "relu"


class ELU(_Act):
    act = "elu"

    def __init__(self, alpha: float = 1.0):
        super().__init__()
        self.param = float(alpha)


class LeakyReLU(_Act):
    act = "leaky_relu"

    def __init__(self, negativeSlope: float = 0.01):
        super().__init__()
        self.param = float(negativeSlope)


_FUSABLE = [GCNConv, GATConv, SAGEConv, GINConv]


def register_fusable(cls):
    """Mark a module whose forward(x, _act=(name, param)) applies an
    elementwise activation in its own epilogue."""
    if cls not in _FUSABLE:
        _FUSABLE.append(cls)
    return cls


class Sequential(Module):
    """src/nn/module.ts:144-178.  A layer (conv or Linear) followed by an
    elementwise activation module runs the activation in the layer's epilogue
    (same operations on the same stored values, one pass).  Takes the modules
    as a list (the reference's form) or as separate arguments."""

    def __init__(self, *modules):
        super().__init__()
        if len(modules) == 1 and isinstance(modules[0], (list, tuple)):
            modules = tuple(modules[0])
        for i, m in enumerate(modules):
            self.registerModule(str(i), m)

    def add(self, module):
        self.registerModule(str(len(self._modules)), module)

    @property
    def length(self) -> int:
        return len(self._modules)

    def __len__(self):
        return len(self._modules)

    def forward(self, input):
        mods = list(self._modules.values())
        i = 0
        x = input
        while i < len(mods):
            m = mods[i]
            nxt = mods[i + 1] if i + 1 < len(mods) else None
            if isinstance(m, tuple(_FUSABLE)) and isinstance(nxt, _Act):
                x = m.forward(x, _act=(nxt.act, nxt.param))
                i += 2
            else:
                x = m.forward(x)
                i += 1
        return x


def global_sum_pool(graph: GraphData, num_graphs: Optional[int] = None):
    """g[b,:] = sum of node rows with batch == b, in node order (no reference
    counterpart: the reference has no readout)."""
    torch = _torch()
    x = graph.x_device()
    ctx = get_context(x.device.index)
    if graph.batch is None:
        batch = torch.zeros(graph.numNodes, dtype=torch.int32, device=x.device)
        b = 1
    else:
        bnp = np.asarray(graph.batch, np.uint32)
        b = int(num_graphs if num_graphs is not None else (int(bnp.max()) + 1 if bnp.size else 0))
        batch, seg = _batch_device(graph, x.device, b)
        if seg is not None:  # graphs' nodes contiguous (batchGraphs): segmented sums
            out = torch.empty((b, graph.numFeatures), dtype=torch.float32, device=x.device)
            ctx.call("bgnn_segment_sum", ptr(x), graph.numFeatures, ptr(seg), b, ptr(out))
            return out
    out = torch.empty((b, graph.numFeatures), dtype=torch.float32, device=x.device)
    ctx.call("bgnn_sum_pool", ptr(x), graph.numNodes, graph.numFeatures, ptr(batch), b, ptr(out))
    return out


def _batch_device(graph: GraphData, device, num_graphs: int):
    """(batch vector, segment offsets or None) on the device, built once and
    kept with the graph's device structure (shared by every withFeatures
    copy).  Offsets exist when the batch vector is non-decreasing and within
    num_graphs, i.e. every graph's nodes are contiguous."""
    torch = _torch()
    dg = graph.device_graph(device.index)
    key = (str(device), int(num_graphs))
    cached = getattr(dg, "_batch_dev", None)
    if cached is not None and cached[0] == key:
        return cached[1], cached[2]
    bnp = np.asarray(graph.batch, np.uint32)
    t = torch.from_numpy(bnp.view(np.int32)).to(device)
    seg = None
    if bnp.size == 0 or (np.all(bnp[1:] >= bnp[:-1]) and int(bnp[-1]) < num_graphs):
        offs = np.searchsorted(bnp, np.arange(num_graphs + 1), side="left").astype(np.uint32)
        seg = torch.from_numpy(offs.view(np.int32)).to(device)
    dg._batch_dev = (key, t, seg)
    return t, seg
