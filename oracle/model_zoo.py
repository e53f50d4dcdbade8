"""CPU restatement of the reference's model zoo forward passes (eval mode).

TEST INFRASTRUCTURE ONLY: composes the C oracle's layer and module
restatements (oracle.py) in the order the reference's models call them, so
the GPU models can be checked end to end.  Parameters come as a dict keyed by
the reference's parameter names (namedParameters order is irrelevant here).

  student_mastery   src/models/StudentMasteryPredictor.ts:159-197
  learning_path     src/models/LearningPathRecommender.ts:173-225
  concept_encode    src/models/ConceptPrerequisiteMapper.ts:189-215
  concept_links     src/models/ConceptPrerequisiteMapper.ts:224-295
"""
from __future__ import annotations

import numpy as np

from . import oracle as o


def _gnn(kind, h, n, ei, e, P, prefix, hid, heads=4, act=None, dropout=0.0, seed=0):
    fin = h.shape[1]
    if kind == "gcn":
        out = o.gcn_forward(h, n, fin, ei, e, P[prefix + "weight"], P.get(prefix + "bias"), hid)
        return out.reshape(n, hid)
    if kind == "gat":
        c = hid // heads
        out = o.gat_forward(h, n, fin, ei, e, P[prefix + "weight"], P[prefix + "att_src"],
                            P[prefix + "att_dst"], P.get(prefix + "bias"), heads, c,
                            dropout=dropout, seed=seed)
        return out.reshape(n, heads * c)
    raise ValueError(kind)


def student_mastery(x, ei, e, P, num_layers=2, use_attention=False, heads=4, residual=True):
    """Linear -> ReLU -> (GCN|GAT -> ReLU [+ residual]) x L -> Linear -> Sigmoid."""
    n = x.shape[0]
    h = o.relu(o.linear(x, P["inputProj.weight"], P["inputProj.bias"]))
    hid = h.shape[1]
    for i in range(num_layers):
        prev = h
        out = _gnn("gat" if use_attention else "gcn", h, n, ei, e, P, f"gnn_{i}.", hid, heads)
        new = o.relu(out)
        if residual and prev.shape[1] == new.shape[1]:
            new = o.add(new, prev).reshape(new.shape)
        h = new
    y = o.linear(h, P["outputHead.0.weight"], P["outputHead.0.bias"])
    return o.sigmoid(y).reshape(n, 1)


def learning_path(x, ei, e, P, num_layers=3, aggregator="mean", use_gin=False, mask=None,
                  normalize_scores=True):
    """Linear -> LeakyReLU(0.1) -> (SAGE(normalize)|GIN [-> LeakyReLU(0.1)]) x L
    -> Linear -> ReLU -> Linear -> mask -> softmax over the nodes."""
    n = x.shape[0]
    h = o.leaky_relu(o.linear(x, P["inputProj.0.weight"], P["inputProj.0.bias"]), 0.1)
    hid = h.shape[1]
    for i in range(num_layers):
        pre = f"gnn_{i}."
        if use_gin:
            eps = float(np.float32(np.asarray(P[pre + "epsilon"]).reshape(-1)[0]))
            w1 = P[pre + "mlp_weight1"]
            out = o.gin_forward(h, n, hid, ei, e, eps, w1, P.get(pre + "mlp_bias1"),
                                w1.shape[1], P[pre + "mlp_weight2"], P.get(pre + "mlp_bias2"), hid)
        else:
            out = o.sage_forward(h, n, hid, ei, e, aggregator, P[pre + "lin_neighbor"],
                                 P.get(pre + "lin_self"), P.get(pre + "bias"), hid,
                                 normalize=True, pool_weight=P.get(pre + "pool_weight"),
                                 pool_bias=P.get(pre + "pool_bias"))
        h = out.reshape(n, hid)
        if i < num_layers - 1:
            h = o.leaky_relu(h, 0.1).reshape(n, hid)
    s = o.relu(o.linear(h, P["scoringHead.0.weight"], P["scoringHead.0.bias"]))
    s = o.linear(s.reshape(n, -1), P["scoringHead.2.weight"], P["scoringHead.2.bias"])
    s = s.reshape(-1).copy()
    if mask is not None:
        m = np.zeros(n, bool)
        m[: min(n, len(mask))] = np.asarray(mask[:n], bool)
        s[m] = np.float32(-1e9)
    if normalize_scores:
        s = o.softmax_rows(s.reshape(1, n))
    return s.reshape(n, 1)


def concept_encode(x, ei, e, P, num_layers=2, use_attention=True, heads=4):
    """Linear -> ELU -> (GAT|GCN [-> ELU]) x L."""
    n = x.shape[0]
    h = o.elu(o.linear(x, P["inputProj.0.weight"], P["inputProj.0.bias"]), 1.0)
    hid = h.shape[1]
    for i in range(num_layers):
        h = _gnn("gat" if use_attention else "gcn", h, n, ei, e, P, f"gnn_{i}.", hid, heads)
        if i < num_layers - 1:
            h = o.elu(h, 1.0).reshape(h.shape)
    return h


def concept_links(emb, src, tgt, P, mode):
    if mode == "dot":
        return o.link_scores(emb, src, tgt, "dot")
    if mode == "bilinear":
        return o.link_scores(emb, src, tgt, "bilinear", w_bilinear=P["bilinearWeight"])
    return o.link_scores(emb, src, tgt, "mlp", w1=P["linkPredictor.0.weight"],
                         b1=P["linkPredictor.0.bias"], w2=P["linkPredictor.3.weight"],
                         b2=P["linkPredictor.3.bias"])
