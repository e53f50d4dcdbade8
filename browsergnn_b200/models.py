"""The reference's model zoo (src/models/) on the cuda backend.

StudentMasteryPredictor, LearningPathRecommender and ConceptPrerequisiteMapper
with the reference's configuration keys and defaults, parameter names (so a
state dict saved by the reference loads unchanged), forward passes and helper
methods.  Every tensor step runs on the GPU: the graph's CSR is built once and
cached on the GraphData, activations run in the producing layer's epilogue,
and only the final scores come back to the host for the list-building helpers
(predict, recommend, discoverPrerequisites ...).

The reference's forward passes are async (they await Sequential.forward);
these are synchronous and return CUDA tensors.  Random parts differ by design:
parameter initialisation and the sample graphs' features come from seeded
numpy generators, and training-mode dropout from the counter-based device
generator, instead of the unseeded Math.random().
"""
from __future__ import annotations

import sys
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import _lib
from .backend import get_context, ptr
from .graph import GraphData
from .layers import GATConv, GCNConv, GINConv, Module, SAGEConv, _param, _torch, next_dropout_seed
from .nn import ELU, Dropout, LeakyReLU, Linear, ReLU, Sequential, Sigmoid, Softmax

__all__ = ["StudentMasteryPredictor", "LearningPathRecommender", "ConceptPrerequisiteMapper"]

_sample_rng = np.random.default_rng(0xB200_5A)


def _cfg(config, kw, defaults):
    cfg = dict(config or {})
    cfg.update(kw)
    out = dict(defaults)
    for k, v in cfg.items():
        if v is not None:
            out[k] = v
    return out


def _dropout(mod: Dropout, x):
    """Dropout.forward on a tensor (identity in eval mode)."""
    return mod.forward(x)


def _add(a, b):
    """residual f32(a + b) (StudentMasteryPredictor.ts:180-187)."""
    torch = _torch()
    out = torch.empty_like(a)
    get_context(a.device.index).call("bgnn_add_dev", ptr(a), ptr(b), a.numel(), ptr(out))
    return out


def _host_edges(graph: GraphData) -> np.ndarray:
    return graph._host_edges()


def _graph(x, n, f, src, dst) -> GraphData:
    ei = np.asarray(list(src) + list(dst), dtype=np.uint32)
    return GraphData(x=np.asarray(x, np.float32), numNodes=n, numFeatures=f, edgeIndex=ei,
                     numEdges=len(src))


# ---------------------------------------------------------------------------
class StudentMasteryPredictor(Module):
    """src/models/StudentMasteryPredictor.ts:80-309.

    inputProj (Linear) -> ReLU -> numLayers x (GCN or GAT -> ReLU -> Dropout
    [-> + residual when widths match]) -> outputHead (Linear -> Sigmoid)."""

    def __init__(self, config: Optional[dict] = None, **kw):
        super().__init__()
        self.config = _cfg(config, kw, dict(hiddenDim=64, numLayers=2, useAttention=False,
                                            numHeads=4, dropout=0.1, residual=True))
        c = self.config
        c["inputFeatures"] = int(c["inputFeatures"])
        hid = int(c["hiddenDim"])
        self.inputProj = Linear(inFeatures=c["inputFeatures"], outFeatures=hid)
        self.registerModule("inputProj", self.inputProj)
        self.gnnLayers: List[Module] = []
        for i in range(int(c["numLayers"])):
            if c["useAttention"]:
                layer = GATConv(inChannels=hid, outChannels=hid // int(c["numHeads"]),
                                heads=int(c["numHeads"]), concat=True, dropout=c["dropout"])
            else:
                layer = GCNConv(inChannels=hid, outChannels=hid)
            self.gnnLayers.append(layer)
            self.registerModule(f"gnn_{i}", layer)
        self.dropout = Dropout(c["dropout"])
        self.registerModule("dropout", self.dropout)
        self.outputHead = Sequential([Linear(inFeatures=hid, outFeatures=1), Sigmoid()])
        self.registerModule("outputHead", self.outputHead)

    def forward(self, graph: GraphData):
        """[numNodes, 1] mastery probabilities (StudentMasteryPredictor.ts:159-197)."""
        h = self.inputProj.forward(graph.x_device(), _act=("relu", 0.0))
        wg = graph.withFeatures(h)
        for layer in self.gnnLayers:
            prev = wg.x
            wg = layer.forward(wg, _act=("relu", 0.0))
            new = _dropout(self.dropout, wg.x)
            if self.config["residual"] and prev.shape[1] == new.shape[1]:
                new = _add(new, prev)
            wg = wg.withFeatures(new)
        return self.outputHead.forward(wg.x)

    forwardAsync = forward

    def predict(self, graph: GraphData) -> Dict[str, list]:
        """StudentMasteryPredictor.ts:205-228 (eval mode, threshold 0.7)."""
        self.eval()
        out = self.forward(graph).reshape(-1).cpu().numpy()
        mastery = [float(out[i]) if i < out.size else 0.0 for i in range(graph.numNodes)]
        predictions = [{"nodeIndex": i, "score": s, "mastered": s >= 0.7}
                       for i, s in enumerate(mastery)]
        return {"mastery": mastery, "predictions": predictions}

    def getWeakConcepts(self, graph: GraphData, topK: int = 5):
        """StudentMasteryPredictor.ts:235-249: lowest scores first (stable)."""
        preds = self.predict(graph)["predictions"]
        preds.sort(key=lambda p: p["score"])
        return [{"nodeIndex": p["nodeIndex"], "score": p["score"]} for p in preds[:topK]]

    @staticmethod
    def createSampleGraph(numConcepts: int = 10, rng=None) -> GraphData:
        """StudentMasteryPredictor.ts:254-301: a chain with cross-links every
        third node; features [embedding(8), difficulty, attempts, success]."""
        rng = rng or _sample_rng
        f = 11
        x = np.zeros((numConcepts, f), np.float32)
        for i in range(numConcepts):
            x[i, :8] = rng.random(8) * 2 - 1
            x[i, 8] = rng.random()
            x[i, 9] = rng.random()
            x[i, 10] = rng.random()
        src, dst = [], []
        for i in range(numConcepts - 1):
            src += [i, i + 1]
            dst += [i + 1, i]
        for i in range(0, numConcepts, 3):
            if i + 2 < numConcepts:
                src += [i, i + 2]
                dst += [i + 2, i]
        return _graph(x, numConcepts, f, src, dst)

    def toString(self) -> str:
        t = "GAT" if self.config["useAttention"] else "GCN"
        return (f"StudentMasteryPredictor({self.config['inputFeatures']} -> {t}x"
                f"{self.config['numLayers']} -> mastery)")

    __repr__ = toString


# ---------------------------------------------------------------------------
class LearningPathRecommender(Module):
    """src/models/LearningPathRecommender.ts:67-380.

    inputProj (Linear -> LeakyReLU(0.1)) -> numLayers x (SAGE(normalize) or
    GIN -> LeakyReLU(0.1) -> Dropout, not after the last) -> scoringHead
    (Linear -> ReLU -> Linear) -> optional mastery mask -> softmax over nodes."""

    def __init__(self, config: Optional[dict] = None, **kw):
        super().__init__()
        self.config = _cfg(config, kw, dict(hiddenDim=64, numLayers=3, aggregator="mean",
                                            useGIN=False, dropout=0.1, normalizeScores=True))
        c = self.config
        c["inputFeatures"] = int(c["inputFeatures"])
        hid = int(c["hiddenDim"])
        if hid % 2:
            # the reference sizes the first head Linear with hiddenDim / 2, a
            # fractional length that Float32Array rejects
            raise ValueError(f"Invalid typed array length: {hid * hid / 2}")
        self.inputProj = Sequential([Linear(inFeatures=c["inputFeatures"], outFeatures=hid),
                                     LeakyReLU(0.1)])
        self.registerModule("inputProj", self.inputProj)
        self.gnnLayers: List[Module] = []
        for i in range(int(c["numLayers"])):
            if c["useGIN"]:
                layer = GINConv(inChannels=hid, outChannels=hid, hiddenChannels=hid * 2,
                                trainEpsilon=True)
            else:
                layer = SAGEConv(inChannels=hid, outChannels=hid, aggregator=c["aggregator"],
                                 normalize=True)
            self.gnnLayers.append(layer)
            self.registerModule(f"gnn_{i}", layer)
        self.dropout = Dropout(c["dropout"])
        self.registerModule("dropout", self.dropout)
        self.scoringHead = Sequential([Linear(inFeatures=hid, outFeatures=hid // 2), ReLU(),
                                       Linear(inFeatures=hid // 2, outFeatures=1)])
        self.registerModule("scoringHead", self.scoringHead)
        self.softmax = Softmax()

    def forward(self, graph: GraphData, maskMastered: Optional[Sequence[bool]] = None):
        """[numNodes, 1] scores (LearningPathRecommender.ts:173-225)."""
        torch = _torch()
        h = self.inputProj.forward(graph.x_device())
        wg = graph.withFeatures(h)
        n_layers = len(self.gnnLayers)
        for i, layer in enumerate(self.gnnLayers):
            if i < n_layers - 1:
                wg = layer.forward(wg, _act=("leaky_relu", 0.1))
                wg = wg.withFeatures(_dropout(self.dropout, wg.x))
            else:
                wg = layer.forward(wg)
        scores = self.scoringHead.forward(wg.x).contiguous()
        n = graph.numNodes
        mask_t = None
        if maskMastered is not None:
            m = np.zeros(n, np.uint8)
            lim = min(n, len(maskMastered))
            m[:lim] = np.asarray([bool(v) for v in maskMastered[:lim]], np.uint8)
            mask_t = torch.from_numpy(m).to(scores.device)
        if self.config["normalizeScores"]:
            out = torch.empty_like(scores)
            get_context(scores.device.index).call(
                "bgnn_softmax_rows", ptr(scores), 1, n, ptr(mask_t), -1e9, 0, ptr(out))
            return out
        if mask_t is not None:
            scores = scores.masked_fill(mask_t.bool().reshape(n, 1), -1e9)
        return scores

    forwardAsync = forward

    def recommend(self, graph: GraphData, masteredNodes: Sequence[int] = (), topK: int = 5):
        """LearningPathRecommender.ts:232-275."""
        self.eval()
        mask = [False] * graph.numNodes
        for idx in masteredNodes:
            mask[int(idx)] = True
        scores = self.forward(graph, mask).reshape(-1).cpu().numpy()
        all_scores = [float(scores[i]) for i in range(graph.numNodes)]
        scored = [{"nodeIndex": i, "score": s} for i, s in enumerate(all_scores) if not mask[i]]
        scored.sort(key=lambda p: -p["score"])
        recs = [dict(p, rank=r + 1) for r, p in enumerate(scored[:topK])]
        return {"recommendations": recs, "allScores": all_scores}

    def getLearningPath(self, graph: GraphData, masteredNodes: Sequence[int],
                        goalNodes: Sequence[int], maxSteps: int = 20):
        """LearningPathRecommender.ts:283-318: greedy one-step recommendations
        until every goal is mastered."""
        path, path_scores = [], []
        mastered = list(dict.fromkeys(int(v) for v in masteredNodes))
        goals = set(int(v) for v in goalNodes)
        for _ in range(maxSteps):
            if all(g in mastered for g in goals):
                break
            recs = self.recommend(graph, mastered, 1)["recommendations"]
            if not recs:
                break
            nxt = recs[0]
            path.append(nxt["nodeIndex"])
            path_scores.append(nxt["score"])
            if nxt["nodeIndex"] not in mastered:
                mastered.append(nxt["nodeIndex"])
        return {"path": path, "scores": path_scores}

    @staticmethod
    def createSampleCurriculum(numConcepts: int = 15, rng=None) -> GraphData:
        """LearningPathRecommender.ts:325-374: a binary tree with sibling links."""
        rng = rng or _sample_rng
        f = 11
        x = np.zeros((numConcepts, f), np.float32)
        for i in range(numConcepts):
            x[i, :8] = rng.random(8) * 2 - 1
            x[i, 8] = i / numConcepts
            x[i, 9] = 0.3 + rng.random() * 0.5
            x[i, 10] = rng.random() * 0.3
        src, dst = [], []
        for i in range(1, numConcepts):
            parent = (i - 1) // 2
            src += [parent, i]
            dst += [i, parent]
            sibling = i + (-1 if i % 2 == 0 else 1)
            if 0 < sibling < numConcepts:
                src.append(i)
                dst.append(sibling)
        return _graph(x, numConcepts, f, src, dst)

    def toString(self) -> str:
        t = "GIN" if self.config["useGIN"] else "SAGE"
        return (f"LearningPathRecommender({self.config['inputFeatures']} -> {t}x"
                f"{self.config['numLayers']} -> scores)")

    __repr__ = toString


# ---------------------------------------------------------------------------
class ConceptPrerequisiteMapper(Module):
    """src/models/ConceptPrerequisiteMapper.ts:78-508.

    encode: inputProj (Linear -> ELU -> Dropout) -> numLayers x (GAT or GCN
    -> ELU -> Dropout, not after the last); link scores by dot product,
    bilinear form or an MLP over [src, tgt, src*tgt], each through a sigmoid.

    The reference's 'mlp' scorer calls the async Sequential.forward without
    awaiting it and reads ``.data`` off the returned Promise, so it throws a
    TypeError for every pair; here it computes the network the code
    describes (eval mode)."""

    def __init__(self, config: Optional[dict] = None, **kw):
        super().__init__()
        self.config = _cfg(config, kw, dict(hiddenDim=64, numLayers=2, useAttention=True,
                                            numHeads=4, dropout=0.2, linkPredictor="mlp"))
        c = self.config
        c["inputFeatures"] = int(c["inputFeatures"])
        hid = int(c["hiddenDim"])
        self.inputProj = Sequential([Linear(inFeatures=c["inputFeatures"], outFeatures=hid),
                                     ELU(), Dropout(c["dropout"])])
        self.registerModule("inputProj", self.inputProj)
        self.gnnLayers: List[Module] = []
        for i in range(int(c["numLayers"])):
            if c["useAttention"]:
                layer = GATConv(inChannels=hid, outChannels=hid // int(c["numHeads"]),
                                heads=int(c["numHeads"]), concat=True, dropout=c["dropout"])
            else:
                layer = GCNConv(inChannels=hid, outChannels=hid)
            self.gnnLayers.append(layer)
            self.registerModule(f"gnn_{i}", layer)
        self.dropout = Dropout(c["dropout"])
        self.registerModule("dropout", self.dropout)
        self.bilinearWeight = None
        self.linkPredictor = None
        if c["linkPredictor"] == "bilinear":
            self.registerParameter("bilinearWeight", _param((hid, hid), np.sqrt(2.0 / hid)))
            self.bilinearWeight = True
        elif c["linkPredictor"] == "mlp":
            self.linkPredictor = Sequential([Linear(inFeatures=hid * 3, outFeatures=hid), ReLU(),
                                             Dropout(c["dropout"] / 2),
                                             Linear(inFeatures=hid, outFeatures=1)])
            self.registerModule("linkPredictor", self.linkPredictor)
        self.sigmoid = Sigmoid()

    def encode(self, graph: GraphData):
        """Node embeddings [numNodes, hidden] (ConceptPrerequisiteMapper.ts:189-215)."""
        h = self.inputProj.forward(graph.x_device())
        wg = graph.withFeatures(h)
        n_layers = len(self.gnnLayers)
        for i, layer in enumerate(self.gnnLayers):
            if i < n_layers - 1:
                wg = layer.forward(wg, _act=("elu", 1.0))
                wg = wg.withFeatures(_dropout(self.dropout, wg.x))
            else:
                wg = layer.forward(wg)
        return wg.x

    forward = encode
    forwardAsync = encode

    def predictLinks(self, embeddings, srcNodes: Sequence[int], tgtNodes: Sequence[int]):
        """Sigmoid link scores for each (src, tgt) pair, as Python floats
        (ConceptPrerequisiteMapper.ts:224-295)."""
        torch = _torch()
        n_pairs = len(srcNodes)
        if n_pairs == 0:
            return []
        mode = self.config["linkPredictor"]
        if mode not in ("dot", "bilinear", "mlp"):
            return [0.0] * n_pairs
        emb = embeddings.contiguous()
        dev = emb.device
        ctx = get_context(dev.index)
        self.to_device(dev.index)
        src = torch.from_numpy(np.asarray(srcNodes, np.int64).astype(np.uint32).view(np.int32))
        tgt = torch.from_numpy(np.asarray(tgtNodes, np.int64).astype(np.uint32).view(np.int32))
        src, tgt = src.to(dev), tgt.to(dev)
        out = torch.empty(n_pairs, dtype=torch.float64, device=dev)
        wb = w1 = b1 = w2 = b2 = None
        if mode == "bilinear":
            wb = self.p("bilinearWeight")
        elif mode == "mlp":
            mods = list(self.linkPredictor._modules.values())
            if self._training and mods[2].p > 0:
                raise NotImplementedError("the mlp link scorer runs in eval mode; call eval()")
            w1, b1 = mods[0].p("weight"), mods[0].p("bias")
            w2, b2 = mods[3].p("weight"), mods[3].p("bias")
        n, d = int(emb.shape[0]), int(emb.shape[1])
        ctx.call("bgnn_link_scores", ptr(emb), n, d, ptr(src), ptr(tgt), n_pairs,
                 _lib.LINK[mode], ptr(wb), ptr(w1), ptr(b1), ptr(w2), ptr(b2), ptr(out))
        ctx.synchronize()
        return [float(v) for v in out.cpu().numpy()]

    def predictAllLinks(self, graph: GraphData, candidatePairs: Optional[dict] = None):
        """ConceptPrerequisiteMapper.ts:308-349: every ordered pair i != j
        (i outer) unless candidate pairs are given."""
        emb = self.encode(graph)
        if candidatePairs is not None:
            src = list(candidatePairs["src"])
            tgt = list(candidatePairs["tgt"])
        else:
            n = graph.numNodes
            src = [i for i in range(n) for j in range(n) if i != j]
            tgt = [j for i in range(n) for j in range(n) if i != j]
        scores = self.predictLinks(emb, src, tgt)
        pairs = [{"src": s, "tgt": t, "score": sc} for s, t, sc in zip(src, tgt, scores)]
        return {"embeddings": emb, "scores": scores, "pairs": pairs}

    def discoverPrerequisites(self, graph: GraphData, threshold: float = 0.7, topK: int = 20):
        """ConceptPrerequisiteMapper.ts:357-388: high-scoring pairs that are
        not edges yet, best first."""
        self.eval()
        ei = _host_edges(graph)
        e = graph.numEdges
        existing = {f"{int(ei[i])}->{int(ei[e + i])}" for i in range(e)}
        pairs = self.predictAllLinks(graph)["pairs"]
        new = [p for p in pairs if f"{p['src']}->{p['tgt']}" not in existing]
        new = [p for p in new if p["score"] >= threshold]
        new.sort(key=lambda p: -p["score"])
        return {"newEdges": new[:topK], "existingEdges": existing}

    def findCriticalPath(self, graph: GraphData, startNode: int):
        """ConceptPrerequisiteMapper.ts:395-444: longest simple path from
        startNode by memoised depth-first search (host-side graph walk)."""
        ei = _host_edges(graph)
        e = graph.numEdges
        adj: Dict[int, List[int]] = {}
        for i in range(e):
            adj.setdefault(int(ei[i]), []).append(int(ei[e + i]))
        visited = set()
        memo: Dict[int, dict] = {}

        def dfs(node):
            if node in memo:
                return memo[node]
            if node in visited:
                return {"path": [node], "length": 0}
            visited.add(node)
            best_path, best_len = [node], 0
            for nxt in adj.get(node, []):
                r = dfs(nxt)
                if r["length"] + 1 > best_len:
                    best_len = r["length"] + 1
                    best_path = [node] + r["path"]
            visited.discard(node)
            res = {"path": best_path, "length": best_len}
            memo[node] = res
            return res

        old = sys.getrecursionlimit()
        sys.setrecursionlimit(max(old, 4 * graph.numNodes + 100))
        try:
            return dfs(int(startNode))
        finally:
            sys.setrecursionlimit(old)

    @staticmethod
    def createSampleConceptGraph(numConcepts: int = 12, rng=None) -> GraphData:
        """ConceptPrerequisiteMapper.ts:451-502: prerequisite chains of three
        plus cross-domain links; features [embedding(16), difficulty, domain(3)]."""
        rng = rng or _sample_rng
        f = 20
        x = np.zeros((numConcepts, f), np.float32)
        for i in range(numConcepts):
            x[i, :16] = rng.random(16) * 2 - 1
            x[i, 16] = i / numConcepts
            x[i, 17 + i % 3] = 1
        src, dst = [], []
        for i in range(0, numConcepts - 3, 3):
            src += [i, i + 1, i + 1, i + 2]
            dst += [i + 1, i + 2, i, i + 1]
        for d in range(3):
            src += [d, d + 3]
            dst += [d + 3, d]
        return _graph(x, numConcepts, f, src, dst)

    def toString(self) -> str:
        t = "GAT" if self.config["useAttention"] else "GCN"
        return (f"ConceptPrerequisiteMapper({self.config['inputFeatures']} -> {t}x"
                f"{self.config['numLayers']} -> {self.config['linkPredictor']})")

    __repr__ = toString
