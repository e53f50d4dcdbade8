"""Seeded synthetic inputs for the five benchmark workloads.

The workloads mimic public datasets by shape only (none of them is on this
machine): a Cora-sized citation graph, an ogbn-products-sized R-MAT graph,
TU-style batched small graphs and a scale-24 R-MAT matrix.

R-MAT edges come from a counter-based hash (splitmix64), so the numpy
generator here and the CUDA generator (csrc/synth.cu, bgnn_synth_rmat) emit
the same edge list for the same seed.  Seeds are 0xB2000000 + workload id.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

M64 = (1 << 64) - 1
SEED_BASE = 0xB2000000
RMAT_ABC = (0.57, 0.19, 0.19)


def seed_for(workload: int) -> int:
    return SEED_BASE + int(workload)


# ---- counter-based hashing (identical to csrc/synth.cu) ----------------------
def splitmix64(x):
    """Vectorised splitmix64 on uint64 numpy arrays (wrapping arithmetic)."""
    x = np.asarray(x, dtype=np.uint64)
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        z = x
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def _sm64_int(x: int) -> int:
    x = (x + 0x9E3779B97F4A7C15) & M64
    z = x
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def _perm_params(seed: int, bits: int):
    s = _sm64_int(seed ^ 0x5045524D5045524D)
    mul, add = [], []
    for _ in range(4):
        s = _sm64_int(s)
        mul.append(s | 1)
        s = _sm64_int(s)
        add.append(s)
    mask = (1 << bits) - 1
    shift = max(1, (bits + 1) // 2)
    return mul, add, mask, shift


def permute_ids(ids: np.ndarray, n: int, seed: int) -> np.ndarray:
    """Seeded bijection of [0, n) (4 multiply-xorshift-add rounds on the
    next power of two, cycle-walking back into range)."""
    bits = max(1, int(np.ceil(np.log2(n))) if n > 1 else 1)
    while (1 << bits) < n:
        bits += 1
    mul, add, mask, shift = _perm_params(seed, bits)
    m = np.uint64(mask)
    sh = np.uint64(shift)

    def f(x):
        with np.errstate(over="ignore"):
            for r in range(4):
                x = (x * np.uint64(mul[r])) & m
                x = x ^ (x >> sh)
                x = (x + np.uint64(add[r])) & m
        return x

    y = f(np.asarray(ids, dtype=np.uint64))
    bad = y >= np.uint64(n)
    while bad.any():
        y[bad] = f(y[bad])
        bad = y >= np.uint64(n)
    return y.astype(np.uint32)


def rmat_edges(scale: int, n: int, e: int, seed: int, abc=RMAT_ABC, permute: bool = True,
               chunk: int = 1 << 20) -> np.ndarray:
    """R-MAT edge list [src(e) | dst(e)] (uint32), duplicates and self-loops
    kept, ids >= n rejected, first e accepted attempts in order."""
    a, b, c = abc
    ab, abc_ = a + b, a + b + c
    key0 = np.uint64(_sm64_int(seed))
    srcs, dsts, have, t0 = [], [], 0, 0
    while have < e:
        t = np.arange(t0, t0 + chunk, dtype=np.uint64)
        s = np.zeros(chunk, np.uint64)
        d = np.zeros(chunk, np.uint64)
        for lvl in range(scale):
            with np.errstate(over="ignore"):
                h = splitmix64(key0 + t * np.uint64(scale) + np.uint64(lvl))
            u = (h >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)
            rb = (u >= ab).astype(np.uint64)
            cb = (((u >= a) & (u < ab)) | (u >= abc_)).astype(np.uint64)
            s = (s << np.uint64(1)) | rb
            d = (d << np.uint64(1)) | cb
        ok = (s < n) & (d < n)
        srcs.append(s[ok].astype(np.uint32))
        dsts.append(d[ok].astype(np.uint32))
        have += int(ok.sum())
        t0 += chunk
    src = np.concatenate(srcs)[:e]
    dst = np.concatenate(dsts)[:e]
    if permute:
        src = permute_ids(src, n, seed)
        dst = permute_ids(dst, n, seed)
    return np.concatenate([src, dst]).astype(np.uint32)


def rmat_edges_gpu(scale: int, n: int, e: int, seed: int, abc=RMAT_ABC, permute: bool = True,
                   device: Optional[int] = None):
    """Same edge list as rmat_edges, generated on the GPU (int32 tensor holding
    uint32 bit patterns)."""
    import torch

    from .backend import get_context, ptr

    ctx = get_context(device)
    out = torch.empty(2 * e, dtype=torch.int32, device=f"cuda:{ctx.device}")
    ctx.call("bgnn_synth_rmat", seed, scale, n, e, abc[0], abc[1], abc[2], int(permute), ptr(out))
    return out


# ---- other generators (host) -------------------------------------------------
def ba_graph(n: int, m: int, target_undirected: int, seed: int) -> np.ndarray:
    """Barabasi-Albert (m edges per new node, preferential attachment), trimmed
    by a seeded draw to exactly `target_undirected` unique undirected edges,
    both directions emitted: [u.., v.. | v.., u..]."""
    rng = np.random.default_rng(seed)
    edges = []
    repeated = list(range(m))
    targets = list(range(m))
    for v in range(m, n):
        for t in set(targets):
            edges.append((min(v, t), max(v, t)))
        repeated.extend(targets)
        repeated.extend([v] * m)
        chosen = set()
        while len(chosen) < m:
            chosen.add(repeated[int(rng.integers(len(repeated)))])
        targets = list(chosen)
    uniq = sorted(set(edges))
    if len(uniq) > target_undirected:
        keep = np.sort(rng.choice(len(uniq), size=target_undirected, replace=False))
        uniq = [uniq[i] for i in keep]
    u = np.array([p[0] for p in uniq], np.uint32)
    v = np.array([p[1] for p in uniq], np.uint32)
    return np.concatenate([u, v, v, u]).astype(np.uint32)


def er_batch(num_graphs: int, nmin: int, nmax: int, p: float, seed: int):
    """Ordered-pair Erdos-Renyi graphs (randomGraph semantics, graph.ts:543-549:
    i != j, each pair kept with probability p), batched block-diagonally
    (batchGraphs, graph.ts:439-492).  Returns (edge_index, sizes)."""
    rng = np.random.default_rng(seed)
    sizes = rng.integers(nmin, nmax + 1, size=num_graphs)
    srcs, dsts, off = [], [], 0
    for n in sizes:
        n = int(n)
        keep = rng.random((n, n)) < p
        np.fill_diagonal(keep, False)
        i, j = np.nonzero(keep)  # row-major = the reference's i/j loop order
        srcs.append((i + off).astype(np.uint32))
        dsts.append((j + off).astype(np.uint32))
        off += n
    return np.concatenate(srcs + dsts).astype(np.uint32), sizes.astype(np.int64)


def normal_features(n: int, f: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed ^ 0xFEA7)
    return rng.standard_normal((n, f), dtype=np.float32)


def bernoulli_features(n: int, f: int, p: float, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed ^ 0xFEA7)
    return (rng.random((n, f)) < p).astype(np.float32)


def one_hot_labels(n: int, classes: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed ^ 0x1AB)
    lab = rng.integers(0, classes, size=n)
    x = np.zeros((n, classes), np.float32)
    x[np.arange(n), lab] = 1.0
    return x


def glorot(fan_in: int, fan_out: int, rng: np.random.Generator, shape=None) -> np.ndarray:
    lim = np.sqrt(6.0 / (fan_in + fan_out))
    shape = shape or (fan_in, fan_out)
    return rng.uniform(-lim, lim, size=shape).astype(np.float32)


# ---- the five workloads -------------------------------------------------------
@dataclass
class Workload:
    name: str
    num_nodes: int
    edge_index: np.ndarray  # host uint32 [src | dst]
    num_edges: int
    x: np.ndarray
    extra: dict


def gcn_cora_like(seed: Optional[int] = None) -> Workload:
    s = seed_for(1) if seed is None else seed
    n = 2708
    ei = ba_graph(n, 2, 5278, s)
    x = bernoulli_features(n, 1433, 0.013, s)
    return Workload("gcn-2708n-10556e-1433f", n, ei, ei.size // 2, x, {})


def gat_rmat(seed: Optional[int] = None, n: int = 20000, e: int = 200000, f: int = 500) -> Workload:
    s = seed_for(2) if seed is None else seed
    scale = max(1, int(np.ceil(np.log2(n))))
    ei = rmat_edges(scale, n, e, s)
    x = normal_features(n, f, s)
    return Workload(f"gat-rmat-{n}n-{e}e-{f}f", n, ei, e, x, {"scale": scale})


def gin_batch(seed: Optional[int] = None, num_graphs: int = 4096) -> Workload:
    s = seed_for(3) if seed is None else seed
    ei, sizes = er_batch(num_graphs, 10, 40, 0.15, s)
    n = int(sizes.sum())
    x = one_hot_labels(n, 32, s)
    batch = np.repeat(np.arange(num_graphs, dtype=np.uint32), sizes)
    return Workload(f"gin-er-{num_graphs}g-{n}n-{ei.size // 2}e", n, ei, ei.size // 2, x,
                    {"batch": batch, "num_graphs": num_graphs})


SAGE_N, SAGE_E, SAGE_SCALE = 2_450_000, 62_000_000, 22
SPMM_SCALE, SPMM_E = 24, 1 << 28


def sage_rmat_small(frac: int = 64, seed: Optional[int] = None) -> Workload:
    """The SAGE workload scaled down by `frac` (same average degree, R-MAT
    skew and widths) for CPU timing and parity checks."""
    s = seed_for(4) if seed is None else seed
    n = SAGE_N // frac
    e = SAGE_E // frac
    scale = max(1, int(np.ceil(np.log2(n))))
    ei = rmat_edges(scale, n, e, s)
    x = normal_features(n, 100, s)
    return Workload(f"sage-rmat-{n}n-{e}e", n, ei, e, x, {"scale": scale})
