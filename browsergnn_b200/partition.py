"""The row-partition plan on the host (numpy), the same plan the device
builds (csrc/partition.cu, bgnn_part_create / bgnn_part_create_csr).

The reference has no multi-device code; the B200 backend runs a layer on
several GPUs by giving rank r the contiguous rows [lo, hi) of a square
graph and exchanging the halo rows its edges read.  Every rank derives the
same plan from the same graph, so the plan needs no communication:

* bounds: rank r starts at the first row j with row_ptr[j] + j >=
  r * (E + N) // world;
* halo: the sorted unique columns of the local rows' entries outside
  [lo, hi) -- sorted by id means grouped by owner in rank order;
* send rows to peer p: the sorted owned rows that some entry of p's rows
  reads, which is exactly p's halo segment from this rank.

This module computes that plan on the CPU (for planning without a GPU, and
to check the device plan) and moves halo rows with ``torch.distributed``
(``exchange``), the same sends and receives the NCCL path makes.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List

import numpy as np


@dataclass
class RowPlan:
    world: int
    rank: int
    bounds: List[int]
    lo: int
    hi: int
    entry_lo: int
    halo_ids: np.ndarray     # [n_halo] global ids
    row_ptr: np.ndarray      # [n_own + 1] local CSR
    col: np.ndarray          # [local entries] relabelled columns
    send_rows: np.ndarray    # [n_send] owned rows (local ids), peer by peer
    send_counts: List[int]
    recv_counts: List[int]

    @property
    def n_own(self) -> int:
        return self.hi - self.lo

    @property
    def n_halo(self) -> int:
        return int(self.halo_ids.size)


def dst_csr(edge_index, num_edges: int, num_nodes: int):
    """Destination-keyed CSR of an edge list [src(E) | dst(E)], each row's
    edges in COO order (a stable counting sort): (row_ptr, src_of)."""
    ei = np.asarray(edge_index, dtype=np.int64).reshape(-1)
    src, dst = ei[:num_edges], ei[num_edges:2 * num_edges]
    order = np.argsort(dst, kind="stable")
    row_ptr = np.zeros(num_nodes + 1, np.int64)
    np.cumsum(np.bincount(dst, minlength=num_nodes), out=row_ptr[1:])
    return row_ptr, src[order]


def row_bounds(row_ptr, world: int) -> List[int]:
    rp = np.asarray(row_ptr, dtype=np.int64)
    n = rp.size - 1
    if n == 0:
        return [0] * (world + 1)
    total = int(rp[n]) + n
    weight = rp[1:] + np.arange(1, n + 1)  # row_ptr[j] + j for j = 1..n
    bounds = [0]
    for r in range(1, world):
        target = total * r // world
        bounds.append(int(np.searchsorted(weight, target, side="left")) + 1)
    bounds.append(n)
    for r in range(1, world + 1):
        bounds[r] = max(bounds[r], bounds[r - 1])
    return bounds


def plan_rows(row_ptr, col, world: int, rank: int) -> RowPlan:
    """Rank `rank`'s plan for the square CSR (row_ptr, col)."""
    rp = np.asarray(row_ptr, dtype=np.int64)
    col = np.asarray(col, dtype=np.int64)
    n = rp.size - 1
    bounds = row_bounds(rp, world)
    lo, hi = bounds[rank], bounds[rank + 1]
    n_own = hi - lo
    e0, e1 = int(rp[lo]), int(rp[hi])
    lcol_g = col[e0:e1]
    if lcol_g.size and (lcol_g.max() >= n or lcol_g.min() < 0):
        raise ValueError("column index out of range")
    own = (lcol_g >= lo) & (lcol_g < hi)
    halo_ids = np.unique(lcol_g[~own])
    lcol = np.where(own, lcol_g - lo, 0)
    lcol[~own] = n_own + np.searchsorted(halo_ids, lcol_g[~own])
    owner_of = np.searchsorted(np.asarray(bounds[1:]), halo_ids, side="right")
    recv_counts = np.bincount(owner_of, minlength=world)[:world].astype(np.int64).tolist()
    # send rows: for each peer, the owned columns its rows read
    send, send_counts = [], []
    for p in range(world):
        if p == rank:
            send_counts.append(0)
            continue
        a, b = int(rp[bounds[p]]), int(rp[bounds[p + 1]])
        c = col[a:b]
        mine = np.unique(c[(c >= lo) & (c < hi)]) - lo
        send.append(mine)
        send_counts.append(int(mine.size))
    send_rows = np.concatenate(send) if send else np.zeros(0, np.int64)
    return RowPlan(world, rank, bounds, lo, hi, e0, halo_ids, rp[lo:hi + 1] - rp[lo], lcol,
                   send_rows.astype(np.int64), send_counts, recv_counts)


def exchange(plan: RowPlan, x_ext, group=None):
    """Fill the halo rows of x_ext ([n_own + n_halo, F] torch tensor, owned
    rows present) over torch.distributed: pack the rows each peer reads, one
    all-to-all with the plan's counts."""
    import torch
    import torch.distributed as dist

    send = x_ext.index_select(0, torch.as_tensor(plan.send_rows, dtype=torch.long,
                                                 device=x_ext.device))
    recv = x_ext[plan.n_own:]
    dist.all_to_all_single(recv, send.contiguous(), plan.recv_counts, plan.send_counts,
                           group=group)
    return x_ext


def block_row(n: int, blocks: int, c: int) -> int:
    """First owned row of row block c of `blocks` over n rows."""
    return (c * n) // blocks


def row_blocks(plan: RowPlan, blocks: int):
    """(send_first, recv_first), [world, blocks + 1] int64 each: where row
    block c of this rank's rows starts in peer q's send list, and where owner
    q's block c starts in the halo slots (entry / slot indices as in the
    plan's lists).  The host restatement of bgnn_part_row_blocks."""
    w = plan.world
    send_off = np.concatenate([[0], np.cumsum(plan.send_counts)]).astype(np.int64)
    recv_off = np.concatenate([[0], np.cumsum(plan.recv_counts)]).astype(np.int64)
    cs = np.arange(blocks + 1, dtype=np.int64)
    send_first = np.zeros((w, blocks + 1), np.int64)
    recv_first = np.zeros((w, blocks + 1), np.int64)
    for q in range(w):
        seg = plan.send_rows[send_off[q]:send_off[q + 1]]
        send_first[q] = send_off[q] + np.searchsorted(seg, (cs * plan.n_own) // blocks)
        nq = plan.bounds[q + 1] - plan.bounds[q]
        hseg = plan.halo_ids[recv_off[q]:recv_off[q + 1]]
        recv_first[q] = recv_off[q] + np.searchsorted(hseg, plan.bounds[q] + (cs * nq) // blocks)
    return send_first, recv_first


def exchange_blocks(plan: RowPlan, x_ext, blocks: int, group=None):
    """exchange() one row block at a time, the order of the early sends: for
    each block c, every rank sends the rows of its block c that each peer
    reads and receives each owner's block c into their halo slots."""
    import torch
    import torch.distributed as dist

    sf, rf = row_blocks(plan, blocks)
    n = plan.n_own
    rows = torch.as_tensor(plan.send_rows, dtype=torch.long, device=x_ext.device)
    for c in range(blocks):
        ops = []
        for q in range(plan.world):
            if q == plan.rank:
                continue
            if sf[q, c + 1] > sf[q, c]:
                ops.append(dist.P2POp(dist.isend, x_ext.index_select(
                    0, rows[sf[q, c]:sf[q, c + 1]]).contiguous(), q, group=group))
            if rf[q, c + 1] > rf[q, c]:
                ops.append(dist.P2POp(dist.irecv, x_ext[n + rf[q, c]:n + rf[q, c + 1]], q,
                                      group=group))
        if ops:
            for r in dist.batch_isend_irecv(ops):
                r.wait()
    return x_ext

