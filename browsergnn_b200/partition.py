"""Node (destination-row) partitioning with a halo exchange plan.

The reference has no multi-device code; this is the B200 build's way to run
the SAGE and SpMM workloads on several GPUs of one box.  Rank r owns a
contiguous range of destination rows [lo, hi) chosen so every rank gets about
E / world edges.  It keeps its rows' incoming edges in COO order -- so every
row is reduced on one GPU in the reference's edge order and the results do
not depend on the number of GPUs -- and relabels their sources to
``[0, n_own)`` for owned rows and ``n_own + k`` for the k-th halo row (the
sorted unique remote sources).  Once per graph the ranks trade halo requests
with two all-to-alls; per layer, ``exchange`` packs the rows other ranks asked
for and moves them with one NCCL all-to-all into a local buffer
``[owned rows | halo rows]``, which the local aggregation reads.  Remote rows
always land in local memory first.
"""
from __future__ import annotations

from typing import Callable, List, Optional


def _torch():
    import torch

    return torch


def edge_balanced_bounds(indeg, world: int) -> List[int]:
    """Row boundaries [0, b1, ..., n] splitting the edges about evenly."""
    torch = _torch()
    n = int(indeg.numel())
    cum = torch.cumsum(indeg.to(torch.int64), 0)
    e = int(cum[-1].item()) if n else 0
    bounds = [0]
    if world > 1 and n:
        targets = torch.tensor([e * r / world for r in range(1, world)], dtype=torch.float64,
                               device=cum.device)
        cuts = torch.searchsorted(cum.to(torch.float64), targets).tolist()
        bounds += [min(n, int(c) + 1) for c in cuts]
    bounds.append(n)
    for i in range(1, len(bounds)):
        bounds[i] = max(bounds[i], bounds[i - 1])
    return bounds


class HaloPlan:
    """One rank's share of a row-partitioned graph and its halo exchange."""

    def __init__(self, src, dst, num_nodes: int, rank: int, world: int, group=None):
        import torch.distributed as dist

        torch = _torch()
        src = src.to(torch.int64)
        dst = dst.to(torch.int64)
        src = torch.where(src < 0, src + (1 << 32), src)  # uint32 ids carried in int32
        dst = torch.where(dst < 0, dst + (1 << 32), dst)
        n = int(num_nodes)
        self.rank, self.world, self.group = rank, world, group
        indeg = torch.bincount(dst, minlength=n)
        self.bounds = edge_balanced_bounds(indeg, world)
        lo, hi = self.bounds[rank], self.bounds[rank + 1]
        self.lo, self.hi, self.n_own = lo, hi, hi - lo
        keep = (dst >= lo) & (dst < hi)  # boolean selection keeps COO order
        ls, ld = src[keep], dst[keep] - lo
        own = (ls >= lo) & (ls < hi)
        halo = torch.unique(ls[~own])  # sorted global ids
        self.halo = halo
        self.n_halo = int(halo.numel())
        col = torch.empty_like(ls)
        col[own] = ls[own] - lo
        col[~own] = self.n_own + torch.searchsorted(halo, ls[~own])
        self.num_edges = int(ls.numel())
        self.edge_index = _as_u32_bits(torch.cat([col, ld]))
        # halo requests grouped by owner: ranges increase with rank and the
        # halo ids are sorted, so the concatenation is already in owner order
        ends = torch.tensor(self.bounds[1:], dtype=torch.int64, device=halo.device)
        owner = torch.searchsorted(ends, halo, right=True)
        want = torch.bincount(owner, minlength=world).to(torch.int64)
        asked = torch.empty_like(want)
        dist.all_to_all_single(asked, want, group=group)
        self.recv_splits = [int(v) for v in want.tolist()]   # rows I receive from each rank
        self.send_splits = [int(v) for v in asked.tolist()]  # rows I send to each rank
        req = torch.empty(sum(self.send_splits), dtype=torch.int64, device=halo.device)
        dist.all_to_all_single(req, halo.to(torch.int64), self.send_splits, self.recv_splits,
                               group=group)
        self.send_rows = _as_u32_bits(req - lo)  # local row ids to pack
        self.n_send = int(self.send_rows.numel())

    def exchange(self, h, pack: Callable):
        """Return [h ; halo rows] with halo rows fetched from their owners.
        ``pack(h, rows, out)`` must write out[i] = h[rows[i]]."""
        import torch.distributed as dist

        torch = _torch()
        f = int(h.shape[1])
        ext = torch.empty((self.n_own + self.n_halo, f), dtype=h.dtype, device=h.device)
        ext[: self.n_own].copy_(h)
        send = torch.empty((self.n_send, f), dtype=h.dtype, device=h.device)
        if self.n_send:
            pack(h, self.send_rows, send)
        dist.all_to_all_single(ext[self.n_own:], send, self.recv_splits, self.send_splits,
                               group=self.group)
        return ext

    def pack_send(self, ext, pack: Callable, send=None):
        """Gather the rows other ranks asked for from the owned part of ext
        into a send buffer (allocated unless given)."""
        torch = _torch()
        f = int(ext.shape[1])
        if send is None:
            send = torch.empty((self.n_send, f), dtype=ext.dtype, device=ext.device)
        if self.n_send:
            pack(ext[: self.n_own], self.send_rows, send)
        return send

    def send_recv(self, ext, send):
        """All-to-all of packed rows into the halo rows ext[n_own:]."""
        import torch.distributed as dist

        dist.all_to_all_single(ext[self.n_own:], send, self.recv_splits, self.send_splits,
                               group=self.group)
        return ext

    def exchange_into(self, ext, pack: Callable):
        """Fill the halo rows ext[n_own:] of a buffer whose owned rows
        ext[:n_own] already hold this rank's features (no copy of the owned
        part)."""
        return self.send_recv(ext, self.pack_send(ext, pack))

    def device_graph(self, device: Optional[int] = None):
        from .graph import DeviceGraph

        return DeviceGraph(self.edge_index, self.num_edges, self.n_own + self.n_halo, self.n_own,
                           device=device)


def _as_u32_bits(t):
    torch = _torch()
    t = t.to(torch.int64)
    return torch.where(t >= (1 << 31), t - (1 << 32), t).to(torch.int32).contiguous()


def cuda_pack(ctx):
    """pack() for HaloPlan.exchange on the GPU (bgnn_pack_rows)."""
    from .backend import ptr

    def pack(h, rows, out):
        ctx.call("bgnn_pack_rows", ptr(h), int(h.shape[0]), ptr(rows), int(rows.numel()),
                 int(h.shape[1]), ptr(out))

    return pack
