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

    def remote_map(self):
        """Where each owned row goes in the other ranks' [owned | halo]
        buffers, for producers that store rows straight into their peers'
        memory instead of an all-to-all.  Rank p's halo holds its rows from
        rank r at n_own(p) + (rows p receives from ranks < r) + k for the k-th
        row r sends it.  Returns (row_ptr [n_own+1] int64, dst [n_send] int64
        packing peer << 32 | destination row, in row order, each row's
        destinations by peer), and peer_rows[p] = rows of p's buffer."""
        import torch.distributed as dist

        torch = _torch()
        dev = self.halo.device
        info = torch.tensor([self.n_own, self.n_halo] + self.recv_splits, dtype=torch.int64,
                            device=dev)
        allinfo = [torch.empty_like(info) for _ in range(self.world)]
        dist.all_gather(allinfo, info, group=self.group)
        allinfo = [t.cpu().tolist() for t in allinfo]
        rows_l, dst_l = [], []
        send_rows = self.send_rows.to(torch.int64).cpu()
        send_rows = torch.where(send_rows < 0, send_rows + (1 << 32), send_rows)
        pos = 0
        for p in range(self.world):
            cnt = self.send_splits[p]
            if cnt == 0:
                continue
            n_own_p = allinfo[p][0]
            off = sum(allinfo[p][2:2 + self.rank])  # rows p receives from ranks before me
            rows_l.append(send_rows[pos:pos + cnt])
            dst_l.append((p << 32) + n_own_p + off + torch.arange(cnt, dtype=torch.int64))
            pos += cnt
        peer_rows = [allinfo[p][0] + allinfo[p][1] for p in range(self.world)]
        if not rows_l:
            return torch.zeros(self.n_own + 1, dtype=torch.int64), \
                torch.zeros(0, dtype=torch.int64), peer_rows
        rows = torch.cat(rows_l)
        dst = torch.cat(dst_l)
        order = torch.argsort(rows, stable=True)
        counts = torch.bincount(rows, minlength=self.n_own)
        row_ptr = torch.zeros(self.n_own + 1, dtype=torch.int64)
        row_ptr[1:] = torch.cumsum(counts, 0)
        return row_ptr, dst[order], peer_rows

    def device_graph(self, device: Optional[int] = None):
        from .graph import DeviceGraph

        return DeviceGraph(self.edge_index, self.num_edges, self.n_own + self.n_halo, self.n_own,
                           device=device)


class SharedBuffer:
    """A [rows, cols] f32 device buffer in its own allocation
    (bgnn_shared_alloc), viewed as a torch tensor; other ranks of the node can
    map it by its IPC handle."""

    def __init__(self, ctx, rows: int, cols: int):
        import ctypes

        torch = _torch()
        self.ctx = ctx
        p = ctypes.c_void_p()
        ctx.call("bgnn_shared_alloc", int(rows) * int(cols) * 4, ctypes.byref(p))
        self.ptr = p.value
        self.__cuda_array_interface__ = {"shape": (int(rows), int(cols)), "typestr": "<f4",
                                         "data": (self.ptr, False), "version": 2}
        self.tensor = torch.as_tensor(self, device=f"cuda:{ctx.device}")

    def handle(self) -> bytes:
        import ctypes

        buf = (ctypes.c_uint8 * 64)()
        self.ctx.call("bgnn_ipc_handle", self.ptr, buf)
        return bytes(buf)

    def free(self):
        if self.ptr:
            self.tensor = None
            self.ctx.call("bgnn_shared_free", self.ptr)
            self.ptr = None


class PeerStores:
    """Everything a rank needs to store its layer outputs straight into the
    other ranks' halo rows (bgnn_linear_add_remote): the remote map of a
    HaloPlan on the device, and for each shared buffer the table of the
    peers' mapped addresses (its own entry is NULL)."""

    def __init__(self, plan: "HaloPlan", ctx, buffers: List[SharedBuffer]):
        import ctypes

        import torch.distributed as dist

        torch = _torch()
        self.plan, self.ctx = plan, ctx
        dev = f"cuda:{ctx.device}"
        row_ptr, dst, peer_rows = plan.remote_map()
        if dst.numel():
            peers = dst >> 32
            rows = dst & 0xFFFFFFFF
            lim = torch.tensor(peer_rows, dtype=torch.int64)[peers]
            if bool((peers == plan.rank).any()) or bool((peers >= plan.world).any()) or \
                    bool((rows < 0).any()) or bool((rows >= lim).any()):
                raise ValueError("remote map out of range")
        self.row_ptr = _as_u32_bits(row_ptr).to(dev)
        self.dst = dst.to(dev)
        self.peer_rows = _as_u32_bits(torch.tensor(peer_rows, dtype=torch.int64)).to(dev)
        handles = [b.handle() for b in buffers]
        everyone = [None] * plan.world
        dist.all_gather_object(everyone, handles, group=plan.group)
        self.opened = []
        self.tables = []
        for j in range(len(buffers)):
            ptrs = []
            for p in range(plan.world):
                if p == plan.rank:
                    ptrs.append(0)
                    continue
                h = (ctypes.c_uint8 * 64).from_buffer_copy(everyone[p][j])
                q = ctypes.c_void_p()
                ctx.call("bgnn_ipc_open", h, ctypes.byref(q))
                self.opened.append(q.value)
                ptrs.append(q.value)
            self.tables.append(torch.tensor(ptrs, dtype=torch.int64, device=dev))

    def close(self):
        """Unmap the peers' buffers (before any rank frees its own)."""
        for q in self.opened:
            self.ctx.call("bgnn_ipc_close", q)
        self.opened = []


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
