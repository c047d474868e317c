"""Spatial (slab) decomposition of one large periodic cell over several GPUs.

One process per GPU. Atoms are renumbered slab by slab along one lattice direction, so rank r
owns a contiguous range of atoms and -- because edges are stored receiver-major -- a contiguous
range of edges: those whose receiver it owns. Every rank builds the same global graph (cheap on
the GPU) and keeps its receivers' edges; the senders of those edges that it does not own are
its halo atoms, stored after its owned atoms in (owner rank, atom id) order.

The engine pauses at its exchange points (``UMAEngine.steps``):
  ("x", i)       halo rows of the layer input x[i] are fetched from their owners;
  ("gx", i)      halo rows of the adjoint of x[i] are sent to their owners and added there
                 (peer by peer, in rank order, so sums are deterministic), then zeroed;
  ("forces", _)  likewise for the halo atoms' partial forces.
Energy and virial are partial sums over owned receivers / local edges and are all-reduced.
Each global edge lives on exactly one rank, so nothing is counted twice.

Exchanges are point-to-point sends and receives (NCCL between GPUs, gloo in the CPU tests);
``LockstepGroup`` runs several partitions inside one process (one GPU) for testing.
"""
from __future__ import annotations

import numpy as np
import torch


def slab_order(pos, cell, nparts, axis=0):
    """(perm, ranges): atoms sorted by slab index floor(frac[axis] * nparts) (stable in atom
    id), perm[new] = old id; ranges[r] = (first, last + 1) of rank r's atoms."""
    pos = np.asarray(pos, np.float64)
    frac = pos @ np.linalg.inv(np.asarray(cell, np.float64))
    f = frac[:, axis] - np.floor(frac[:, axis])
    slab = np.minimum((f * nparts).astype(np.int64), nparts - 1)
    perm = np.argsort(slab, kind="stable")
    counts = np.bincount(slab, minlength=nparts)
    bounds = np.concatenate([[0], np.cumsum(counts)])
    return perm, [(int(bounds[r]), int(bounds[r + 1])) for r in range(nparts)]


class Plan:
    """Local graph and exchange plan of one rank, from the global receiver-major graph."""

    def __init__(self, src, tgt, img, recv_ptr, ranges, rank):
        """src, tgt, img: global edge arrays (receiver-major, int64 tensors on any device);
        recv_ptr: global receiver CSR [N+1]; ranges: per-rank owned atom ranges."""
        dev = src.device
        N = ranges[-1][1]
        self.rank, self.ranges = rank, ranges
        self.nparts = len(ranges)
        a, b = ranges[rank]
        self.n_own = b - a
        e0, e1 = int(recv_ptr[a]), int(recv_ptr[b])
        s, t = src[e0:e1], tgt[e0:e1]
        self.img = img[e0:e1]
        self.edge_range = (e0, e1)
        owner_of = self._owner_fn(dev)
        halo = torch.unique(s[(s < a) | (s >= b)])               # sorted by atom id
        if halo.numel():
            own = owner_of(halo)
            halo = halo[torch.argsort(own * N + halo)]
        self.halo = halo                                          # (owner, id) order
        self.halo_owner = owner_of(halo) if halo.numel() else halo
        self.n_halo = int(halo.numel())
        # local numbering: owned atoms first, then the halo
        self.global_ids = torch.cat([torch.arange(a, b, device=dev), halo])
        lut = torch.full((N,), -1, dtype=torch.long, device=dev)
        lut[self.global_ids] = torch.arange(self.global_ids.numel(), device=dev)
        self.src = lut[s]
        self.tgt = lut[t]
        rp = recv_ptr[a:b + 1] - e0
        self.recv_ptr = torch.cat([rp, rp[-1:].expand(self.n_halo)])
        # what every peer needs from me (its halo atoms that I own), in its halo order
        self.send_idx = {}
        self.recv_count = {}
        for q in range(self.nparts):
            if q == rank:
                continue
            qa, qb = ranges[q]
            qs = src[int(recv_ptr[qa]):int(recv_ptr[qb])]
            qh = torch.unique(qs[(qs < qa) | (qs >= qb)])
            mine = qh[(qh >= a) & (qh < b)]                       # sorted by id
            if mine.numel():
                self.send_idx[q] = (mine - a)                      # local rows
            cnt = int((self.halo_owner == q).sum()) if self.n_halo else 0
            if cnt:
                self.recv_count[q] = cnt
        # halo block of each owner (contiguous, in rank order)
        self.halo_block = {}
        off = self.n_own
        for q in range(self.nparts):
            c = self.recv_count.get(q, 0)
            if c:
                self.halo_block[q] = (off, off + c)
                off += c

    def _owner_fn(self, dev):
        starts = torch.tensor([r[0] for r in self.ranges] + [self.ranges[-1][1]], device=dev)

        def owner(ids):
            return torch.searchsorted(starts, ids, right=True) - 1
        return owner


class DistExchange:
    """Halo exchange between ranks of a torch.distributed process group (point-to-point)."""

    def __init__(self, plan, group=None, timed=False):
        self.p, self.group = plan, group
        # timed: CUDA events on the current stream bracket each exchange (its span includes
        # waiting for the slowest peer); read with timing_ms() after a synchronize
        self.timed = timed
        self.reset_timing()

    def reset_timing(self):
        self._events = {"forward": [], "reverse": []}

    def timing_ms(self):
        return {k: sum(a.elapsed_time(b) for a, b in v) for k, v in self._events.items()}

    def count_per_step(self, steps):
        return {k: len(v) // max(steps, 1) for k, v in self._events.items()}

    def _span(self, kind):
        if not self.timed:
            return None
        pair = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        pair[0].record()
        self._events[kind].append(pair)
        return pair[1]

    def _p2p(self, sends, recvs):
        import torch.distributed as dist
        ops = [dist.P2POp(dist.isend, t, q, group=self.group) for q, t in sends]
        ops += [dist.P2POp(dist.irecv, t, q, group=self.group) for q, t in recvs]
        if ops:
            for r in dist.batch_isend_irecv(ops):
                r.wait()

    def forward(self, x):
        """Fill halo rows of x [N_local, ...] with their owners' rows."""
        p = self.p
        end = self._span("forward")
        sends = [(q, x[idx].contiguous()) for q, idx in p.send_idx.items()]
        recvs = [(q, torch.empty((c,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device))
                 for q, c in p.recv_count.items()]
        self._p2p(sends, recvs)
        for q, buf in recvs:
            lo, hi = p.halo_block[q]
            x[lo:hi] = buf
        if end is not None:
            end.record()

    def reverse(self, g):
        """Send halo rows of the adjoint g to their owners, add the received rows into owned
        rows (peers in rank order), zero the halo rows."""
        p = self.p
        end = self._span("reverse")
        sends = [(q, g[p.halo_block[q][0]:p.halo_block[q][1]].contiguous())
                 for q in p.recv_count]
        recvs = [(q, torch.empty((idx.numel(),) + tuple(g.shape[1:]), dtype=g.dtype,
                                 device=g.device)) for q, idx in p.send_idx.items()]
        self._p2p(sends, recvs)
        for q, buf in sorted(recvs, key=lambda t: t[0]):
            g.index_add_(0, p.send_idx[q], buf)
        g[p.n_own:] = 0
        if end is not None:
            end.record()


class LockstepGroup:
    """Several partitions driven in lock step inside one process (exchanges are copies);
    the single-GPU stand-in for ``DistExchange`` used by the tests."""

    def __init__(self, plans):
        self.plans = plans

    def forward(self, xs):
        for r, p in enumerate(self.plans):
            for q, (lo, hi) in p.halo_block.items():
                src_rows = self.plans[q].send_idx[r]
                xs[r][lo:hi] = xs[q][src_rows]

    def reverse(self, gs):
        bufs = {}
        for r, p in enumerate(self.plans):
            for q, (lo, hi) in p.halo_block.items():
                bufs[(q, r)] = gs[r][lo:hi].clone()
        for q, p in enumerate(self.plans):
            for r in sorted(p.send_idx):
                if (q, r) in bufs:
                    gs[q].index_add_(0, p.send_idx[r], bufs[(q, r)])
        for r, p in enumerate(self.plans):
            gs[r][p.n_own:] = 0


def local_graph(g, plan):
    """The engine's Graph for one rank: owned atoms then halo atoms, the rank's edges, energy
    summed over owned atoms only. ``g`` is the global Graph (on this rank's GPU)."""
    import ctypes

    from . import _lib as L
    from ._lib import call, ptr
    from .graph import Graph
    dev = g.src.device
    i32 = lambda t: t.to(device=dev, dtype=torch.int32).contiguous()  # noqa: E731
    N, E = plan.global_ids.numel(), plan.src.numel()
    src, tgt, img = i32(plan.src), i32(plan.tgt), i32(plan.img)
    Z = g.Z[plan.global_ids.to(dev)].contiguous()
    s = L.stream_ptr()
    send_ptr = torch.empty(N + 1, dtype=torch.int32, device=dev)
    send_eid = torch.empty(max(E, 1), dtype=torch.int32, device=dev)
    scratch = torch.empty(max(N, 1), dtype=torch.int32, device=dev)
    call("atom_sender_csr", ptr(src), E, N, ptr(scratch), ptr(send_ptr), ptr(send_eid), s)
    zs = torch.empty(max(E, 1), dtype=torch.int32, device=dev)
    zt = torch.empty(max(E, 1), dtype=torch.int32, device=dev)
    call("atom_edge_species", ptr(Z), ptr(src), ptr(tgt), E, ptr(zs), ptr(zt), s)
    return Graph(N=N, E=E, nsys=1, periodic=g.periodic, Z=Z,
                 sys_id=torch.zeros(N, dtype=torch.int32, device=dev),
                 sys_ptr=torch.tensor([0, plan.n_own], dtype=torch.int32, device=dev),
                 sys_ptr_host=[0, plan.n_own], src=src, tgt=tgt, img=img, shifts=g.shifts,
                 recv_ptr=i32(plan.recv_ptr), send_ptr=send_ptr, send_eid=send_eid[:E],
                 zs=zs[:E], zt=zt[:E])


def plans_for(g, ranges):
    """Plans of every rank from a global Graph (all ranks compute all plans identically)."""
    src, tgt, img = g.src.long(), g.tgt.long(), g.img.long()
    rp = g.recv_ptr.long().cpu()
    return [Plan(src, tgt, img, rp, ranges, r) for r in range(len(ranges))]


def run_partition(eng, ws, exch, forces=True, virial=True, stream=None):
    """One partitioned step on this rank: the engine's exchange points are served by
    ``exch`` (``DistExchange``); energy and virial are left as this rank's partial sums."""
    for kind, i in eng.steps(ws, ws.pos, forces, virial, stream):
        if kind == "x":
            exch.forward(ws.x[i])
        elif kind == "gx":
            exch.reverse(ws.gx)
        elif kind == "forces":
            exch.reverse(ws.forces)


def run_lockstep(eng, wss, group, forces=True, virial=True):
    """All partitions of one cell in one process, advanced together between exchange points."""
    gens = [eng.steps(ws, ws.pos, forces, virial) for ws in wss]
    while True:
        evs = [next(gn, None) for gn in gens]
        if all(e is None for e in evs):
            return
        kind, i = evs[0]
        assert all(e == evs[0] for e in evs)
        if kind == "x":
            group.forward([ws.x[i] for ws in wss])
        elif kind == "gx":
            group.reverse([ws.gx for ws in wss])
        elif kind == "forces":
            group.reverse([ws.forces for ws in wss])
