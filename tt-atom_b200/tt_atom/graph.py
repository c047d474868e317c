"""Graph construction on the GPU: neighbour list, receiver/sender CSR, per-edge species.

``radius_graph`` keeps the reference's signature and result (tt_atom/geometry.py:48-81): the
same fp32 cutoff predicate and edge order, computed by ``atom_neighbor_list``. ``build_graph``
returns the receiver-major ``Graph`` the engine consumes (one or many systems back to back).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

from . import _lib as L
from ._lib import call, ptr


def image_reps(cell, pbc, cutoff):
    """Image offsets r per axis, r = ceil(cutoff * |b_k|) with b_k the reciprocal rows (0 on
    a non-periodic axis): the host arithmetic of tt_atom/geometry.py:66-75 in torch fp32."""
    cell = torch.as_tensor(cell, dtype=torch.float32).cpu()
    pbc = torch.as_tensor(pbc, dtype=torch.bool).reshape(-1).expand(3)
    recip = torch.linalg.inv(cell).transpose(0, 1)
    return [int(math.ceil(float(cutoff * torch.linalg.norm(recip[k])))) if bool(pbc[k]) else 0
            for k in range(3)]


def image_shifts(cell, pbc, cutoff):
    """Cartesian image shifts ``cells @ cell`` for integer offsets in [-r, r] per periodic axis
    (``image_reps``), in cartesian-product order -- tt_atom/geometry.py:66-75, kept in torch
    fp32 on the CPU so the shifts are the reference's bit for bit."""
    cell = torch.as_tensor(cell, dtype=torch.float32).cpu()
    ranges = [torch.arange(-r, r + 1, dtype=torch.float32) for r in image_reps(cell, pbc, cutoff)]
    cells = torch.cartesian_prod(*ranges).reshape(-1, 3)
    return cells @ cell


MAX_CELL_CAND = 256       # the cell-list kernel sorts at most this many candidates per receiver


def cell_grid_params(cell, pbc, cutoff, N):
    """Bins of the cell list for a fully periodic cell (see atom_cell_grid): nb bins per
    lattice direction, each at least the cutoff (plus slack) wide across its lattice planes,
    and the reach in bins that covers the cutoff; None when the cell is not fully periodic."""
    if cell is None or pbc is None or not bool(np.all(np.asarray(pbc))):
        return None
    c = np.asarray(cell, dtype=np.float32).astype(np.float64)
    inv = np.linalg.inv(c)
    rc = float(cutoff) * (1.0 + 1e-5) + 1e-4
    bn = np.linalg.norm(inv, axis=0)            # |b_k|: columns of inv(cell)
    nb = [max(1, min(512, int(math.floor(1.0 / (rc * b))))) for b in bn]
    while nb[0] * nb[1] * nb[2] > max(64, 4 * N):  # no more bins than atoms need
        k = int(np.argmax(nb))
        nb[k] = max(1, nb[k] // 2)
    reach = [max(1, int(math.ceil(rc * b * n))) for b, n in zip(bn, nb)]
    return dict(inv=inv, nb=nb, reach=reach, img_r=image_reps(cell, pbc, cutoff))


class CellScratch:
    """Device scratch of the cell list for N atoms, and the ``CellGrid`` argument over it."""

    def __init__(self, params, N, dev):
        i32 = lambda n: torch.empty(max(n, 1), dtype=torch.int32, device=dev)  # noqa: E731
        nbins = params["nb"][0] * params["nb"][1] * params["nb"][2]
        self.t = [i32(N), i32(3 * N), i32(nbins), i32(nbins + 1), i32(N)]
        g = L.CellGrid()
        for k in range(9):
            g.inv_cell[k] = float(params["inv"].reshape(-1)[k])
        for k in range(3):
            g.nb[k], g.reach[k], g.img_r[k] = (params["nb"][k], params["reach"][k],
                                               params["img_r"][k])
        g.atom_bin, g.atom_off, g.bin_cnt, g.bin_ptr, g.bin_atoms = [t.data_ptr() for t in self.t]
        self.grid = g

    def arg(self):
        return ctypes.byref(self.grid)


_SHIFT_CACHE = {}
_SYS_CACHE = {}


def _device_shifts(cell, pbc, cutoff, dev):
    """``image_shifts`` on the device, cached per (cell, pbc, cutoff, device): MD and relaxation
    call the neighbour list every step with the same cell."""
    key = (np.asarray(cell, np.float32).tobytes(), tuple(np.broadcast_to(np.asarray(pbc, bool), 3)),
           float(cutoff), str(dev))
    t = _SHIFT_CACHE.get(key)
    if t is None:
        if len(_SHIFT_CACHE) > 64:
            _SHIFT_CACHE.clear()
        t = _SHIFT_CACHE[key] = image_shifts(cell, pbc, cutoff).to(dev).contiguous()
    return t


def _device_sys(sys_ptr, dev):
    """(sys_id [N], sys_ptr [nsys + 1]) int32 device tensors for atom offsets ``sys_ptr``, cached."""
    key = (tuple(sys_ptr), str(dev))
    v = _SYS_CACHE.get(key)
    if v is None:
        if len(_SYS_CACHE) > 64:
            _SYS_CACHE.clear()
        N = sys_ptr[-1]
        sys_id = torch.empty(N, dtype=torch.int32)
        for k in range(len(sys_ptr) - 1):
            sys_id[sys_ptr[k]:sys_ptr[k + 1]] = k
        v = _SYS_CACHE[key] = (sys_id.to(dev),
                               torch.tensor(sys_ptr, dtype=torch.int32, device=dev))
    return v


def csd_embedding(w, charge, spin, C, dataset="omat"):
    """System (charge / spin / dataset) embedding [nsys, C], tt_atom/geometry.py:23-45. Host
    glue: a few hundred flops per system, computed once per system."""
    charge = torch.as_tensor(charge, dtype=torch.float32).reshape(-1)
    spin = torch.as_tensor(spin, dtype=torch.float32).reshape(-1)
    if "charge_embedding.rand_emb.weight" in w:
        chg = F.embedding(charge.long() + 100, w["charge_embedding.rand_emb.weight"])
        sp = F.embedding(spin.long(), w["spin_embedding.rand_emb.weight"])
    else:
        def enc(v, W, zero_at_0):
            a = v[:, None] * W[None, :] * 2 * math.pi
            e = torch.cat([torch.sin(a), torch.cos(a)], -1)
            if zero_at_0:
                e = e.clone()
                e[v == 0] = 0
            return e
        chg = enc(charge, w["charge_embedding.W"], False)
        sp = enc(spin, w["spin_embedding.W"], True)
    ds = w[f"dataset_embedding.dataset_emb_dict.{dataset}.weight"][0].expand(charge.shape[0], -1)
    return F.silu(F.linear(torch.cat([chg, sp, ds], 1), w["mix_csd.weight"], w["mix_csd.bias"]))


@dataclass
class Graph:
    N: int
    E: int
    nsys: int
    periodic: bool
    Z: torch.Tensor          # [N] int32
    sys_id: torch.Tensor     # [N] int32
    sys_ptr: torch.Tensor    # [nsys + 1] int32 (device)
    sys_ptr_host: list
    src: torch.Tensor        # [E] int32, receiver-major
    tgt: torch.Tensor
    img: torch.Tensor        # [E] int32 image index into shifts
    shifts: torch.Tensor     # [S, 3] fp32
    recv_ptr: torch.Tensor   # [N + 1]
    send_ptr: torch.Tensor   # [N + 1]
    send_eid: torch.Tensor   # [E]
    zs: torch.Tensor         # [E] species of source
    zt: torch.Tensor         # [E] species of target
    max_cand: int = 64       # candidate slots per receiver the build needed
    cutoff: float = 0.0
    max_neighbors: int = 0   # 0: uncapped
    cell_grid: dict = None   # cell-list bins (fully periodic single systems), else None

    def reference_order(self):
        """(edge_index [2, E] int64, image index [E]) in the reference's edge order: periodic
        graphs are receiver-major already; aperiodic ones are ordered by (source, target)."""
        if self.periodic:
            perm = torch.arange(self.E, device=self.src.device)
        else:
            perm = self.send_eid.long()
        ei = torch.stack([self.src.long()[perm], self.tgt.long()[perm]])
        return ei, self.img.long()[perm], perm

    def same_topology(self, other):
        return (other is not None and self.N == other.N and self.E == other.E
                and torch.equal(self.src, other.src) and torch.equal(self.tgt, other.tgt)
                and torch.equal(self.img, other.img) and torch.equal(self.shifts, other.shifts))


def build_graph(pos, Z, cutoff, cell=None, pbc=None, max_neighbors=None, sys_ptr=None,
                device="cuda", max_cand=None, stream=None, use_cells=True):
    """Neighbour list of one system, or of several aperiodic systems stored back to back
    (``sys_ptr`` atom offsets; no edges between systems), on the GPU. A fully periodic single
    system takes its candidates from a cell list (``use_cells``), others from all pairs; the
    edge list is the same either way."""
    dev = torch.device(device)
    pos_host = None if torch.is_tensor(pos) else np.asarray(pos, dtype=np.float32)
    pos = torch.as_tensor(pos, dtype=torch.float32).to(dev).contiguous()
    N = pos.shape[0]
    Zt = torch.as_tensor(np.asarray(Z), dtype=torch.int32).to(dev).contiguous()
    periodic = cell is not None and pbc is not None and bool(np.asarray(pbc).any())
    if sys_ptr is None:
        sys_ptr = [0, N]
    sys_ptr = [int(v) for v in sys_ptr]
    nsys = len(sys_ptr) - 1
    if periodic and nsys != 1:
        raise ValueError("periodic batches are built one system at a time")
    shifts = (_device_shifts(cell, pbc, cutoff, dev) if periodic
              else torch.zeros(1, 3, device=dev))
    S = shifts.shape[0]
    s = L.stream_ptr(stream)
    if max_cand is None:
        max_cand = 64 if max_neighbors is None else max(64, 2 * max_neighbors)
    cap = 0 if max_neighbors is None else int(max_neighbors)
    recv_cnt = torch.empty(N, dtype=torch.int32, device=dev)
    small = torch.empty(nsys + 2, dtype=torch.int64, device=dev)
    sp_host = L.host_i64(sys_ptr)
    need = ctypes.c_int(0)
    # the bounding box from the caller's host array when there is one (no device round trip)
    pos_np = None
    if periodic:
        pos_np = pos_host if pos_host is not None else pos.detach().cpu().numpy()
    bbox = (L.host_f32(list(pos_np.min(0)) + list(pos_np.max(0)))
            if periodic and N > 0 else None)
    grid_params = cell_grid_params(cell, pbc, cutoff, N) if (periodic and nsys == 1 and
                                                             use_cells) else None
    cells = CellScratch(grid_params, N, dev) if grid_params is not None else None
    while True:
        cand_idx = torch.empty(max(N * max_cand, 1), dtype=torch.int32, device=dev)
        cand_d = torch.empty(max(N * max_cand, 1), dtype=torch.float32, device=dev)
        grid = cells.arg() if cells is not None and max_cand <= MAX_CELL_CAND else None
        rc = L.lib().atom_neighbor_list(ptr(pos), N, sp_host, nsys, ptr(shifts), S, float(cutoff),
                                        int(periodic), cap, max_cand, ptr(cand_idx), ptr(cand_d),
                                        ptr(recv_cnt), None, None, None, None, bbox,
                                        ptr(small), ctypes.byref(need), grid, s)
        if rc == L.ATOM_ERR_CAPACITY:
            max_cand = int(need.value * 1.25) + 32
            continue
        if rc != 0:
            raise L.AtomError("atom_neighbor_list", rc)
        break
    recv_ptr = torch.empty(N + 1, dtype=torch.int32, device=dev)
    total = ctypes.c_int(0)
    call("atom_exclusive_scan", ptr(recv_cnt), N, ptr(recv_ptr), ctypes.byref(total), s)
    E = int(total.value)
    src = torch.empty(max(E, 1), dtype=torch.int32, device=dev)
    tgt = torch.empty(max(E, 1), dtype=torch.int32, device=dev)
    img = torch.empty(max(E, 1), dtype=torch.int32, device=dev)
    call("atom_neighbor_list", ptr(pos), N, sp_host, nsys, ptr(shifts), S, float(cutoff),
         int(periodic), cap, max_cand, ptr(cand_idx), ptr(cand_d), ptr(recv_cnt), ptr(recv_ptr),
         ptr(src), ptr(tgt), ptr(img), bbox, ptr(small), None, None, s)
    src, tgt, img = src[:E], tgt[:E], img[:E]
    send_ptr = torch.empty(N + 1, dtype=torch.int32, device=dev)
    send_eid = torch.empty(max(E, 1), dtype=torch.int32, device=dev)
    scratch = torch.empty(max(N, 1), dtype=torch.int32, device=dev)
    call("atom_sender_csr", ptr(src), E, N, ptr(scratch), ptr(send_ptr), ptr(send_eid), s)
    send_eid = send_eid[:E]
    zs = torch.empty(max(E, 1), dtype=torch.int32, device=dev)
    zt = torch.empty(max(E, 1), dtype=torch.int32, device=dev)
    call("atom_edge_species", ptr(Zt), ptr(src), ptr(tgt), E, ptr(zs), ptr(zt), s)
    sys_id, sys_ptr_d = _device_sys(sys_ptr, dev)
    return Graph(N=N, E=E, nsys=nsys, periodic=periodic, Z=Zt, sys_id=sys_id, sys_ptr=sys_ptr_d,
                 sys_ptr_host=sys_ptr, src=src, tgt=tgt, img=img, shifts=shifts,
                 recv_ptr=recv_ptr, send_ptr=send_ptr, send_eid=send_eid, zs=zs[:E], zt=zt[:E],
                 max_cand=max_cand, cutoff=float(cutoff), max_neighbors=cap,
                 cell_grid=grid_params)


class TopologyRefresh:
    """Rebuilds one system's neighbour list on the device, in place, into a graph's own arrays
    (``atom_neighbor_refresh`` + sender CSR + edge species): no host synchronisation, so the
    launches can be captured in a CUDA graph together with the step that uses the graph.

    The edge count is fixed by the arrays: when the new list has a different number of edges,
    or a receiver overflows its candidate slots, the arrays keep the previous topology and
    ``status[0]`` says so (``ATOM_REFRESH_*``); the caller reads it after the stream has run
    and rebuilds through ``build_graph`` then. Candidate slots get headroom over what the
    first build needed, for atoms that move."""

    OK, OVERFLOW, SIZE_CHANGED = 0, 1, 2

    def __init__(self, graph, headroom=32):
        if graph.nsys != 1:
            raise ValueError("the device refresh handles one system")
        dev = graph.src.device
        N = graph.N
        self.g = graph
        self.max_cand = int(graph.max_cand) + headroom
        i32 = lambda n: torch.empty(max(n, 1), dtype=torch.int32, device=dev)  # noqa: E731
        self.cand_idx = i32(N * self.max_cand)
        self.cand_d = torch.empty(max(N * self.max_cand, 1), dtype=torch.float32, device=dev)
        self.recv_cnt, self.stage_ptr, self.csr_scratch = i32(N), i32(N + 1), i32(N)
        self.box = torch.empty(6, dtype=torch.float32, device=dev)
        self.status = torch.zeros(4, dtype=torch.int32, device=dev)
        self.cells = (CellScratch(graph.cell_grid, N, dev)
                      if graph.cell_grid is not None and self.max_cand <= MAX_CELL_CAND else None)

    def launch(self, pos, stream=None):
        g, s = self.g, L.stream_ptr(stream)
        call("atom_neighbor_refresh", ptr(pos), g.N, ptr(g.shifts), g.shifts.shape[0],
             float(g.cutoff), int(g.periodic), int(g.max_neighbors), self.max_cand,
             ptr(self.cand_idx), ptr(self.cand_d), ptr(self.recv_cnt), ptr(self.stage_ptr),
             ptr(self.box), ptr(self.status), g.E, ptr(g.recv_ptr), ptr(g.src), ptr(g.tgt),
             ptr(g.img), self.cells.arg() if self.cells is not None else None, s)
        call("atom_sender_csr", ptr(g.src), g.E, g.N, ptr(self.csr_scratch), ptr(g.send_ptr),
             ptr(g.send_eid), s)
        call("atom_edge_species", ptr(g.Z), ptr(g.src), ptr(g.tgt), g.E, ptr(g.zs), ptr(g.zt), s)


def radius_graph(pos, cutoff, cell=None, pbc=None, max_neighbors=None, device="cuda"):
    """``(edge_index [2, E], cell_shift [E, 3])`` with the reference's edge order and fp32
    predicate (tt_atom/geometry.py:48-81), computed on the GPU. Returns CPU tensors like the
    reference."""
    Z = np.zeros(len(pos), dtype=np.int64)
    g = build_graph(pos, Z, cutoff, cell, pbc, max_neighbors=max_neighbors, device=device)
    ei, im, _ = g.reference_order()
    shift = g.shifts[im] if g.E else torch.zeros(0, 3, device=g.shifts.device)
    if not g.periodic:
        shift = torch.zeros_like(shift)
    return ei.cpu(), shift.cpu()
