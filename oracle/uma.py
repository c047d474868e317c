"""CPU oracle for the eSCN-MD (UMA) energy + force + stress path -- TEST INFRASTRUCTURE ONLY.

This module is the checker the CUDA path is compared against. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it; the product path
(``tt_atom``) never does.

It restates, in fp32 torch on the CPU, the reference's own CPU path:

* neighbour list          -- tt_atom/geometry.py:48-81 (``radius_graph``)
* host geometry           -- tt_atom/geometry.py:87-280 (Euler angles with the safe acos/atan2
                             guards, the e3nn ``J`` Wigner-D construction, Gaussian basis,
                             polynomial envelope p=5, edge-degree node init)
* system embedding        -- tt_atom/geometry.py:23-45 (``csd_embedding``)
* backbone forward        -- tests/mirror.py:21-134 (radial MLP, SO(2) conv, RMS-norm-SH, gate,
                             grid feed-forward, edgewise block, energy head)
* forces / stress         -- tt_atom/forces.py:515-524 (strain leaf ``r' = r (I + sym eps)``) and
                             torch autograd, as tt_atom/forces.py:580-589 does;
                             stress = virial / volume (tt_atom/calculator.py:159-165)

plus one rule that the reference does not have: an optional per-receiver neighbour cap
(``cap_neighbors``), shared verbatim with the GPU neighbour list.

Parity of this restatement is pinned two ways: against the reference's committed fairchem
goldens (``tests/golden/ref_golden_*.npz``: energy and forces of ethanol and bulk Si), and against
outputs of the reference's own code run on this framework's seeded configs
(``tests/golden/ref_run_*.npz``, written by ``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

EPS = 1e-7


# ------------------------------------------------------------------------- neighbour list


def radius_graph(pos, cutoff, cell=None, pbc=None):
    """Brute-force neighbour list, tt_atom/geometry.py:48-81.

    Aperiodic: pairs (a, b), a != b, with ``||pos[a] - pos[b]|| < cutoff``, ordered by (a, b), as
    ``edge_index = [a, b]`` (a = source, b = target/receiver).
    Periodic: triples (i, j, c) with ``d2 = |pos[i] - (pos[j] + shift[c])|^2 <= cutoff^2`` and
    ``d2 > 1e-8``, ordered by (i, j, c), as ``edge_index = [j, i]`` and ``shift[c]``; the image
    range per axis is ``ceil(cutoff * |b_k|)`` (b = reciprocal rows)."""
    periodic = cell is not None and pbc is not None and bool(torch.as_tensor(pbc).any())
    if not periodic:
        d = torch.linalg.norm(pos[:, None, :] - pos[None, :, :], dim=-1)
        keep = (d < cutoff) & (d > 0)
        a, b = torch.nonzero(keep, as_tuple=True)
        return torch.stack([a, b]), pos.new_zeros(a.shape[0], 3)
    cell = torch.as_tensor(cell, dtype=pos.dtype)
    pbc = torch.as_tensor(pbc, dtype=torch.bool).reshape(-1).expand(3)
    shifts = image_shifts(cell, pbc, cutoff, pos.dtype)
    disp = pos[:, None, None, :] - (pos[None, :, None, :] + shifts[None, None, :, :])
    d2 = (disp ** 2).sum(-1)
    keep = (d2 <= cutoff * cutoff) & (d2 > 1e-8)
    i, j, c = torch.nonzero(keep, as_tuple=True)
    return torch.stack([j, i]), shifts[c]


def image_reps(cell, pbc, cutoff):
    """Images per axis: ``ceil(cutoff * ||b_k||)`` where b_k are reciprocal rows
    (tt_atom/geometry.py:70-73); 0 along non-periodic axes."""
    recip = torch.linalg.inv(cell).transpose(0, 1)
    return [int(math.ceil(float(cutoff * torch.linalg.norm(recip[k])))) if bool(pbc[k]) else 0
            for k in range(3)]


def image_shifts(cell, pbc, cutoff, dtype=torch.float32):
    """Cartesian image shifts ``cells @ cell`` for integer offsets in ``[-r, r]^3``, offsets in
    cartesian-product order (tt_atom/geometry.py:74-75)."""
    reps = image_reps(cell, pbc, cutoff)
    ranges = [torch.arange(-r, r + 1, dtype=dtype) for r in reps]
    cells = torch.cartesian_prod(*ranges).reshape(-1, 3)
    return cells @ cell


def edge_rank_key(pos, edge_index, shift, periodic):
    """The per-edge distance measure the cutoff test uses: ``||pos[a]-pos[b]||`` (aperiodic) or
    ``|pos[i] - (pos[j] + shift)|^2`` (periodic), recomputed with the same fp32 expressions."""
    src, tgt = edge_index[0], edge_index[1]
    if not periodic:
        return torch.linalg.norm(pos[src] - pos[tgt], dim=-1)
    disp = pos[tgt] - (pos[src] + shift)
    return (disp ** 2).sum(-1)


def cap_neighbors(pos, edge_index, shift, periodic, max_neighbors):
    """Per-receiver neighbour cap (this framework's rule; the reference's UMA graph is uncapped).

    For every receiver (``edge_index[1]``) keep the ``max_neighbors`` edges with the smallest
    distance measure (``edge_rank_key``), ties broken by the edge's position in the uncapped
    reference order. Surviving edges keep that reference order. Returns the kept-edge mask."""
    E = edge_index.shape[1]
    if max_neighbors is None or E == 0:
        return torch.ones(E, dtype=torch.bool)
    key = edge_rank_key(pos, edge_index, shift, periodic)
    tgt = edge_index[1]
    order = torch.arange(E)
    # sort by (receiver, key, reference index): stable sorts from the least significant key
    o = torch.sort(key, stable=True).indices
    o = o[torch.sort(tgt[o], stable=True).indices]
    rec = tgt[o]
    first = torch.ones(E, dtype=torch.bool)
    first[1:] = rec[1:] != rec[:-1]
    start = torch.cummax(torch.where(first, order, torch.zeros_like(order)), 0).values
    rank = order - start
    keep = torch.zeros(E, dtype=torch.bool)
    keep[o[rank < max_neighbors]] = True
    return keep


def neighbor_list(pos, cutoff, cell=None, pbc=None, max_neighbors=None):
    """``radius_graph`` followed by ``cap_neighbors``; returns (edge_index, shift)."""
    periodic = cell is not None and pbc is not None and bool(torch.as_tensor(pbc).any())
    ei, sh = radius_graph(pos, cutoff, cell, pbc)
    keep = cap_neighbors(pos, ei, sh, periodic, max_neighbors)
    return ei[:, keep], sh[keep]


# --------------------------------------------------------------------------- geometry


class _SafeAcos(torch.autograd.Function):
    """acos with the guarded derivative of tt_atom/geometry.py:87-96."""

    @staticmethod
    def forward(ctx, x):
        ctx.save_for_backward(x.clamp(-1 + EPS, 1 - EPS))
        return torch.acos(x)

    @staticmethod
    def backward(ctx, g):
        (xc,) = ctx.saved_tensors
        return -g / torch.sqrt(1 - xc * xc).clamp(min=EPS)


class _SafeAtan2(torch.autograd.Function):
    """atan2 with the clamped-denominator derivative of tt_atom/geometry.py:99-109."""

    @staticmethod
    def forward(ctx, y, x):
        ctx.save_for_backward(y, x)
        return torch.atan2(y, x)

    @staticmethod
    def backward(ctx, g):
        y, x = ctx.saved_tensors
        den = (x * x + y * y).clamp(min=EPS)
        return g * x / den, -g * y / den


def _zrot(theta, l):
    """Wigner z-rotation block for degree l: cos(f*theta) on the diagonal, sin(f*theta) on the
    anti-diagonal, frequencies f = l..-l (tt_atom/geometry.py:124-136)."""
    f = torch.arange(l, -l - 1, -1, dtype=theta.dtype)
    ft = f * theta[:, None]
    return torch.diag_embed(torch.cos(ft)) + torch.diag_embed(torch.sin(ft)).flip(-1)


def wigner_m(edge_vec, Jd, to_m, lmax=2):
    """Per-edge Wigner matrix in the m-primed row order, ``[E, 9, 9]``.

    Euler angles of the normalised edge (beta = acos(y), alpha = atan2(x, z), roll fixed to 0;
    tt_atom/geometry.py:112-118), then per degree ``D_l = Z(0) J Z(-beta) J Z(-alpha)``
    (tt_atom/geometry.py:139-155), block-diagonal, rows permuted by ``to_m``
    (tt_atom/geometry.py:209-224). The inverse used for the rotate-back is its transpose."""
    xyz = F.normalize(edge_vec).clamp(-1.0, 1.0)
    x, y, z = xyz[:, 0], xyz[:, 1], xyz[:, 2]
    beta = _SafeAcos.apply(y)
    alpha = _SafeAtan2.apply(x, z)
    E = edge_vec.shape[0]
    n = (lmax + 1) ** 2
    blocks = []
    for l in range(lmax + 1):
        J = Jd[l]
        zero = torch.zeros_like(alpha)
        blocks.append(_zrot(zero, l) @ J @ _zrot(-beta, l) @ J @ _zrot(-alpha, l))
    wig = torch.zeros(E, n, n, dtype=edge_vec.dtype)
    s = 0
    for b in blocks:
        d = b.shape[-1]
        wig[:, s:s + d, s:s + d] = b
        s += d
    perm = to_m.abs().argmax(dim=1)
    return wig[:, perm, :]


def envelope(dist, cutoff, p=5):
    """Polynomial envelope (tt_atom/geometry.py:201-206,249-251): for d = dist/cutoff < 1,
    ``1 + d^p (a + d (b + c d))`` with a = -(p+1)(p+2)/2, b = p(p+2), c = -p(p+1)/2; else 0."""
    a, b, c = -(p + 1) * (p + 2) / 2, p * (p + 2), -p * (p + 1) / 2
    ds = dist / cutoff
    val = 1 + (ds ** p) * (a + ds * (b + c * ds))
    return torch.where(ds < 1, val, torch.zeros_like(val))


def csd_embedding(w, charge, spin, C, dataset="omat"):
    """System embedding [nsys, C] (tt_atom/geometry.py:23-45): sin/cos charge & spin encodings
    (spin 0 zeroed) or learned lookups, plus the dataset token, mixed by a SiLU linear."""
    if "charge_embedding.rand_emb.weight" in w:
        chg = F.embedding(charge.long() + 100, w["charge_embedding.rand_emb.weight"])
        sp = F.embedding(spin.long(), w["spin_embedding.rand_emb.weight"])
    else:
        def enc(v, W, zero_at_0):
            arg = v[:, None] * W[None, :] * 2 * math.pi
            e = torch.cat([torch.sin(arg), torch.cos(arg)], dim=-1)
            if zero_at_0:
                e = e.clone()
                e[v == 0] = 0
            return e
        chg = enc(charge, w["charge_embedding.W"], False)
        sp = enc(spin, w["spin_embedding.W"], True)
    ds = w[f"dataset_embedding.dataset_emb_dict.{dataset}.weight"][0].expand(charge.shape[0], -1)
    return F.silu(F.linear(torch.cat([chg, sp, ds], 1), w["mix_csd.weight"], w["mix_csd.bias"]))


def radial_mlp(x, w, p):
    """Linear -> LayerNorm -> SiLU -> Linear -> LayerNorm -> SiLU -> Linear (tests/mirror.py:21-28)."""
    x = F.linear(x, w[f"{p}.net.0.weight"], w[f"{p}.net.0.bias"])
    x = F.silu(F.layer_norm(x, (x.shape[-1],), w[f"{p}.net.1.weight"], w[f"{p}.net.1.bias"], 1e-5))
    x = F.linear(x, w[f"{p}.net.3.weight"], w[f"{p}.net.3.bias"])
    x = F.silu(F.layer_norm(x, (x.shape[-1],), w[f"{p}.net.4.weight"], w[f"{p}.net.4.bias"], 1e-5))
    return F.linear(x, w[f"{p}.net.6.weight"], w[f"{p}.net.6.bias"])


def geometry(w, cfg, tables, pos, Z, edge_index, sys_emb, edge_vec=None, shift=None):
    """Per-edge geometric terms and the edge-degree node init (tt_atom/geometry.py:226-280)."""
    C, lmax = cfg["sphere_channels"], cfg["lmax"]
    src, tgt = edge_index[0], edge_index[1]
    if edge_vec is None:
        edge_vec = pos[src] - pos[tgt]
        if shift is not None:
            edge_vec = edge_vec + shift
    dist = torch.linalg.norm(edge_vec, dim=1)
    wig = wigner_m(edge_vec, [tables[f"Jd_{l}"] for l in range(lmax + 1)], tables["to_m"], lmax)
    gauss = torch.exp(tables["gauss_coeff"].reshape(-1)[0]
                      * (dist[:, None] - tables["gauss_offset"][None, :]) ** 2)
    x_edge = torch.cat([gauss, w["source_embedding.weight"][Z[src]],
                        w["target_embedding.weight"][Z[tgt]]], 1)
    env = envelope(dist, cfg["cutoff"]).reshape(-1, 1, 1)
    N, nsph = Z.shape[0], (lmax + 1) ** 2
    l0 = w["sphere_embedding.weight"][Z] + sys_emb
    edm = radial_mlp(x_edge, w, "edge_degree_embedding.rad_func").reshape(-1, lmax + 1, C)
    edm = F.pad(edm, (0, 0, 0, nsph - (lmax + 1)))
    edm = torch.bmm(wig.transpose(1, 2), edm) * env
    x_init = torch.zeros(N, nsph, C, dtype=pos.dtype).index_add(0, tgt, edm / 5.0)
    x_init = x_init + F.pad(l0[:, None, :], (0, 0, 0, nsph - 1))
    return dict(wigner=wig, x_edge=x_edge, envelope=env, x_init=x_init, dist=dist,
                edge_vec=edge_vec)


# --------------------------------------------------------------------------- backbone


def _l_of(lmax):
    return [l for l in range(lmax + 1) for _ in range(2 * l + 1)]


def gate_index(lmax, mmax):
    """Gate row per vector coefficient in m-primed order (tt_atom/activation.py:19-26)."""
    idx = list(range(lmax))
    for m in range(1, mmax + 1):
        r = list(range(m - 1, lmax))
        idx += r + r
    return idx


def so2_conv(x, x_edge, w, p, lmax, mmax, cin, extra):
    """SO(2) convolution over m-primed coefficients (tests/mirror.py:31-61): optional radial
    multiplier, m=0 dense linear with bias, and per m>0 one linear on [real; imag] combined as
    (a - d, c + b). Returns (out [E, nsph, Hout], extra gating scalars or None)."""
    E, nsph = x.shape[0], (lmax + 1) ** 2
    xf = x.reshape(E, nsph * cin)
    nc = [lmax - m + 1 for m in range(mmax + 1)]
    if f"{p}.rad_func.net.0.weight" in w:
        rad = radial_mlp(x_edge, w, f"{p}.rad_func")
        parts, o = [], 0
        for m in range(mmax + 1):
            parts.append(rad[:, o:o + nc[m] * cin])
            o += nc[m] * cin
        mult = torch.cat([parts[0]] + [t for m in range(1, mmax + 1) for t in (parts[m], parts[m])], 1)
        xf = xf * mult
    y0 = F.linear(xf[:, :nc[0] * cin], w[f"{p}.fc_m0.weight"], w[f"{p}.fc_m0.bias"])
    gating = None
    if extra:
        gating, y0 = y0[:, :extra], y0[:, extra:]
    outs, off = [y0], nc[0] * cin
    for m in range(1, mmax + 1):
        k = nc[m] * cin
        blk = xf[:, off:off + 2 * k].reshape(E, 2, k) @ w[f"{p}.so2_m_conv.{m-1}.fc.weight"].T
        h = blk.shape[-1] // 2
        a, b = blk[:, 0, :h], blk[:, 0, h:]
        c, d = blk[:, 1, :h], blk[:, 1, h:]
        outs += [a - d, c + b]
        off += 2 * k
    out = torch.cat(outs, 1).reshape(E, nsph, -1)
    return out, gating


def rms_norm_sh(x, w, p, lmax, eps=1e-5):
    """Equivariant RMS norm (tests/mirror.py:64-75): centre l=0 over channels, degree-balanced
    mean square with weights 1/(2l+1)/(lmax+1), per-degree affine, l=0 bias."""
    lc = _l_of(lmax)
    nsph = len(lc)
    bdw = torch.tensor([1.0 / (2 * l + 1) / (lmax + 1) for l in lc]).view(1, nsph, 1)
    l0 = x[:, :1, :]
    x = torch.cat([l0 - l0.mean(2, keepdim=True), x[:, 1:, :]], 1)
    ms = (x * x * bdw).sum(1, keepdim=True).mean(2, keepdim=True)
    out = x * (torch.rsqrt(ms + eps) * w[f"{p}.affine_weight"][torch.tensor(lc)][None])
    return torch.cat([out[:, :1, :] + w[f"{p}.affine_bias"].view(1, 1, -1), out[:, 1:, :]], 1)


def gate(gating, x, lmax, mmax):
    """SiLU on l=0, sigmoid(gating[degree]) on every vector coefficient (tests/mirror.py:78-82)."""
    E, H = x.shape[0], x.shape[2]
    g = torch.sigmoid(gating).view(E, lmax, H)[:, gate_index(lmax, mmax), :]
    return torch.cat([F.silu(x[:, :1, :]), x[:, 1:, :] * g], 1)


def grid_ff(x, w, p, to_grid, from_grid):
    """Grid feed-forward (tests/mirror.py:85-92): project to the S2 grid, 3-layer SiLU MLP
    without bias, project back."""
    tg = to_grid.reshape(-1, to_grid.shape[-1])
    fg = from_grid.reshape(-1, from_grid.shape[-1])
    g = torch.einsum("pi,nic->npc", tg, x)
    g = F.silu(g @ w[f"{p}.grid_mlp.0.weight"].T)
    g = F.silu(g @ w[f"{p}.grid_mlp.2.weight"].T)
    g = g @ w[f"{p}.grid_mlp.4.weight"].T
    return torch.einsum("pi,npc->nic", fg, g)


def spectral_ff(x, w, p, lmax):
    """Spectral feed-forward (tt_atom/spectral.py:168-188, fairchem SpectralAtomwise): gating =
    SiLU(scalar MLP on l = 0); per-degree SO3 linear (one weight per l, bias on l = 0); SiLU on
    l = 0 and sigmoid(gating[degree]) on l >= 1; second SO3 linear."""
    N, nsph, _ = x.shape
    lc = torch.tensor(_l_of(lmax))
    gating = F.silu(F.linear(x[:, 0], w[f"{p}.scalar_mlp.0.weight"], w[f"{p}.scalar_mlp.0.bias"]))
    W1, b1 = w[f"{p}.so3_linear_1.weight"], w[f"{p}.so3_linear_1.bias"]
    h = torch.einsum("nic,ihc->nih", x, W1[lc])
    h = torch.cat([h[:, :1] + b1, h[:, 1:]], 1)
    H = h.shape[2]
    sg = torch.sigmoid(gating).view(N, lmax, H)
    g = torch.cat([F.silu(h[:, :1])] + [h[:, l * l:(l + 1) ** 2] * sg[:, l - 1:l]
                                         for l in range(1, lmax + 1)], 1)
    W2, b2 = w[f"{p}.so3_linear_2.weight"], w[f"{p}.so3_linear_2.bias"]
    out = torch.einsum("nih,ich->nic", g, W2[lc])
    return torch.cat([out[:, :1] + b2, out[:, 1:]], 1)


def edgewise(x, w, p, cfg, wig, x_edge, env, edge_index, N):
    """Edgewise message block (tests/mirror.py:95-109)."""
    C, H, lmax, mmax = cfg["sphere_channels"], cfg["hidden_channels"], cfg["lmax"], cfg["mmax"]
    src, tgt = edge_index[0], edge_index[1]
    m = torch.bmm(wig, torch.cat([x[src], x[tgt]], 2))
    m, gating = so2_conv(m, x_edge, w, f"{p}.so2_conv_1", lmax, mmax, 2 * C, lmax * H)
    m = gate(gating, m, lmax, mmax)
    m, _ = so2_conv(m, x_edge, w, f"{p}.so2_conv_2", lmax, mmax, H, 0)
    m = torch.bmm(wig.transpose(1, 2), m * env)
    return torch.zeros(N, m.shape[1], C, dtype=m.dtype).index_add(0, tgt, m)


def backbone(w, cfg, tables, x_init, wig, x_edge, env, sys_emb, edge_index):
    """Blocks of norm -> +sys_emb(l0) -> edgewise -> residual -> norm -> grid FF -> residual,
    then the final norm (tests/mirror.py:112-126)."""
    lmax, N = cfg["lmax"], x_init.shape[0]
    x = x_init
    for i in range(cfg["num_layers"]):
        p = f"blocks.{i}"
        n = rms_norm_sh(x, w, f"{p}.norm_1", lmax)
        n = torch.cat([n[:, :1, :] + sys_emb[:, None, :], n[:, 1:, :]], 1)
        x = edgewise(n, w, f"{p}.edge_wise", cfg, wig, x_edge, env, edge_index, N) + x
        n = rms_norm_sh(x, w, f"{p}.norm_2", lmax)
        if cfg.get("ff_type", "grid") == "spectral":
            x = spectral_ff(n, w, f"{p}.atom_wise", lmax) + x
        else:
            x = grid_ff(n, w, f"{p}.atom_wise", tables["to_grid_mat"], tables["from_grid_mat"]) + x
    return rms_norm_sh(x, w, "norm", lmax)


def node_energy(node_emb, w):
    """Energy head on the l=0 row: Linear-SiLU-Linear-SiLU-Linear (tests/mirror.py:129-134),
    per node (the caller sums)."""
    h = node_emb[:, 0, :]
    h = F.silu(F.linear(h, w["energy_block.0.weight"], w["energy_block.0.bias"]))
    h = F.silu(F.linear(h, w["energy_block.2.weight"], w["energy_block.2.bias"]))
    return F.linear(h, w["energy_block.4.weight"], w["energy_block.4.bias"]).reshape(-1)


# --------------------------------------------------------------------------- E, F, stress


def energy_forces(w, cfg, tables, pos, Z, edge_index, shift=None, sys_emb=None,
                  compute_stress=False, batch=None, nsys=1, charge=0.0, spin=0.0):
    """Energy, forces ``-dE/dpos`` and (optionally) the virial ``dE/d(strain)`` by autograd.

    ``batch`` (per-atom system id) gives per-system energies for a disjoint-union batch; forces
    of the summed energy are per-system forces because the graph is block-diagonal
    (tt_atom/forces.py:616-637). Returns dict(energy [nsys], forces [N,3], virial [3,3]|None)."""
    C = cfg["sphere_channels"]
    if sys_emb is None:
        se = csd_embedding(w, torch.tensor([float(charge)]), torch.tensor([float(spin)]), C,
                           cfg.get("task", "omat"))
        sys_emb = se.expand(Z.shape[0], -1)
    pos = pos.detach().clone().requires_grad_(True)
    src, tgt = edge_index[0], edge_index[1]
    strain, edge_vec = None, None
    if compute_stress:
        strain = torch.zeros(3, 3, dtype=pos.dtype, requires_grad=True)
        ev = pos[src] - pos[tgt]
        if shift is not None:
            ev = ev + shift
        edge_vec = ev + ev @ (0.5 * (strain + strain.transpose(0, 1)))
    t = geometry(w, cfg, tables, pos, Z, edge_index, sys_emb, edge_vec=edge_vec, shift=shift)
    ne = backbone(w, cfg, tables, t["x_init"], t["wigner"], t["x_edge"], t["envelope"], sys_emb,
                  edge_index)
    e_node = node_energy(ne, w)
    if batch is None:
        energies = e_node.sum().reshape(1)
    else:
        energies = torch.zeros(nsys, dtype=e_node.dtype).index_add(0, batch, e_node)
    inputs = [pos] if strain is None else [pos, strain]
    grads = torch.autograd.grad(energies.sum(), inputs)
    return dict(energy=energies.detach(), forces=-grads[0],
                virial=grads[1] if compute_stress else None, node_emb=ne.detach())


def voigt_stress(virial, volume):
    """3x3 virial / volume -> Voigt (xx, yy, zz, yz, xz, xy), as ASE's
    ``full_3x3_to_voigt_6_stress`` (tt_atom/calculator.py:159-165)."""
    s = virial / volume
    s = 0.5 * (s + s.T)
    return torch.stack([s[0, 0], s[1, 1], s[2, 2], s[1, 2], s[0, 2], s[0, 1]])
