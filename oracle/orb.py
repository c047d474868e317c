"""CPU oracle for the Orb-v3 conservative energy + force + stress path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may import it. It
restates, in fp32 torch on the CPU, the reference's Orb port:

* edge features   -- tt_atom/orb_geometry.py:29-97 (Bessel basis, real SH lmax = 3 with
                     component normalisation, polynomial cutoff p = 4 from
                     tt_atom/orb_model.py:69-82); edge vector = pos[receiver] - pos[sender] +
                     shift, receivers/senders = UMA source/target (tt_atom/orb_calculator.py:110)
* MLPNorm         -- tt_atom/orb_model.py:92-173 (3 linears, SiLU after the first two,
                     RMSNorm eps 1e-6 without bias)
* interaction     -- tt_atom/orb_model.py:225-266 (sigmoid attention x cutoff, gathered edge
                     input, two segment sums, node MLP, residuals)
* energy head     -- tt_atom/orb_model.py:307-338 (node mean -> Linear-SiLU-Linear)
* conditioning    -- tt_atom/orb_model.py:32-57, 219-237 (OrbMol checkpoints: a closed-form
                     sin / cos embedding of the system's charge and spin, projected per layer
                     and added to the nodes at the layer's start)
* forces / stress -- autograd of the raw (normalised-space) energy w.r.t. positions and a
                     symmetric strain leaf on the edge vectors (tt_atom/orb_geometry.py:83-88)

* ZBL repulsion   -- tt_atom/orb_model.py:491-587 (host_zbl_energy and its autograd forces /
                     strain virial), in float64; covalent radii passed in (the reference reads
                     ase.data.covalent_radii, absent here)

Not restated: the energy normaliser / per-element references (host-side scalar glue,
tt_atom/orb_model.py:588-600). Parity is unpinned by
any committed Orb golden (the reference has none); it rests on this restatement of the
reference's own Orb code.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def bessel_basis(r, r_max=6.0, num_bases=8):
    n = torch.arange(1, num_bases + 1, dtype=r.dtype)
    w = math.pi / r_max * n
    return math.sqrt(2.0 / r_max) * torch.sin(w * r[:, None]) / r[:, None]


def spherical_harmonics_l3(u):
    """Real SH l = 0..3 of unit vectors, component normalisation (16 columns)."""
    x, y, z = u[:, 0], u[:, 1], u[:, 2]
    s3 = math.sqrt(3.0)
    y2, x2z2 = y * y, x * x + z * z
    s20, s21 = s3 * x * z, s3 * x * y
    s22, s23 = y2 - 0.5 * x2z2, s3 * y * z
    s24 = s3 / 2.0 * (z * z - x * x)
    cols = [torch.ones_like(x), x, y, z, s20, s21, s22, s23, s24,
            math.sqrt(5.0 / 6.0) * (s20 * z + s24 * x), math.sqrt(5.0) * s20 * y,
            math.sqrt(3.0 / 8.0) * (4.0 * y2 - x2z2) * x, 0.5 * y * (2.0 * y2 - 3.0 * x2z2),
            math.sqrt(3.0 / 8.0) * z * (4.0 * y2 - x2z2), math.sqrt(5.0) * s24 * y,
            math.sqrt(5.0 / 6.0) * (s24 * z - s20 * x)]
    sh = torch.stack(cols, -1)
    mult = torch.tensor([math.sqrt(2 * l + 1) for l in range(4) for _ in range(2 * l + 1)],
                        dtype=sh.dtype)
    return sh * mult


def cutoff_env(r, r_max=6.0, p=4):
    q = r / r_max
    v = (1.0 - ((p + 1.0) * (p + 2.0) / 2.0) * q ** p + p * (p + 2.0) * q ** (p + 1)
         - (p * (p + 1.0) / 2.0) * q ** (p + 2))
    return v * (r < r_max)


def edge_features(vectors, r_max, num_bases):
    r = torch.linalg.norm(vectors, dim=-1)
    rbf = bessel_basis(r, r_max, num_bases)
    ang = spherical_harmonics_l3(F.normalize(vectors, dim=-1))
    cut = cutoff_env(r, r_max)
    feat = cut[:, None] * (rbf[:, :, None] * ang[:, None, :]).reshape(r.shape[0], -1)
    return feat, cut


def mlp_norm(x, w, p):
    h = F.silu(F.linear(x, w[f"{p}.mlp.NN-0.weight"], w[f"{p}.mlp.NN-0.bias"]))
    h = F.silu(F.linear(h, w[f"{p}.mlp.NN-1.weight"], w[f"{p}.mlp.NN-1.bias"]))
    h = F.linear(h, w[f"{p}.mlp.NN-2.weight"], w[f"{p}.mlp.NN-2.bias"])
    inv = torch.rsqrt((h * h).mean(-1, keepdim=True) + 1e-6)
    return h * inv * w[f"{p}.layer_norm.weight"]


def charge_spin_embedding(w, charge, spin):
    """[1, latent] embedding of a system's total charge and spin: [sin, cos] of value * W * 2 pi
    for each, a zero spin giving zeros (tt_atom/orb_model.py:32-57)."""
    def emb(v, W, is_spin):
        x = float(v) * W * 2.0 * math.pi
        e = torch.cat([torch.sin(x), torch.cos(x)])
        return torch.zeros_like(e) if is_spin and v == 0 else e
    return torch.cat([emb(charge, w["conditioner.charge_embedding.W"], False),
                      emb(spin, w["conditioner.spin_embedding.W"], True)])[None]


def interaction(nodes, edges, w, p, senders, receivers, cut, cond=None):
    N = nodes.shape[0]
    if cond is not None and f"{p}._cond_node_proj.weight" in w:
        nodes = nodes + F.linear(cond, w[f"{p}._cond_node_proj.weight"],
                                 w[f"{p}._cond_node_proj.bias"])
    ra = torch.sigmoid(F.linear(edges, w[f"{p}._receive_attn.weight"],
                                w[f"{p}._receive_attn.bias"])) * cut[:, None]
    sa = torch.sigmoid(F.linear(edges, w[f"{p}._send_attn.weight"],
                                w[f"{p}._send_attn.bias"])) * cut[:, None]
    e_in = torch.cat([edges, nodes[senders], nodes[receivers]], 1)
    ue = mlp_norm(e_in, w, f"{p}._edge_mlp")
    sent = torch.zeros(N, ue.shape[1], dtype=ue.dtype).index_add(0, senders, ue * sa)
    recv = torch.zeros(N, ue.shape[1], dtype=ue.dtype).index_add(0, receivers, ue * ra)
    un = mlp_norm(torch.cat([nodes, recv, sent], 1), w, f"{p}._node_mlp")
    return nodes + un, edges + ue


def energy_forces(w, cfg, pos, Z, edge_index, shift=None, compute_stress=False, charge=0.0,
                  spin=0.0):
    """Raw (normalised-space) energy, forces = -dE/dpos and virial dE/dstrain. ``edge_index``
    is the UMA-convention graph [src, tgt]; Orb uses senders = tgt, receivers = src."""
    src, tgt = edge_index[0], edge_index[1]
    senders, receivers = tgt, src
    pos = pos.detach().clone().requires_grad_(True)
    vec = pos[receivers] - pos[senders]
    if shift is not None:
        vec = vec + shift
    strain = None
    if compute_stress:
        strain = torch.zeros(3, 3, requires_grad=True)
        vec = vec + vec @ (0.5 * (strain + strain.T))
    feat, cut = edge_features(vec, cfg["cutoff"], cfg["num_bases"])
    nodes = mlp_norm(w["atom_emb.embeddings.weight"][Z], w, "_encoder._node_fn")
    edges = mlp_norm(feat, w, "_encoder._edge_fn")
    cond = (charge_spin_embedding(w, charge, spin)
            if "conditioner.charge_embedding.W" in w else None)
    for i in range(cfg["num_message_passing_steps"]):
        nodes, edges = interaction(nodes, edges, w, f"gnn_stacks.{i}", senders, receivers, cut,
                                   cond)
    mean = nodes.mean(0, keepdim=True)
    h = F.silu(F.linear(mean, w["energy_head.mlp.NN-0.weight"], w["energy_head.mlp.NN-0.bias"]))
    E = F.linear(h, w["energy_head.mlp.NN-1.weight"], w["energy_head.mlp.NN-1.bias"]).reshape(())
    ins = [pos] if strain is None else [pos, strain]
    g = torch.autograd.grad(E, ins)
    return dict(energy=E.detach(), forces=-g[0], virial=g[1] if compute_stress else None)


def zbl_energy_forces_virial(Z, src, tgt, pos, shift, rcov, node_aggregation="mean", p=6):
    """ZBL pair repulsion of tt_atom/orb_model.py:491-537 in float64 with its forces
    (-dE/dpos) and strain virial (dE/dstrain) by autograd. Orb senders = tgt, receivers = src;
    atomic numbers enter as Z + 1 (the upstream embedding-index convention kept by the
    reference)."""
    c = torch.tensor([0.1818, 0.5099, 0.2802, 0.02817], dtype=torch.float64).unsqueeze(1)
    d = torch.tensor([3.2, 0.9423, 0.4028, 0.2016], dtype=torch.float64).unsqueeze(1)
    rcov = torch.as_tensor(rcov, dtype=torch.float64)
    senders, receivers = tgt.long(), src.long()
    pos = pos.detach().double().clone().requires_grad_(True)
    strain = torch.zeros(3, 3, dtype=torch.float64, requires_grad=True)
    vec = pos[receivers] - pos[senders]
    if shift is not None:
        vec = vec + shift.double()
    vec = vec @ (torch.eye(3, dtype=torch.float64) + 0.5 * (strain + strain.T))
    Zu = Z[senders].double() + 1
    Zv = Z[receivers].double() + 1
    a = 0.4543 * 0.529 / (Zu.pow(0.300) + Zv.pow(0.300))
    x = vec.norm(dim=1)
    phi = (c * torch.exp(-d * (x / a).unsqueeze(0))).sum(dim=0)
    v_raw = 14.3996 * Zu * Zv / x * phi
    r_max = rcov[Zu.long()] + rcov[Zv.long()]
    t = x / r_max
    env = (1.0 - ((p + 1.0) * (p + 2.0) / 2.0) * t.pow(p) + p * (p + 2.0) * t.pow(p + 1)
           - (p * (p + 1.0) / 2.0) * t.pow(p + 2)) * (x < r_max).double()
    V = torch.zeros(Z.shape[0], dtype=torch.float64).index_add(0, senders, 0.5 * v_raw * env)
    E = V.mean() if node_aggregation == "mean" else V.sum()
    gp, gs = torch.autograd.grad(E, [pos, strain])
    return float(E.detach()), -gp, gs


def direct_predict(w, cfg, pos, Z, edge_index, shift=None, charge=0.0, spin=0.0):
    """Direct checkpoints: raw energy, raw per-atom forces with the net force removed and raw
    Voigt-6 stress from the final node features (tt_atom/orb_model.py:307-436: EnergyHead,
    ForceHead, StressHead), one forward pass without autograd."""
    src, tgt = edge_index[0], edge_index[1]
    senders, receivers = tgt, src
    with torch.no_grad():
        vec = pos[receivers] - pos[senders]
        if shift is not None:
            vec = vec + shift
        feat, cut = edge_features(vec, cfg["cutoff"], cfg["num_bases"])
        nodes = mlp_norm(w["atom_emb.embeddings.weight"][Z], w, "_encoder._node_fn")
        edges = mlp_norm(feat, w, "_encoder._edge_fn")
        cond = (charge_spin_embedding(w, charge, spin)
                if "conditioner.charge_embedding.W" in w else None)
        for i in range(cfg["num_message_passing_steps"]):
            nodes, edges = interaction(nodes, edges, w, f"gnn_stacks.{i}", senders, receivers,
                                       cut, cond)
        mean = nodes.mean(0, keepdim=True)

        def head(x, p):
            h = F.silu(F.linear(x, w[f"{p}.mlp.NN-0.weight"], w[f"{p}.mlp.NN-0.bias"]))
            return F.linear(h, w[f"{p}.mlp.NN-1.weight"], w[f"{p}.mlp.NN-1.bias"])
        E = head(mean, "energy_head").reshape(())
        fr = head(nodes, "forces_head")
        fr = fr - fr.mean(0, keepdim=True)
        sr = head(mean, "stress_head").reshape(6)
    return dict(energy=E, forces=fr, stress=sr)
