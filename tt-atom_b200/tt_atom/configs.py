"""Seeded synthetic workloads: model shapes, random-init weight bundles and input structures.

There are no real checkpoints or datasets on the benchmark machines, so every workload is
generated here from a seed:

* ``model_config(name)`` -- the eSCN-MD (UMA) hyper-parameters of a named shape:
  ``"tiny"`` (16 sphere channels, 2 layers, 8 Gaussians, cutoff 6) and ``"uma-s-1"``
  (128 channels, 4 layers, 512 Gaussians, cutoff 6, at most 30 neighbours per receiver).
* ``random_weights(cfg, seed)`` -- a full weight dict with the reference's key names and shapes
  (the ``w@`` keys of tt_atom/weights.py:90-130 in the reference) plus the fixed lmax=2 tables.
* ``system(name)`` -- the input structures: a 24-atom molecule, an fcc Cu/Ni alloy, a batch of
  screening molecules and a bcc Fe supercell.

The weight *distribution* is this framework's own choice (uniform fan-in scaled linears, unit-ish
norm affines, N(0,1) embeddings); only names, shapes and semantics follow the reference.
"""
from __future__ import annotations

import json
import math
import pathlib

import numpy as np
import torch

_TABLES = pathlib.Path(__file__).with_name("data") / "lmax2_tables.npz"

MODEL_SHAPES = {
    # config 1: tiny, CPU-runnable
    "tiny": dict(sphere_channels=16, hidden_channels=16, edge_channels=32, num_distance_basis=8,
                 lmax=2, mmax=2, num_layers=2, cutoff=6.0, max_neighbors=None),
    # configs 2, 4, 5: uma-s-1 shape (single merged expert)
    "uma-s-1": dict(sphere_channels=128, hidden_channels=128, edge_channels=128,
                    num_distance_basis=512, lmax=2, mmax=2, num_layers=4, cutoff=6.0,
                    max_neighbors=30),
}


def model_config(name, ff_type="grid"):
    """``ff_type``: "grid" (the reference's mirror and goldens) or "spectral" (real uma-s-1)."""
    cfg = dict(MODEL_SHAPES[name])
    cfg.update(norm_type="rms_norm_sh", act_type="gate", ff_type=ff_type, task="omat",
               max_num_elements=100)
    return cfg


def lmax2_tables():
    """The fixed lmax=mmax=2 tables: ``Jd_0..2``, ``to_m``, ``to_grid_mat``, ``from_grid_mat``."""
    z = np.load(_TABLES)
    return {k: torch.from_numpy(z[k].copy()).float() for k in z.files}


def gaussian_basis(cfg):
    """Gaussian radial basis buffers: ``offset = linspace(0, cutoff, NB)`` and
    ``coeff = -0.5 / (2 * spacing)^2`` (the reference bundles' ``host@gauss_offset`` /
    ``host@gauss_coeff``; width factor 2 as in fairchem's GaussianSmearing)."""
    nb, cut = cfg["num_distance_basis"], float(cfg["cutoff"])
    offset = torch.linspace(0.0, cut, nb, dtype=torch.float32)
    spacing = float(offset[1] - offset[0]) if nb > 1 else cut
    coeff = torch.tensor([-0.5 / (2.0 * spacing) ** 2], dtype=torch.float32)
    return offset, coeff


def random_weights(cfg, seed=0):
    """Random-init eSCN-MD weights with the reference key names (see module docstring)."""
    g = torch.Generator().manual_seed(seed)
    C, H, EC = cfg["sphere_channels"], cfg["hidden_channels"], cfg["edge_channels"]
    NB, L, lmax, mmax = cfg["num_distance_basis"], cfg["num_layers"], cfg["lmax"], cfg["mmax"]
    nel = cfg.get("max_num_elements", 100)
    w = {}

    def lin(name, fan_out, fan_in, bias=True):
        b = 1.0 / math.sqrt(fan_in)
        w[f"{name}.weight"] = (torch.rand(fan_out, fan_in, generator=g) * 2 - 1) * b
        if bias:
            w[f"{name}.bias"] = (torch.rand(fan_out, generator=g) * 2 - 1) * b

    def affine(name, *shape):
        w[f"{name}.weight"] = 1.0 + 0.1 * torch.randn(*shape, generator=g)
        w[f"{name}.bias"] = 0.1 * torch.randn(*shape, generator=g)

    def radial(p, out):
        fin = NB + 2 * EC
        lin(f"{p}.net.0", EC, fin)
        affine(f"{p}.net.1", EC)
        lin(f"{p}.net.3", EC, EC)
        affine(f"{p}.net.4", EC)
        lin(f"{p}.net.6", out, EC)

    w["sphere_embedding.weight"] = torch.randn(nel, C, generator=g)
    w["source_embedding.weight"] = torch.randn(nel, EC, generator=g)
    w["target_embedding.weight"] = torch.randn(nel, EC, generator=g)
    w["charge_embedding.W"] = torch.randn(C // 2, generator=g)
    w["spin_embedding.W"] = torch.randn(C // 2, generator=g)
    w[f"dataset_embedding.dataset_emb_dict.{cfg.get('task', 'omat')}.weight"] = \
        torch.randn(1, C, generator=g)
    lin("mix_csd", C, 3 * C)
    radial("edge_degree_embedding.rad_func", (lmax + 1) * C)
    ncoef = [lmax - m + 1 for m in range(mmax + 1)]
    for i in range(L):
        p = f"blocks.{i}"
        for nn in ("norm_1", "norm_2"):
            w[f"{p}.{nn}.affine_weight"] = 1.0 + 0.1 * torch.randn(lmax + 1, C, generator=g)
            w[f"{p}.{nn}.affine_bias"] = 0.1 * torch.randn(C, generator=g)
        # so2_conv_1: Cin = 2C, out H, extra lmax*H gating scalars, with a radial function
        cin = 2 * C
        radial(f"{p}.edge_wise.so2_conv_1.rad_func", sum(ncoef) * cin)
        lin(f"{p}.edge_wise.so2_conv_1.fc_m0", lmax * H + ncoef[0] * H, ncoef[0] * cin)
        for m in range(1, mmax + 1):
            lin(f"{p}.edge_wise.so2_conv_1.so2_m_conv.{m-1}.fc", 2 * ncoef[m] * H,
                ncoef[m] * cin, bias=False)
        # so2_conv_2: Cin = H, out C, no radial function
        lin(f"{p}.edge_wise.so2_conv_2.fc_m0", ncoef[0] * C, ncoef[0] * H)
        for m in range(1, mmax + 1):
            lin(f"{p}.edge_wise.so2_conv_2.so2_m_conv.{m-1}.fc", 2 * ncoef[m] * C,
                ncoef[m] * H, bias=False)
        if cfg.get("ff_type", "grid") == "spectral":
            lin(f"{p}.atom_wise.scalar_mlp.0", lmax * H, C)
            for name, fo, fi in (("so3_linear_1", H, C), ("so3_linear_2", C, H)):
                b = 1.0 / math.sqrt(fi)
                w[f"{p}.atom_wise.{name}.weight"] = \
                    (torch.rand(lmax + 1, fo, fi, generator=g) * 2 - 1) * b
                w[f"{p}.atom_wise.{name}.bias"] = (torch.rand(fo, generator=g) * 2 - 1) * b
        else:
            for gi in (0, 2, 4):
                lin(f"{p}.atom_wise.grid_mlp.{gi}", C, C, bias=False)
    w["norm.affine_weight"] = 1.0 + 0.1 * torch.randn(lmax + 1, C, generator=g)
    w["norm.affine_bias"] = 0.1 * torch.randn(C, generator=g)
    lin("energy_block.0", H, C)
    lin("energy_block.2", H, H)
    lin("energy_block.4", 1, H)
    t = lmax2_tables()
    for l in range(lmax + 1):
        w[f"Jd_{l}"] = t[f"Jd_{l}"]
    return {k: v.float().contiguous() for k, v in w.items()}


def random_bundle_arrays(cfg, seed=0):
    """The ``.npz`` arrays of a random-init bundle in the reference's bundle layout: ``config``
    (JSON bytes), ``w@<key>`` weights and the ``host@`` geometry buffers."""
    w = random_weights(cfg, seed)
    t = lmax2_tables()
    off, coeff = gaussian_basis(cfg)
    arrs = {"config": np.frombuffer(json.dumps(cfg).encode(), dtype=np.uint8)}
    arrs.update({f"w@{k}": v.numpy() for k, v in w.items()})
    arrs["host@to_m"] = t["to_m"].numpy()
    arrs["host@to_grid_mat"] = t["to_grid_mat"].numpy()
    arrs["host@from_grid_mat"] = t["from_grid_mat"].numpy()
    arrs["host@gauss_offset"] = off.numpy()
    arrs["host@gauss_coeff"] = coeff.numpy()
    return arrs


# ------------------------------------------------------------------------------- structures


def _reject_uniform(rng, n, box, min_dist, max_tries=200000):
    """Sequential rejection sampling: each new atom uniform in ``[0, box)^3`` and at least
    ``min_dist`` from all atoms placed before it."""
    pts = np.zeros((n, 3), dtype=np.float64)
    k, tries = 0, 0
    while k < n:
        p = rng.uniform(0.0, box, size=3)
        if k == 0 or np.min(np.linalg.norm(pts[:k] - p, axis=1)) >= min_dist:
            pts[k] = p
            k += 1
        tries += 1
        if tries > max_tries:
            raise RuntimeError("rejection sampling did not converge")
    return pts


def tiny_molecule(seed=0):
    """Config 1: 24 atoms (8 C, 10 H, 4 N, 2 O) uniform in an 8 A cube, min distance 0.9 A."""
    rng = np.random.default_rng(seed)
    Z = np.array([6] * 8 + [1] * 10 + [7] * 4 + [8] * 2, dtype=np.int64)
    pos = _reject_uniform(rng, len(Z), 8.0, 0.9)
    return dict(pos=pos.astype(np.float32), Z=Z, cell=None, pbc=False)


def fcc_alloy(reps=(10, 10, 5), a=3.55, jitter=0.05, seed=1):
    """Config 2: fcc Cu/Ni 50:50 random alloy, ``reps`` conventional cells, Gaussian jitter."""
    rng = np.random.default_rng(seed)
    basis = np.array([[0, 0, 0], [0.5, 0.5, 0], [0.5, 0, 0.5], [0, 0.5, 0.5]])
    grid = np.stack(np.meshgrid(*[np.arange(r) for r in reps], indexing="ij"), -1).reshape(-1, 3)
    frac = (grid[:, None, :] + basis[None, :, :]).reshape(-1, 3)
    pos = frac * a
    n = len(pos)
    Z = np.array([29] * (n // 2) + [28] * (n - n // 2), dtype=np.int64)
    Z = Z[rng.permutation(n)]
    pos = pos + rng.normal(0.0, jitter, size=pos.shape)
    cell = np.diag(np.array(reps, dtype=np.float64) * a)
    return dict(pos=pos.astype(np.float32), Z=Z, cell=cell.astype(np.float32), pbc=True)


def bcc_iron(reps=(32, 32, 32), a=2.87, jitter=0.05, seed=4):
    """Config 5: bcc Fe supercell (``reps`` cubic cells, 2 atoms each), Gaussian jitter."""
    rng = np.random.default_rng(seed)
    basis = np.array([[0, 0, 0], [0.5, 0.5, 0.5]])
    grid = np.stack(np.meshgrid(*[np.arange(r) for r in reps], indexing="ij"), -1).reshape(-1, 3)
    pos = (grid[:, None, :] + basis[None, :, :]).reshape(-1, 3) * a
    pos = pos + rng.normal(0.0, jitter, size=pos.shape)
    Z = np.full(len(pos), 26, dtype=np.int64)
    cell = np.diag(np.array(reps, dtype=np.float64) * a)
    return dict(pos=pos.astype(np.float32), Z=Z, cell=cell.astype(np.float32), pbc=True)


_SCREEN_EL = np.array([1, 6, 7, 8, 9, 16])
_SCREEN_P = np.array([0.45, 0.30, 0.10, 0.10, 0.03, 0.02])


def screening_set(count=512, nmin=10, nmax=60, seed=3):
    """Config 4: ``count`` independent molecules, n ~ U{nmin..nmax}, elements drawn
    H:C:N:O:F:S = .45/.30/.10/.10/.03/.02, cube side (12 n)^(1/3) A, min distance 0.9 A."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(count):
        n = int(rng.integers(nmin, nmax + 1))
        Z = rng.choice(_SCREEN_EL, size=n, p=_SCREEN_P).astype(np.int64)
        pos = _reject_uniform(rng, n, (12.0 * n) ** (1.0 / 3.0), 0.9)
        out.append(dict(pos=pos.astype(np.float32), Z=Z, cell=None, pbc=False))
    return out


def system(name):
    if name == "tiny":
        return tiny_molecule()
    if name == "fcc":
        return fcc_alloy()
    if name == "fcc-small":
        return fcc_alloy(reps=(3, 3, 3), seed=1)
    if name == "bcc-fe":
        return bcc_iron()
    raise KeyError(name)


# ------------------------------------------------------------------------------- Orb-v3 shape

ORB_SHAPES = {
    # config 3: Orb-v3-conservative shape (random init)
    "orb-v3": dict(latent_dim=256, hidden_dim=1024, node_embed_size=256, edge_embed_size=128,
                   num_bases=8, num_message_passing_steps=5, cutoff=6.0, max_num_neighbors=20,
                   head_hidden=256),
    # CPU-sized variant for tests
    "orb-tiny": dict(latent_dim=32, hidden_dim=64, node_embed_size=32, edge_embed_size=128,
                     num_bases=8, num_message_passing_steps=2, cutoff=6.0, max_num_neighbors=20,
                     head_hidden=32),
}


def orb_config(name):
    cfg = dict(ORB_SHAPES[name])
    cfg.update(family="orb", task="omat")
    return cfg


def orb_random_weights(cfg, seed=0, direct=False, cond=False):
    """Random-init Orb weights with the reference's key names (gns.MoleculeGNS naming as read by
    tt_atom/orb_model.py:127-338 in the reference); ``direct`` adds the force and stress heads
    and their normalisers of direct checkpoints (tt_atom/orb_model.py:358-457); ``cond`` the
    charge / spin conditioning of OrbMol checkpoints (embedding frequencies and per-layer node
    projections, tt_atom/orb_model.py:32-57, 219-237)."""
    g = torch.Generator().manual_seed(seed)
    C, Hd, L = cfg["latent_dim"], cfg["hidden_dim"], cfg["num_message_passing_steps"]
    w = {}

    def lin(name, fo, fi):
        b = 1.0 / math.sqrt(fi)
        w[f"{name}.weight"] = (torch.rand(fo, fi, generator=g) * 2 - 1) * b
        w[f"{name}.bias"] = (torch.rand(fo, generator=g) * 2 - 1) * b

    def mlpnorm(p, fi):
        lin(f"{p}.mlp.NN-0", Hd, fi)
        lin(f"{p}.mlp.NN-1", Hd, Hd)
        lin(f"{p}.mlp.NN-2", C, Hd)
        w[f"{p}.layer_norm.weight"] = 1.0 + 0.1 * torch.randn(C, generator=g)

    w["atom_emb.embeddings.weight"] = torch.randn(119, cfg["node_embed_size"], generator=g)
    mlpnorm("_encoder._node_fn", cfg["node_embed_size"])
    mlpnorm("_encoder._edge_fn", cfg["edge_embed_size"])
    for i in range(L):
        p = f"gnn_stacks.{i}"
        mlpnorm(f"{p}._edge_mlp", 3 * C)
        mlpnorm(f"{p}._node_mlp", 3 * C)
        lin(f"{p}._receive_attn", 1, C)
        lin(f"{p}._send_attn", 1, C)
        if cond:
            lin(f"{p}._cond_node_proj", C, C)
    if cond:
        w["conditioner.charge_embedding.W"] = torch.randn(C // 4, generator=g)
        w["conditioner.spin_embedding.W"] = torch.randn(C // 4, generator=g)
    lin("energy_head.mlp.NN-0", cfg["head_hidden"], C)
    lin("energy_head.mlp.NN-1", 1, cfg["head_hidden"])
    if direct:
        lin("forces_head.mlp.NN-0", cfg["head_hidden"], C)
        lin("forces_head.mlp.NN-1", 3, cfg["head_hidden"])
        lin("stress_head.mlp.NN-0", cfg["head_hidden"], C)
        lin("stress_head.mlp.NN-1", 6, cfg["head_hidden"])
        for p_, mu, var in (("forces_head.normalizer", 0.01, 0.3),
                            ("stress_head.diag_normalizer", -0.002, 0.0004),
                            ("stress_head.offdiag_normalizer", 0.0, 0.0001)):
            w[f"{p_}.bn.running_mean"] = torch.tensor([mu])
            w[f"{p_}.bn.running_var"] = torch.tensor([var])
    return {k: v.float().contiguous() for k, v in w.items()}


def amorphous_sio2(n_si=334, n_o=668, density=2.2, min_dist=1.4, seed=2):
    """Config 3: amorphous SiO2, uniform random positions at ``density`` g/cm^3 in a cubic box,
    rejection-sampled to ``min_dist`` A."""
    rng = np.random.default_rng(seed)
    mass = n_si * 28.0855 + n_o * 15.999                        # amu
    vol = mass * 1.66053906660e-24 / density * 1e24             # A^3
    side = vol ** (1.0 / 3.0)
    Z = np.array([14] * n_si + [8] * n_o, dtype=np.int64)
    Z = Z[rng.permutation(len(Z))]
    pos = _reject_uniform(rng, len(Z), side, min_dist)
    return dict(pos=pos.astype(np.float32), Z=Z,
                cell=np.diag([side] * 3).astype(np.float32), pbc=True)
