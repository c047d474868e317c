"""The CPU oracle against the reference's goldens and the reference's own CPU-path outputs."""
import numpy as np
import pytest
import torch

from oracle import uma as O


def _cfg_from(fx_cfg):
    cfg = dict(fx_cfg)
    cfg.setdefault("task", "omat")
    return cfg


@pytest.mark.parametrize("name,periodic", [("ref_golden_tiny.npz", False),
                                           ("ref_golden_bulk.npz", True)])
def test_oracle_matches_fairchem_golden(fx, name, periodic):
    """Oracle geometry + backbone + autograd reproduce the fairchem golden energy and forces."""
    g = fx(name)
    cfg, w, tb = _cfg_from(g.config), g.w(), g.tables()
    pos, Z = g.t("in@pos").float(), g.t("in@atomic_numbers").long()
    cell = g.t("in@cell")[0].float()
    ei, sh = O.radius_graph(pos, cfg["cutoff"], cell if periodic else None,
                            [True] * 3 if periodic else None)
    gold = g.t("in@edge_index").long()
    assert ei.shape == gold.shape
    assert set(map(tuple, ei.T.tolist())) == set(map(tuple, gold.T.tolist()))
    se = g.t("host@sys_node_embedding").float()
    r = O.energy_forces(w, cfg, tb, pos, Z, ei, sh if periodic else None, sys_emb=se)
    E_ref = float(g.t("out@energy")[0])
    assert abs(float(r["energy"][0]) - E_ref) <= 1e-5 * abs(E_ref)
    assert (r["forces"] - g.t("out@forces")).abs().max() < 1e-6
    # the system embedding restatement matches fairchem's
    se2 = O.csd_embedding(w, torch.tensor([0.0]), torch.tensor([0.0]), cfg["sphere_channels"])
    assert (se2[0] - se[0]).abs().max() < 1e-6


def test_oracle_geometry_matches_golden_host_terms(fx):
    g = fx("ref_golden_tiny.npz")
    cfg, w, tb = _cfg_from(g.config), g.w(), g.tables()
    pos, Z = g.t("in@pos").float(), g.t("in@atomic_numbers").long()
    ei = g.t("in@edge_index").long()
    t = O.geometry(w, cfg, tb, pos, Z, ei, g.t("host@sys_node_embedding").float())
    assert (t["dist"] - g.t("host@edge_distance")).abs().max() < 1e-6
    assert (t["x_edge"] - g.t("host@x_edge")).abs().max() < 1e-5
    assert (t["envelope"] - g.t("host@edge_envelope")).abs().max() < 1e-6


@pytest.mark.parametrize("name", ["ref_run_tiny_molecule.npz", "ref_run_tiny_fcc.npz"])
def test_oracle_matches_reference_cpu_path(fx, name):
    """Edge lists bit-exact, E/F/virial equal to the reference's own CPU path outputs."""
    g = fx(name)
    cfg, w, tb = g.config, g.w(), g.tables()
    pos, Z = g.t("in@pos").float(), g.t("in@Z").long()
    periodic = bool(g.d["in@pbc"])
    cell = g.t("in@cell").float() if periodic else None
    ei, sh = O.radius_graph(pos, cfg["cutoff"], cell, [True] * 3 if periodic else None)
    assert torch.equal(ei, g.t("out@edge_index").long())
    assert torch.equal(sh, g.t("out@shift"))
    r = O.energy_forces(w, cfg, tb, pos, Z, ei, sh if periodic else None,
                        compute_stress=periodic)
    E_ref = float(g.t("out@energy")[0])
    assert abs(float(r["energy"][0]) - E_ref) <= 1e-6 * abs(E_ref)
    assert (r["forces"] - g.t("out@forces")).abs().max() < 1e-6
    if periodic:
        assert (r["virial"] - g.t("out@virial")).abs().max() < 1e-5


def _fma32(a, b, c):
    """Exact fp32 fma(a, b, c) for fp32 numpy arrays: the product is exact in fp64; the fp64 sum
    is corrected with TwoSum so the final rounding to fp32 is a single correct rounding."""
    a, b, c = (np.asarray(v, np.float64) for v in (a, b, c))
    p = a * b
    s = p + c
    bb = s - p
    err = (p - (s - bb)) + (c - bb)                  # exact: p + c = s + err
    f = s.astype(np.float32)
    lo = np.where(f.astype(np.float64) > s, np.nextafter(f, np.float32(-np.inf)), f)
    hi = np.nextafter(lo, np.float32(np.inf))
    mid = (lo.astype(np.float64) + hi.astype(np.float64)) / 2
    tie = s == mid
    out = f.copy()
    out[tie & (err > 0)] = hi[tie & (err > 0)]
    out[tie & (err < 0)] = lo[tie & (err < 0)]
    return out


def test_fma_norm_matches_torch_linalg_norm():
    """The aperiodic cutoff test uses torch.linalg.norm; on the CPU that equals the correctly
    rounded sqrt(fma(z, z, fma(y, y, x*x))) in fp32, which the GPU neighbour list evaluates."""
    g = torch.Generator().manual_seed(0)
    for n in (7, 33, 1000, 100003):
        d = (torch.rand(n, 3, generator=g) * 14 - 7).float()
        x, y, z = (d[:, k].numpy() for k in range(3))
        s = _fma32(z, z, _fma32(y, y, x * x))
        # np.sqrt is correctly rounded (torch's vectorised CPU fp32 sqrt is not always)
        assert np.array_equal(np.sqrt(s), torch.linalg.norm(d, dim=-1).numpy())


def test_cap_rule_keeps_nearest_per_receiver():
    g = torch.Generator().manual_seed(1)
    pos = torch.rand(60, 3, generator=g) * 6
    ei, sh = O.radius_graph(pos, 4.0)
    keep = O.cap_neighbors(pos, ei, sh, False, 5)
    d = O.edge_rank_key(pos, ei, sh, False)
    for r in range(60):
        sel = ei[1] == r
        kd = d[sel & keep]
        dropped = d[sel & ~keep]
        assert kd.numel() == min(5, int(sel.sum()))
        if dropped.numel():
            assert kd.max() <= dropped.min()


def test_orb_oracle_geometry_matches_reference(fx):
    """Orb edge features of the oracle equal the reference's host_edge_features; the autograd
    VJP equals the reference's closed-form host_edge_features_vjp."""
    from oracle import orb as OB
    d = fx("ref_orb_geometry.npz").d
    pos = torch.from_numpy(d["pos"]).requires_grad_(True)
    ei = torch.from_numpy(d["edge_index"]).long()
    vec = pos[ei[0]] - pos[ei[1]] + torch.from_numpy(d["shift"])
    feat, cut = OB.edge_features(vec, 4.0, 8)
    assert (feat - torch.from_numpy(d["feat"])).abs().max() < 1e-5
    assert (cut - torch.from_numpy(d["cut"]).reshape(-1)).abs().max() < 1e-6
    (g,) = torch.autograd.grad([feat, cut], [pos], [torch.from_numpy(d["g_feat"]),
                                                   torch.from_numpy(d["g_cut"]).reshape(-1)])
    assert (-g - torch.from_numpy(d["forces"])).abs().max() < 1e-4


def test_orb_oracle_runs_tiny():
    import sys
    from oracle import orb as OB
    from tt_atom import configs
    cfg = configs.orb_config("orb-tiny")
    w = configs.orb_random_weights(cfg)
    s = configs.tiny_molecule()
    pos = torch.from_numpy(s["pos"])
    from oracle import uma as O
    ei, _ = O.neighbor_list(pos, cfg["cutoff"], max_neighbors=cfg["max_num_neighbors"])
    r = OB.energy_forces(w, cfg, pos, torch.from_numpy(s["Z"]), ei)
    assert torch.isfinite(r["energy"]) and torch.isfinite(r["forces"]).all()
    # net force of a conservative, translation-invariant model vanishes
    assert r["forces"].sum(0).abs().max() < 1e-4


def test_covalent_radii_table_matches_ase_when_available():
    """The ZBL term's covalent radii are ASE's table (Cordero et al. 2008); checked against
    ase.data where ASE is installed (it is not in every environment)."""
    from tt_atom.orb import COVALENT_RADII
    assert len(COVALENT_RADII) == 119 and COVALENT_RADII[14] == 1.11 and COVALENT_RADII[8] == 0.66
    ase_data = pytest.importorskip("ase.data")
    assert np.allclose(np.asarray(ase_data.covalent_radii), np.asarray(COVALENT_RADII))


def test_orb_charge_spin_embedding_restatement():
    """The OrbMol conditioning embedding of the oracle (tt_atom/orb_model.py:32-57): latent
    width, [sin, cos] halves per quantity, a zero spin giving zeros, charge-dependent."""
    import torch

    from oracle import orb as OB
    from tt_atom import configs
    cfg = configs.orb_config("orb-tiny")
    w = configs.orb_random_weights(cfg, seed=0, cond=True)
    C = cfg["latent_dim"]
    e = OB.charge_spin_embedding(w, 1.0, 0.0)
    assert e.shape == (1, C)
    assert torch.all(e[0, C // 2:] == 0)                        # spin 0 -> zero spin half
    x = w["conditioner.charge_embedding.W"] * 2 * torch.pi
    assert torch.allclose(e[0, :C // 4], torch.sin(x)) and torch.allclose(e[0, C // 4:C // 2], torch.cos(x))
    assert not torch.equal(OB.charge_spin_embedding(w, -1.0, 2.0)[0, :C // 2], e[0, :C // 2])
    assert torch.any(OB.charge_spin_embedding(w, 0.0, 2.0)[0, C // 2:] != 0)
