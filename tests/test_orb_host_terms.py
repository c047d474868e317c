"""Orb host-side terms pinned to the reference's own code (tests/golden/ref_orb_host_terms.npz,
written by tests/golden/make_golden.py from tt_atom/orb_model.py:491-600 of the reference):

* the ZBL pair repulsion (energy with per-node mean and sum aggregation, forces, Voigt stress):
  the float64 oracle restatement on CPU, and ``atom_orb_zbl`` on the GPU;
* the normalisers (energy head; conservative forces and stress; direct force and stress heads)
  and OrbMol's charge / spin conditioning vector: this package's host functions.

The fixture's covalent-radius table is this package's (ASE is not installed where the fixture
was made), so the table is not pinned; the formula, the Z + 1 indexing, the envelope and the
aggregation are."""
import numpy as np
import pytest
import torch

from oracle import orb as OB
from tt_atom.orb import (COVALENT_RADII, charge_spin_embedding, conservative_scale,
                         conservative_stress, energy_denormalize, force_denormalize,
                         stress_denormalize)

TOL_E, TOL_F, TOL_S = 1e-9, 1e-7, 1e-9


def _voigt(V, vol):
    S = V / vol
    return np.array([S[0, 0], S[1, 1], S[2, 2], 0.5 * (S[1, 2] + S[2, 1]),
                     0.5 * (S[0, 2] + S[2, 0]), 0.5 * (S[0, 1] + S[1, 0])])


@pytest.mark.parametrize("tag", ["p", "m"])
@pytest.mark.parametrize("agg", ["mean", "sum"])
def test_oracle_zbl_matches_reference(fx, tag, agg):
    d = fx("ref_orb_host_terms.npz").d
    ei = torch.from_numpy(d[f"{tag}_edge_index"])
    periodic = tag == "p"
    E, F, V = OB.zbl_energy_forces_virial(
        torch.from_numpy(d[f"{tag}_Z"]), ei[0], ei[1], torch.from_numpy(d[f"{tag}_pos"]),
        torch.from_numpy(d[f"{tag}_shift"]) if periodic else None, COVALENT_RADII,
        node_aggregation=agg)
    e_ref = float(d[f"{tag}_zbl_energy_{agg}"])
    assert abs(e_ref) > 1e-2
    assert abs(E - e_ref) <= TOL_E * max(1.0, abs(e_ref))
    assert np.abs(F.numpy() - d[f"{tag}_zbl_forces_{agg}"]).max() <= TOL_F * max(1.0, abs(e_ref))
    if periodic:
        vol = abs(np.linalg.det(d["p_cell"].astype(np.float64)))
        assert np.abs(_voigt(V.numpy(), vol) - d[f"p_zbl_stress_{agg}"]).max() <= TOL_S


def test_energy_denormalize_matches_reference(fx):
    d = fx("ref_orb_host_terms.npz").d
    w = {"energy_head.normalizer.bn.running_mean": torch.from_numpy(d["denorm_mean"]),
         "energy_head.normalizer.bn.running_var": torch.from_numpy(d["denorm_var"]),
         "energy_head.reference.linear.weight": torch.from_numpy(d["denorm_ref"]).reshape(1, -1)}
    for k in range(3):
        out = energy_denormalize(float(d["denorm_raw"][k]), d["p_Z"], w)
        assert abs(out - float(d["denorm_out"][k])) <= 1e-12 * max(1.0, abs(out))
        # the device path hands it a tensor
        t = energy_denormalize(torch.tensor(float(d["denorm_raw"][k]), dtype=torch.float64),
                               d["p_Z"], w)
        assert abs(float(t) - float(d["denorm_out"][k])) <= 1e-12 * max(1.0, abs(out))
    assert energy_denormalize(1.5, d["p_Z"], {}) == 1.5


def test_head_normalisers_match_reference(fx):
    d = fx("ref_orb_host_terms.npz").d
    t = lambda k: torch.from_numpy(d[k])  # noqa: E731
    w = {"forces_head.normalizer.bn.running_mean": t("fnorm_mean"),
         "forces_head.normalizer.bn.running_var": t("fnorm_var"),
         "stress_head.diag_normalizer.bn.running_mean": t("snorm_dmean"),
         "stress_head.diag_normalizer.bn.running_var": t("snorm_dvar"),
         "stress_head.offdiag_normalizer.bn.running_mean": t("snorm_omean"),
         "stress_head.offdiag_normalizer.bn.running_var": t("snorm_ovar"),
         "energy_head.normalizer.bn.running_var": t("denorm_var")}
    assert np.abs(force_denormalize(t("fnorm_raw"), w).numpy() - d["fnorm_out"]).max() <= 1e-12
    assert np.abs(stress_denormalize(t("snorm_raw"), w).numpy() - d["snorm_out"]).max() <= 1e-12
    # conservative checkpoints: forces and stress of the raw energy through sigma * n
    f = conservative_scale(w, 48) * d["fnorm_raw"]
    assert np.abs(f - d["cons_forces"]).max() <= 1e-12 * np.abs(f).max()
    s = conservative_stress(d["cons_virial"], 48, d["p_cell"], w)
    assert np.abs(s - d["cons_stress"]).max() <= 1e-12 * np.abs(s).max()


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_charge_spin_embedding_matches_reference(fx, tag):
    d = fx("ref_orb_host_terms.npz").d
    q, sp = d[f"cs_{tag}"]
    e = charge_spin_embedding(torch.from_numpy(d["cs_Wc"]), torch.from_numpy(d["cs_Ws"]), q, sp)
    assert np.abs(e.numpy() - d[f"cs_out_{tag}"]).max() <= 1e-12


@pytest.mark.gpu
@pytest.mark.parametrize("tag", ["p", "m"])
def test_gpu_zbl_matches_reference(fx, tag):
    """``atom_orb_zbl`` (+ the deterministic edge reduction to forces and virial) on the
    calculator's own graph of the fixture's structure, against the reference's values."""
    from tt_atom import configs
    from tt_atom.ase_compat import SimpleAtoms
    from tt_atom.orb import OrbCalculator
    d = fx("ref_orb_host_terms.npz").d
    cfg = configs.orb_config("orb-tiny")
    w = configs.orb_random_weights(cfg, seed=0)
    periodic = tag == "p"
    calc = OrbCalculator(w, cfg=cfg, zbl=False, max_num_neighbors=None)
    a = SimpleAtoms(d[f"{tag}_Z"], d[f"{tag}_pos"], d["p_cell"] if periodic else None, periodic)
    calc.calculate(a, ("energy", "forces", "stress") if periodic else ("energy", "forces"))
    for agg, scale in (("mean", None), ("sum", 1.0)):
        E, F, V = calc._zbl(calc._ws, periodic, scale=scale)
        e_ref = float(d[f"{tag}_zbl_energy_{agg}"])
        assert abs(E - e_ref) <= 1e-6 * max(1.0, abs(e_ref)), (agg, E, e_ref)
        f_ref = d[f"{tag}_zbl_forces_{agg}"]
        assert np.abs(F.numpy() - f_ref).max() <= 1e-4 * max(1.0, np.abs(f_ref).max())
        if periodic:
            vol = abs(np.linalg.det(d["p_cell"].astype(np.float64)))
            s_ref = d[f"p_zbl_stress_{agg}"]
            assert np.abs(_voigt(V.numpy(), vol) - s_ref).max() <= 1e-4 * max(1e-3, np.abs(s_ref).max())
