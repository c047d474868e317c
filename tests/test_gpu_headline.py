"""Parity at the benchmarked sizes: the CUDA path against the oracle on the configurations
``bench.py`` measures, not only on small cells.

* Config 2 (the headline): periodic 2,000-atom fcc Cu/Ni, uma-s-1 shape, cap 30 (E = 60,000),
  energy / forces / stress in every precision mode, and the neighbour list bit-exact.
* Config 3: periodic 1,002-atom amorphous SiO2, Orb-v3 shape, cap 20, E / F / stress, and its
  neighbour list bit-exact.
* Config 4 (screening): a subset of the 512 molecules that includes molecules with more than 31
  atoms, where the cap of 30 neighbours binds, through ``evaluate_batch`` (one disjoint union).

Tolerances are the fp32 ones of the hot path's contract: energy <= 1e-5 relative, forces
<= 1e-4 eV/A max-abs, stress <= 1e-5 eV/A^3 max-abs; edge lists and image shifts bit-exact.
The oracle (fp32 torch on the host) takes ~10-25 s per config-2 evaluation; it runs once per
module and is shared by the precision modes."""
import os

import numpy as np
import pytest
import torch

from oracle import orb as OB
from oracle import uma as O
from tt_atom import configs
from tt_atom.calculator import TTAtomCalculator
from tt_atom.graph import radius_graph
from tt_atom.orb import OrbCalculator
from tt_atom.weights import WeightBundle

pytestmark = pytest.mark.gpu

E_REL, F_ABS, S_ABS = 1e-5, 1e-4, 1e-5
PRECISIONS = ["fp32", "3xtf32", "3xf16"]


def _tables(cfg):
    t = configs.lmax2_tables()
    off, coeff = configs.gaussian_basis(cfg)
    return dict(t, gauss_offset=off, gauss_coeff=coeff)


@pytest.fixture(scope="module")
def config2():
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = configs.model_config("uma-s-1")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    s = configs.fcc_alloy(reps=(10, 10, 5), seed=1)
    pos, cell = torch.from_numpy(s["pos"]), torch.from_numpy(s["cell"])
    ei, sh = O.neighbor_list(pos, cfg["cutoff"], cell, [True] * 3, cfg["max_neighbors"])
    r = O.energy_forces(b.weights, cfg, _tables(cfg), pos, torch.from_numpy(s["Z"]), ei, sh,
                        compute_stress=True)
    return cfg, b, s, ei, sh, r


def test_config2_neighbor_list_bit_exact(config2):
    cfg, _, s, ei_o, sh_o, _ = config2
    ei, sh = radius_graph(s["pos"], cfg["cutoff"], s["cell"], [True] * 3,
                          max_neighbors=cfg["max_neighbors"])
    assert ei.shape[1] == 60000
    assert torch.equal(ei, ei_o)
    assert torch.equal(sh, sh_o)


@pytest.mark.parametrize("precision", PRECISIONS)
def test_config2_energy_forces_stress_vs_oracle(config2, precision):
    cfg, b, s, _, _, r = config2
    calc = TTAtomCalculator(b, precision=precision)
    E, F, V = calc._evaluate(s["pos"], s["Z"], s["cell"], [True] * 3, [0.0], [0.0],
                             forces=True, stress=True)
    assert calc._ws.graph.E == 60000
    E_ref = float(r["energy"][0])
    assert abs(float(E[0]) - E_ref) <= E_REL * abs(E_ref), (float(E[0]), E_ref)
    assert (F.float() - r["forces"]).abs().max() <= F_ABS
    vol = abs(np.linalg.det(s["cell"].astype(np.float64)))
    assert (V.float() - r["virial"]).abs().max() / vol <= S_ABS


@pytest.fixture(scope="module")
def config3():
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = configs.orb_config("orb-v3")
    w = configs.orb_random_weights(cfg, seed=0)
    s = configs.amorphous_sio2()
    pos, cell = torch.from_numpy(s["pos"]), torch.from_numpy(s["cell"])
    ei, sh = O.neighbor_list(pos, cfg["cutoff"], cell, [True] * 3, cfg["max_num_neighbors"])
    r = OB.energy_forces(w, cfg, pos, torch.from_numpy(s["Z"]), ei, sh, compute_stress=True)
    return cfg, w, s, ei, sh, r


def test_config3_neighbor_list_bit_exact(config3):
    cfg, _, s, ei_o, sh_o, _ = config3
    ei, sh = radius_graph(s["pos"], cfg["cutoff"], s["cell"], [True] * 3,
                          max_neighbors=cfg["max_num_neighbors"])
    assert ei.shape[1] == 20 * len(s["Z"])
    assert torch.equal(ei, ei_o)
    assert torch.equal(sh, sh_o)


@pytest.mark.parametrize("precision", PRECISIONS)
def test_config3_orb_energy_forces_stress_vs_oracle(config3, precision):
    cfg, w, s, _, _, r = config3
    calc = OrbCalculator(w, cfg=cfg, precision=precision)
    E, F, V = calc._evaluate(s["pos"], s["Z"], s["cell"], [True] * 3, True, True)
    E_ref = float(r["energy"])
    assert abs(E - E_ref) <= E_REL * max(abs(E_ref), 1.0), (E, E_ref)
    assert (F.float() - r["forces"]).abs().max() <= F_ABS
    vol = abs(np.linalg.det(s["cell"].astype(np.float64)))
    assert (V.float() - r["virial"]).abs().max() / vol <= S_ABS


@pytest.mark.parametrize("precision", ["fp32", "3xtf32"])
def test_config4_subset_with_binding_cap_vs_oracle(precision):
    cfg = configs.model_config("uma-s-1")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    mols = configs.screening_set()[:24]
    assert sum(len(m["Z"]) > 31 for m in mols) >= 5
    calc = TTAtomCalculator(b, precision=precision)
    out = calc.evaluate_batch(mols)
    tables = _tables(cfg)
    torch.set_num_threads(os.cpu_count() or 1)
    binding = 0
    for k, m in enumerate(mols):
        pos = torch.from_numpy(m["pos"])
        ei, _ = O.neighbor_list(pos, cfg["cutoff"], None, None, cfg["max_neighbors"])
        full, _ = O.neighbor_list(pos, cfg["cutoff"], None, None, None)
        binding += int(full.shape[1] > ei.shape[1])
        r = O.energy_forces(b.weights, cfg, tables, pos, torch.from_numpy(m["Z"]), ei, None)
        e_ref = b.scale_rmsd * float(r["energy"][0]) + b.scale_mean
        if b.elem_refs is not None:
            e_ref += float(b.elem_refs[torch.from_numpy(m["Z"])].sum())
        assert abs(out["energy"][k] - e_ref) <= E_REL * max(abs(e_ref), 1.0), (k, out["energy"][k], e_ref)
        f_ref = b.scale_rmsd * r["forces"].double()
        assert np.abs(out["forces"][k] - f_ref.numpy()).max() <= F_ABS, k
    assert binding >= 5          # the cap dropped edges in these molecules
