"""The Orb backbone pinned to the reference's own code (tests/golden/ref_run_orb.npz).

``make_golden.py`` ran the reference's Orb forward and hand-written reverse pass
(tt_atom/orb_model.py:92-338, tt_atom/orb_forces.py:307-372, with the host autograd finish
through tt_atom/orb_geometry.py) on the CPU through an fp32 torch stand-in for its ttnn calls,
on this framework's seeded inputs and random-init weights: an amorphous SiO2 cell at the tiny
shape and at the Orb-v3 shape (latent 256, hidden 1024, 5 layers), a molecule, and a molecule
with OrbMol charge / spin conditioning. The CPU tests pin the oracle restatement
(``oracle/orb.py``) to those values; the GPU tests pin the calculator (raw, normalised-space
energy, forces and virial, uncapped edges, no ZBL term) at the fp32 tolerances."""
import numpy as np
import pytest
import torch

from oracle import orb as OB
from tt_atom import configs

E_REL, F_ABS, S_ABS = 1e-5, 1e-4, 1e-5
CASES = {
    "tiny_sio2": ("orb-tiny", dict(seed=0)),
    "tiny_mol": ("orb-tiny", dict(seed=0)),
    "tiny_omol": ("orb-tiny", dict(seed=3, cond=True)),
    "v3_sio2": ("orb-v3", dict(seed=0)),
}


def _case(fx, name):
    d = fx("ref_run_orb.npz").d
    shape, kw = CASES[name]
    cfg = configs.orb_config(shape)
    w = configs.orb_random_weights(cfg, **kw)
    g = {k.split("@", 1)[1]: d[k] for k in d.files if k.startswith(name + "@")}
    return cfg, w, g


@pytest.mark.parametrize("name", list(CASES))
def test_oracle_matches_reference_orb_run(fx, name):
    cfg, w, g = _case(fx, name)
    periodic = "cell" in g
    q, sp = g["charge_spin"]
    r = OB.energy_forces(w, cfg, torch.from_numpy(g["pos"]), torch.from_numpy(g["Z"]),
                         torch.from_numpy(g["edge_index"]),
                         torch.from_numpy(g["shift"]) if periodic else None,
                         compute_stress=periodic, charge=float(q), spin=float(sp))
    e_ref = float(g["energy"])
    assert abs(float(r["energy"]) - e_ref) <= 1e-6 * max(1.0, abs(e_ref))
    assert (r["forces"] - torch.from_numpy(g["forces"])).abs().max() <= 1e-6
    if periodic:
        assert (r["virial"] - torch.from_numpy(g["virial"])).abs().max() <= 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("precision", ["fp32", "3xtf32", "3xf16"])
@pytest.mark.parametrize("name", list(CASES))
def test_gpu_orb_matches_reference_orb_run(fx, name, precision):
    from tt_atom.orb import OrbCalculator
    cfg, w, g = _case(fx, name)
    periodic = "cell" in g
    q, sp = g["charge_spin"]
    calc = OrbCalculator(w, cfg=cfg, precision=precision, zbl=False, max_num_neighbors=None)
    E, F, V = calc._evaluate(g["pos"], g["Z"], g["cell"] if periodic else None,
                             [True] * 3 if periodic else None, True, periodic,
                             charge=float(q), spin=float(sp))
    assert calc._ws.graph.E == g["edge_index"].shape[1]
    e_ref = float(g["energy"])
    assert abs(E - e_ref) <= E_REL * max(1.0, abs(e_ref)), (E, e_ref)
    assert np.abs(F.numpy() - g["forces"]).max() <= F_ABS
    if periodic:
        vol = abs(np.linalg.det(g["cell"].astype(np.float64)))
        assert np.abs(V.numpy() - g["virial"]).max() / vol <= S_ABS
