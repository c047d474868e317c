"""Orb-v3 conservative path on the GPU against the CPU oracle and the reference's geometry."""
import numpy as np
import pytest
import torch

from oracle import orb as OB
from oracle import uma as O
from tt_atom import _lib as L
from tt_atom import configs
from tt_atom._lib import call, ptr
from tt_atom.graph import build_graph
from tt_atom.orb import OrbCalculator

pytestmark = pytest.mark.gpu
E_REL, F_ABS, S_ABS = 1e-5, 1e-4, 1e-5


def test_orb_edge_features_and_vjp_vs_reference(fx):
    d = fx("ref_orb_geometry.npz").d
    pos = torch.from_numpy(d["pos"]).cuda()
    g = build_graph(d["pos"], np.zeros(40, np.int64), 4.0, d["cell"], [True] * 3)
    ei, _, perm = g.reference_order()
    assert torch.equal(ei.cpu(), torch.from_numpy(d["edge_index"]).long())
    E = g.E
    feat, cut, ev = torch.empty(E, 128).cuda(), torch.empty(E).cuda(), torch.empty(E, 3).cuda()
    s = L.stream_ptr()
    call("atom_orb_edge_features", ptr(pos), ptr(g.src), ptr(g.tgt), ptr(g.img), ptr(g.shifts),
         E, 4.0, 8, ptr(feat), ptr(cut), ptr(ev), s)
    assert (feat[perm].cpu() - torch.from_numpy(d["feat"])).abs().max() < 1e-5
    # the p = 4 polynomial cancels near r_max: compare to fp32 rounding of its terms
    assert (cut[perm].cpu() - torch.from_numpy(d["cut"]).reshape(-1)).abs().max() < 1e-5
    # VJP: feed the reference's random adjoints (in reference order) and reduce to forces
    gf, gc = torch.empty(E, 128), torch.empty(E)
    gf[perm.cpu()] = torch.from_numpy(d["g_feat"])
    gc[perm.cpu()] = torch.from_numpy(d["g_cut"]).reshape(-1)
    gf, gc = gf.cuda(), gc.cuda()
    gev = torch.empty(E, 3).cuda()
    call("atom_orb_edge_features_bwd", ptr(pos), ptr(g.src), ptr(g.tgt), ptr(g.img),
         ptr(g.shifts), E, 4.0, 8, ptr(gf), ptr(gc), ptr(gev), s)
    F = torch.empty(40, 3).cuda()
    call("atom_forces_virial", ptr(gev), ptr(ev), E, 40, ptr(g.recv_ptr), ptr(g.send_ptr),
         ptr(g.send_eid), ptr(F), None, None, s)
    assert (F.cpu() - torch.from_numpy(d["forces"])).abs().max() < 1e-4


def _run(shape, sysd, precision):
    cfg = configs.orb_config(shape)
    w = configs.orb_random_weights(cfg, seed=0)
    calc = OrbCalculator(w, cfg=cfg, precision=precision)
    periodic = sysd["pbc"]
    E, F, V = calc._evaluate(sysd["pos"], sysd["Z"], sysd["cell"] if periodic else None,
                             [True] * 3 if periodic else None, True, periodic)
    pos = torch.from_numpy(sysd["pos"])
    cell = torch.from_numpy(sysd["cell"]) if periodic else None
    ei, sh = O.neighbor_list(pos, cfg["cutoff"], cell, [True] * 3 if periodic else None,
                             cfg["max_num_neighbors"])
    r = OB.energy_forces(w, cfg, pos, torch.from_numpy(sysd["Z"]), ei,
                         sh if periodic else None, compute_stress=periodic)
    return E, F, V, r


@pytest.mark.parametrize("precision", ["fp32", "3xtf32", "3xf16"])
@pytest.mark.parametrize("shape,sysname", [("orb-tiny", "mol"), ("orb-v3", "sio2")])
def test_orb_energy_forces_stress_vs_oracle(shape, sysname, precision):
    if sysname == "mol":
        sysd = configs.tiny_molecule()
    else:
        sysd = configs.amorphous_sio2(n_si=20, n_o=40, seed=2)
    E, F, V, r = _run(shape, sysd, precision)
    E_ref = float(r["energy"])
    assert abs(E - E_ref) <= E_REL * max(abs(E_ref), 1.0), (E, E_ref)
    assert (F.float() - r["forces"]).abs().max() <= F_ABS
    if V is not None:
        vol = abs(np.linalg.det(sysd["cell"].astype(np.float64)))
        assert (V.float() - r["virial"]).abs().max() / vol <= S_ABS


def test_orb_trace_replays_bit_exact_across_topology_changes():
    """OrbCalculator(trace=True) captures the model pass once and replays it, also after the
    capped edge set changes at the same size (the workspace's topology arrays are updated in
    place); energies, forces and stresses equal the eager calculator bit for bit."""
    from tt_atom.ase_compat import SimpleAtoms
    cfg = configs.orb_config("orb-v3")
    w = configs.orb_random_weights(cfg, seed=0)
    sysd = configs.amorphous_sio2(n_si=40, n_o=80, seed=3)
    rng = np.random.default_rng(1)
    tr, ea = OrbCalculator(w, cfg=cfg, trace=True), OrbCalculator(w, cfg=cfg)
    step = None
    for k in range(3):
        p = sysd["pos"] + (rng.normal(0.0, 0.1, sysd["pos"].shape) if k else 0.0)
        out = []
        for calc in (tr, ea):
            calc.calculate(SimpleAtoms(sysd["Z"], p, sysd["cell"], True),
                           ("energy", "forces", "stress"))
            out.append((calc.results["energy"], calc.results["forces"].copy(),
                        calc.results["stress"].copy()))
        if step is None:
            step = tr._step
        assert tr._step is step
        (e0, f0, s0), (e1, f1, s1) = out
        assert e0 == e1 and np.array_equal(f0, f1) and np.array_equal(s0, s1)


def test_zbl_pair_repulsion_vs_oracle():
    """calculate() with zbl=True minus zbl=False is the ZBL term: energy, forces and stress
    against the float64 oracle restatement on the same edges (a compressed SiO2 cell, so many
    pairs sit inside r_cov(Z+1) sums)."""
    from tt_atom.ase_compat import SimpleAtoms
    from tt_atom.orb import COVALENT_RADII
    cfg = configs.orb_config("orb-tiny")
    w = configs.orb_random_weights(cfg, seed=0)
    s = configs.amorphous_sio2(n_si=20, n_o=40, seed=4)
    pos, cell = 0.85 * s["pos"], 0.85 * s["cell"]
    res = {}
    for zbl in (False, True):
        calc = OrbCalculator(w, cfg=cfg, zbl=zbl, max_num_neighbors=None)
        a = SimpleAtoms(s["Z"], pos, cell, True)
        calc.calculate(a, ("energy", "forces", "stress"))
        res[zbl] = (calc.results["energy"], calc.results["forces"], calc.results["stress"], calc)
    g = res[True][3]._ws.graph
    shift = g.shifts.double().cpu()[g.img.long().cpu()]
    Ez, Fz, Vz = OB.zbl_energy_forces_virial(torch.from_numpy(s["Z"]), g.src.cpu(), g.tgt.cpu(),
                                             torch.from_numpy(pos), shift, COVALENT_RADII)
    assert abs(Ez) > 1e-3                                    # the term is exercised
    dE = res[True][0] - res[False][0]
    assert abs(dE - Ez) <= 1e-6 * max(1.0, abs(Ez))
    dF = res[True][1] - res[False][1]
    assert np.abs(dF - Fz.numpy()).max() <= 1e-4 * max(1.0, np.abs(Fz.numpy()).max())
    vol = abs(np.linalg.det(cell.astype(np.float64)))
    S = Vz.numpy() / vol
    voigt = np.array([S[0, 0], S[1, 1], S[2, 2], 0.5 * (S[1, 2] + S[2, 1]),
                      0.5 * (S[0, 2] + S[2, 0]), 0.5 * (S[0, 1] + S[1, 0])])
    dS = res[True][2] - res[False][2]
    assert np.abs(dS - voigt).max() <= 1e-4 * max(1e-3, np.abs(voigt).max())


def test_direct_checkpoint_heads_vs_oracle():
    """A direct checkpoint (force and stress heads, no backward pass): the calculator's
    energy / forces / stress without ZBL equal the oracle's head outputs through the
    normalisers."""
    from tt_atom.ase_compat import SimpleAtoms
    cfg = configs.orb_config("orb-tiny")
    w = configs.orb_random_weights(cfg, seed=1, direct=True)
    s = configs.amorphous_sio2(n_si=20, n_o=40, seed=4)
    calc = OrbCalculator(w, cfg=cfg, zbl=False, max_num_neighbors=None)
    assert calc.engine.direct and calc.engine.has_stress_head
    a = SimpleAtoms(s["Z"], s["pos"], s["cell"], True)
    calc.calculate(a, ("energy", "forces", "stress"))
    pos = torch.from_numpy(s["pos"])
    ei, sh = O.neighbor_list(pos, cfg["cutoff"], torch.from_numpy(s["cell"]), [True] * 3, None)
    r = OB.direct_predict(w, cfg, pos, torch.from_numpy(s["Z"]), ei, sh)
    assert abs(calc.results["energy"] - float(r["energy"])) <= 1e-5 * max(1.0, abs(float(r["energy"])))
    fs = float(w["forces_head.normalizer.bn.running_var"].sqrt())
    fm = float(w["forces_head.normalizer.bn.running_mean"])
    assert np.abs(calc.results["forces"] - (r["forces"].numpy() * fs + fm)).max() <= 1e-4
    ds = float(w["stress_head.diag_normalizer.bn.running_var"].sqrt())
    dm = float(w["stress_head.diag_normalizer.bn.running_mean"])
    os_ = float(w["stress_head.offdiag_normalizer.bn.running_var"].sqrt())
    om = float(w["stress_head.offdiag_normalizer.bn.running_mean"])
    ref_s = np.concatenate([r["stress"][:3].numpy() * ds + dm, r["stress"][3:].numpy() * os_ + om])
    assert np.abs(calc.results["stress"] - ref_s).max() <= 1e-6
    # net force removed (before the per-component normaliser's mean is added back)
    assert np.abs((calc.results["forces"] - fm).sum(0)).max() <= 1e-3 * fs


def test_calculator_dispatches_orb_bundles(tmp_path):
    """tt_atom.Calculator picks the family from the bundle (tt_atom/auto.py:40-89): an Orb bundle
    gives an OrbCalculator whose results equal a directly built one; `task` is UMA-only."""
    import json

    import tt_atom
    from tt_atom.ase_compat import SimpleAtoms
    cfg = configs.orb_config("orb-tiny")
    w = configs.orb_random_weights(cfg, seed=0)
    arrs = {"config": np.frombuffer(json.dumps(cfg).encode(), dtype=np.uint8)}
    arrs.update({f"w@{k}": v.numpy() for k, v in w.items()})
    path = tmp_path / "orb_tiny.npz"
    np.savez(path, **arrs)
    m = configs.tiny_molecule()
    a = SimpleAtoms(m["Z"], m["pos"])
    calc = tt_atom.Calculator(a, str(path))
    assert isinstance(calc, OrbCalculator) and a.calc is calc
    e = a.get_potential_energy()
    ref = OrbCalculator(w, cfg=cfg)
    b = SimpleAtoms(m["Z"], m["pos"])
    b.calc = ref
    assert e == b.get_potential_energy()
    assert np.array_equal(a.get_forces(), b.get_forces())
    with pytest.raises(ValueError, match="applies only to UMA"):
        tt_atom.Calculator(None, str(path), task="omat")


def test_orb_evaluate_batch_matches_single_systems():
    """evaluate_batch (the reference's Orb batch API): per-system energies and forces equal what
    calculate gives for each system alone; mixed sizes allowed."""
    from tt_atom.ase_compat import SimpleAtoms
    cfg = configs.orb_config("orb-tiny")
    w = configs.orb_random_weights(cfg, seed=0)
    sysl = configs.screening_set(count=3, seed=11)
    calc = OrbCalculator(w, cfg=cfg, max_num_neighbors=None)
    out = calc.evaluate_batch(sysl)
    assert out["energy"].shape == (3,) and len(out["forces"]) == 3
    for k, s in enumerate(sysl):
        a = SimpleAtoms(s["Z"], s["pos"])
        a.calc = OrbCalculator(w, cfg=cfg, max_num_neighbors=None)
        assert out["energy"][k] == a.get_potential_energy()
        assert np.array_equal(out["forces"][k], a.get_forces())
    assert calc.evaluate_batch(sysl, properties=("energy",))["forces"] is None
    calc.close()
    assert calc._ws is None
    assert calc.evaluate_batch(sysl[:1])["energy"][0] == out["energy"][0]     # usable again


def test_orbmol_charge_spin_conditioning_vs_oracle():
    """OrbMol checkpoints (tt_atom/orb_model.py:32-57, 219-237): each layer adds the projected
    charge / spin embedding to its input nodes. Energy and forces match the oracle restatement
    for a charged, spin-polarised system and for charge 0 / spin 0 (whose spin embedding is
    zero), and the conditioning changes the energy."""
    cfg = configs.orb_config("orb-tiny")
    w = configs.orb_random_weights(cfg, seed=0, cond=True)
    m = configs.tiny_molecule()
    calc = OrbCalculator(w, cfg=cfg)
    assert calc.engine.has_cond
    pos = torch.from_numpy(m["pos"])
    ei, _ = O.neighbor_list(pos, cfg["cutoff"], None, None, cfg["max_num_neighbors"])
    energies = []
    for charge, spin in ((1.0, 2.0), (0.0, 0.0)):
        E, F, _ = calc._evaluate(m["pos"], m["Z"], None, None, True, False, charge=charge,
                                 spin=spin)
        r = OB.energy_forces(w, cfg, pos, torch.from_numpy(m["Z"]), ei, None, False,
                             charge=charge, spin=spin)
        assert abs(E - float(r["energy"])) <= E_REL * max(abs(float(r["energy"])), 1.0)
        assert (F.float() - r["forces"]).abs().max() <= F_ABS
        energies.append(E)
    assert energies[0] != energies[1]
