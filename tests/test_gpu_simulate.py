"""GPU-resident relaxation and MD through the calculator (tt_atom.simulate native loops), and
MultiCardSim relax / md workers, which use those loops when ASE is absent."""
import numpy as np
import pytest
import torch

from tt_atom import configs, dynamics as D
from tt_atom.ase_compat import SimpleAtoms
from tt_atom.calculator import TTAtomCalculator
from tt_atom.simulate import md_atoms, relax_atoms
from tt_atom.weights import WeightBundle

pytestmark = pytest.mark.gpu


def _tiny():
    cfg = configs.model_config("tiny")
    return cfg, WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))


def _molecule(calc, seed=0):
    m = configs.tiny_molecule(seed=seed)
    a = SimpleAtoms(m["Z"], m["pos"])
    a.calc = calc
    return a


def test_native_relax_lowers_energy_and_forces():
    _, b = _tiny()
    atoms = _molecule(TTAtomCalculator(b))
    e0 = float(atoms.get_potential_energy())
    f0 = float(np.linalg.norm(atoms.get_forces(), axis=1).max())
    res = relax_atoms(atoms, fmax=1e-3, steps=60, native=True)
    assert res["nsteps"] > 0 and f0 > 1e-3
    assert res["energy"] < e0                     # FIRE does not lower fmax monotonically
    assert res["converged"] == (res["fmax"] <= 1e-3) and (res["converged"] or res["nsteps"] == 60)
    # the result matches a fresh single point at the relaxed positions
    calc2 = TTAtomCalculator(b)
    a2 = SimpleAtoms(atoms.get_atomic_numbers(), atoms.get_positions())
    a2.calc = calc2
    assert abs(float(a2.get_potential_energy()) - res["energy"]) <= 1e-5 * abs(res["energy"])


def test_native_nve_conserves_energy_and_langevin_is_seeded():
    _, b = _tiny()
    calc = TTAtomCalculator(b)
    atoms = _molecule(calc)
    m = D.masses_of(atoms.get_atomic_numbers(), device="cuda")
    from tt_atom.simulate import _native_forces
    force_fn, pos = _native_forces(atoms)
    vel = D.maxwell_boltzmann(m, 300.0, torch.Generator(device="cuda").manual_seed(1))
    E0 = float(force_fn(pos)[0]) + D.kinetic_energy(vel, m)
    res = D.langevin(force_fn, pos, m, steps=40, dt_fs=0.25, friction_fs=0.0, vel=vel)
    E1 = res["energy"] + D.kinetic_energy(vel, m)
    assert abs(E1 - E0) <= 2e-3 * max(1.0, abs(E0))
    runs = []
    for _ in range(2):
        a = _molecule(TTAtomCalculator(b))
        md_atoms(a, steps=10, dt=0.5, temp=300.0, seed=7, native=True)
        runs.append(a.get_positions())
    assert np.array_equal(runs[0], runs[1])


def test_periodic_relax_wraps_positions_for_the_neighbour_list():
    cfg = configs.model_config("uma-s-1")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    s = configs.fcc_alloy(reps=(3, 3, 3), seed=2)
    a = SimpleAtoms(s["Z"], s["pos"] + np.array([20.0, -15.0, 9.0]), s["cell"], True)
    a.calc = TTAtomCalculator(b)
    ref = SimpleAtoms(s["Z"], s["pos"], s["cell"], True)
    ref.calc = TTAtomCalculator(b)
    from tt_atom.simulate import _native_forces
    e_shift = float(_native_forces(a)[0](_native_forces(a)[1])[0])
    e_ref = float(ref.get_potential_energy())
    assert abs(e_shift - e_ref) <= 1e-5 * abs(e_ref)
    res = relax_atoms(a, fmax=0.5, steps=5, native=True)
    assert np.isfinite(res["energy"])


def test_multicardsim_relax_and_md_without_ase(tmp_path):
    from tt_atom import MultiCardSim
    cfg, _ = _tiny()
    path = str(tmp_path / "tiny.npz")
    np.savez(path, **configs.random_bundle_arrays(cfg, seed=0))
    mols = [configs.tiny_molecule(seed=k) for k in range(3)]
    with MultiCardSim(path, device_ids=(0,), sim_params=dict(mode="relax", fmax=0.01,
                                                               steps=20)) as sim:
        out = sim.run([(m["pos"], m["Z"]) for m in mols])
    assert all(r["ok"] for r in out), [r.get("error") for r in out]
    assert all(r["nsteps"] > 0 for r in out)
    with MultiCardSim(path, device_ids=(0,), sim_params=dict(mode="md", steps=5, dt=0.5,
                                                               temp=300.0, seed=1)) as sim:
        out = sim.run([(m["pos"], m["Z"]) for m in mols])
    assert all(r["ok"] for r in out), [r.get("error") for r in out]


def test_native_relax_and_md_with_the_orb_calculator():
    """The GPU-resident loops also drive an OrbCalculator (its energy normaliser and ZBL term
    applied on the device): FIRE lowers the energy and ends at what a fresh single point gives;
    a few Langevin steps run."""
    from tt_atom.orb import OrbCalculator
    cfg = configs.orb_config("orb-tiny")
    w = configs.orb_random_weights(cfg, seed=0)
    m = configs.tiny_molecule(seed=0)
    atoms = SimpleAtoms(m["Z"], m["pos"])
    atoms.calc = OrbCalculator(w, cfg=cfg)
    e0 = float(atoms.get_potential_energy())
    res = relax_atoms(atoms, fmax=1e-3, steps=30, native=True)
    assert res["nsteps"] > 0 and res["energy"] < e0
    fresh = SimpleAtoms(atoms.get_atomic_numbers(), atoms.get_positions())
    fresh.calc = OrbCalculator(w, cfg=cfg)
    assert abs(float(fresh.get_potential_energy()) - res["energy"]) <= 1e-5 * max(1.0, abs(res["energy"]))
    out = md_atoms(atoms, steps=5, dt=0.5, temp=300.0, seed=3, native=True)
    assert out["nsteps"] == 5 and np.isfinite(out["energy"])


def test_multicard_energies_for_uma_and_orb_bundles(tmp_path):
    """MultiCard (tt_atom/batch.py:218-243) detects the family from the bundle: its energies
    equal a calculator's on the same structures, for a UMA bundle and for an Orb bundle (Orb
    energy with its normaliser and ZBL term)."""
    import json

    from tt_atom import MultiCard
    from tt_atom.orb import OrbCalculator
    mols = [configs.tiny_molecule(seed=k) for k in range(3)]
    systems = [(m["pos"], m["Z"]) for m in mols]
    cfg, b = _tiny()
    upath = str(tmp_path / "uma_tiny.npz")
    np.savez(upath, **configs.random_bundle_arrays(cfg, seed=0))
    ocfg = configs.orb_config("orb-tiny")
    ow = configs.orb_random_weights(ocfg, seed=0)
    arrs = {"config": np.frombuffer(json.dumps(ocfg).encode(), dtype=np.uint8)}
    arrs.update({f"w@{k}": v.numpy() for k, v in ow.items()})
    opath = str(tmp_path / "orb_tiny.npz")
    np.savez(opath, **arrs)
    for path, make in ((upath, lambda: TTAtomCalculator(b)),
                       (opath, lambda: OrbCalculator(ow, cfg=ocfg))):
        with MultiCard(path, device_ids=(0,)) as pool:
            en, edges = pool.energies(systems)
        assert edges > 0
        calc = make()
        for e, m in zip(en, mols):
            a = SimpleAtoms(m["Z"], m["pos"])
            a.calc = calc
            assert abs(e - float(a.get_potential_energy())) <= 1e-6 * max(1.0, abs(e)), path


def test_multicardsim_by_model_name_uses_the_bundle_cache(tmp_path):
    """MultiCardSim("uma-s-1", ...) picks each structure's merged bundle from the cache by
    (reduced composition, charge, spin), as the reference's workers do; energies equal a
    calculator on that bundle."""
    from tt_atom import MultiCardSim
    from tt_atom import bundle_cache as BC
    cfg, b = _tiny()
    mols = [configs.tiny_molecule(seed=k) for k in range(2)]
    b.save(BC.bundle_path("uma-s-1", b.task, mols[0]["Z"], 0, 0, cache_dir=tmp_path))
    with MultiCardSim("uma-s-1", device_ids=(0,), task=b.task, cache_dir=str(tmp_path),
                      sim_params=dict(mode="energy")) as sim:
        out = sim.run([dict(pos=m["pos"], Z=m["Z"], charge=0, spin=0) for m in mols])
    assert all(r["ok"] for r in out), [r.get("error") for r in out]
    calc = TTAtomCalculator(b)
    for r, m in zip(out, mols):
        a = SimpleAtoms(m["Z"], m["pos"], info=dict(charge=0, spin=0))
        a.calc = calc
        assert abs(r["energy"] - float(a.get_potential_energy())) <= 1e-6 * max(1.0, abs(r["energy"]))


def test_multicardsim_poisoned_structure_fails_alone(tmp_path):
    """One structure with no edges within the cutoff (two atoms 20 A apart) comes back as
    {ok: False, error, tb} with the calculator's error; the others return the energies a
    calculator gives (tt_atom/batch.py:318-325)."""
    from tt_atom import MultiCardSim
    cfg, b = _tiny()
    path = str(tmp_path / "tiny.npz")
    np.savez(path, **configs.random_bundle_arrays(cfg, seed=0))
    mols = [configs.tiny_molecule(seed=k) for k in range(3)]
    lonely = dict(pos=np.array([[0.0, 0.0, 0.0], [20.0, 0.0, 0.0]], np.float32),
                  Z=np.array([6, 8], np.int64))
    systems = [dict(pos=mols[0]["pos"], Z=mols[0]["Z"]), lonely,
               dict(pos=mols[1]["pos"], Z=mols[1]["Z"]), dict(pos=mols[2]["pos"], Z=mols[2]["Z"])]
    with MultiCardSim(path, device_ids=(0,), sim_params=dict(mode="energy")) as sim:
        out = sim.run(systems)
    assert out[1]["ok"] is False
    assert out[1]["error"].startswith("ValueError: no edges within cutoff")
    assert "Traceback" in out[1]["tb"]
    calc = TTAtomCalculator(b)
    for r, m in zip([out[0], out[2], out[3]], mols):
        assert r["ok"], r.get("error")
        a = SimpleAtoms(m["Z"], m["pos"])
        a.calc = calc
        assert abs(r["energy"] - float(a.get_potential_energy())) <= 1e-6 * max(1.0, abs(r["energy"]))
