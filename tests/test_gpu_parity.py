"""End-to-end parity of the CUDA path with the oracle and the reference fixtures.

Tolerances (fp32 mode): energy <= 1e-5 relative, forces <= 1e-4 eV/A max-abs, stress
<= 1e-5 eV/A^3 max-abs; neighbour lists and edge order bit-exact."""
import numpy as np
import pytest
import torch

from oracle import uma as O
from tt_atom import configs
from tt_atom.calculator import TTAtomCalculator
from tt_atom.graph import build_graph, radius_graph
from tt_atom.weights import WeightBundle

pytestmark = pytest.mark.gpu

E_REL, F_ABS, S_ABS = 1e-5, 1e-4, 1e-5


def bundle_from_fixture(g):
    arrs = {"config": g.d["config"]}
    cfg = dict(g.config)
    cfg.setdefault("task", "omat")
    cfg.setdefault("max_neighbors", None)
    import json
    arrs["config"] = np.frombuffer(json.dumps(cfg).encode(), dtype=np.uint8)
    for k in g.d.files:
        if k.startswith("w@") or k.startswith("host@"):
            arrs[k] = g.d[k]
    return WeightBundle.from_arrays(arrs), cfg


PRECISIONS = ["fp32", "3xtf32", "3xf16"]


def engine_eval(bundle, pos, Z, cell=None, pbc=None, stress=False, trace=False, calc=None,
                precision="fp32"):
    calc = calc or TTAtomCalculator(bundle, max_neighbors=bundle.config.get("max_neighbors"),
                                    precision=precision)
    E, Fo, V = calc._evaluate(pos, Z, cell, pbc, [0.0], [0.0], forces=True, stress=stress,
                              trace=trace)
    return calc, float(E[0]), Fo, V


@pytest.mark.parametrize("name", ["ref_run_tiny_molecule.npz", "ref_run_tiny_fcc.npz"])
def test_neighbor_list_bit_exact_vs_reference(fx, name):
    g = fx(name)
    periodic = bool(g.d["in@pbc"])
    pos = g.d["in@pos"]
    ei, sh = radius_graph(pos, g.config["cutoff"], g.d["in@cell"] if periodic else None,
                          [True] * 3 if periodic else None)
    assert torch.equal(ei, g.t("out@edge_index").long())
    assert torch.equal(sh, g.t("out@shift"))


@pytest.mark.parametrize("seed,periodic,cap", [(0, False, None), (1, True, None),
                                               (2, False, 6), (3, True, 12)])
def test_neighbor_list_matches_oracle_random(seed, periodic, cap):
    rng = np.random.default_rng(seed)
    n = 150
    pos = (rng.uniform(0, 9.0, size=(n, 3))).astype(np.float32)
    cell = np.diag([9.0, 9.5, 10.0]).astype(np.float32) if periodic else None
    pbc = [True] * 3 if periodic else None
    ei, sh = radius_graph(pos, 4.5, cell, pbc, max_neighbors=cap)
    ei_o, sh_o = O.neighbor_list(torch.from_numpy(pos), 4.5,
                                 torch.from_numpy(cell) if periodic else None, pbc, cap)
    assert torch.equal(ei, ei_o)
    assert torch.equal(sh, sh_o)


def test_neighbor_list_batched_systems_stay_disjoint():
    sysl = configs.screening_set(count=6, seed=5)
    pos = np.concatenate([s["pos"] for s in sysl])
    Z = np.concatenate([s["Z"] for s in sysl])
    ptr_ = np.cumsum([0] + [len(s["Z"]) for s in sysl])
    g = build_graph(pos, Z, 6.0, sys_ptr=ptr_, max_neighbors=30)
    ei, _, _ = g.reference_order()
    off = 0
    got = []
    for s, (a, b) in zip(sysl, zip(ptr_[:-1], ptr_[1:])):
        e1, _ = O.neighbor_list(torch.from_numpy(s["pos"]), 6.0, max_neighbors=30)
        got.append(e1 + int(a))
    assert torch.equal(ei.cpu(), torch.cat(got, 1))


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("name,periodic", [("ref_golden_tiny.npz", False),
                                           ("ref_golden_bulk.npz", True)])
def test_energy_forces_vs_fairchem_golden(fx, name, periodic, precision):
    g = fx(name)
    b, cfg = bundle_from_fixture(g)
    pos = g.d["in@pos"]
    Z = g.d["in@atomic_numbers"]
    cell = g.d["in@cell"][0] if periodic else None
    pbc = [True] * 3 if periodic else None
    calc, E, Fo, _ = engine_eval(b, pos, Z, cell, pbc, precision=precision)
    E_ref = float(g.d["out@energy"][0])
    assert abs(E - E_ref) <= E_REL * abs(E_ref), (E, E_ref)
    assert (Fo.float() - g.t("out@forces")).abs().max() <= F_ABS


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("name", ["ref_run_tiny_molecule.npz", "ref_run_tiny_fcc.npz"])
def test_energy_forces_stress_vs_reference_cpu_path(fx, name, precision):
    g = fx(name)
    b, cfg = bundle_from_fixture(g)
    periodic = bool(g.d["in@pbc"])
    pos, Z = g.d["in@pos"], g.d["in@Z"]
    cell = g.d["in@cell"] if periodic else None
    pbc = [True] * 3 if periodic else None
    calc, E, Fo, V = engine_eval(b, pos, Z, cell, pbc, stress=periodic, precision=precision)
    E_ref = float(g.d["out@energy"][0])
    assert abs(E - E_ref) <= E_REL * abs(E_ref), (E, E_ref)
    assert (Fo.float() - g.t("out@forces")).abs().max() <= F_ABS
    if periodic:
        vol = abs(np.linalg.det(cell.astype(np.float64)))
        assert (V.float() - g.t("out@virial")).abs().max() / vol <= S_ABS


def _oracle(cfg, w, tables, s, stress):
    pos = torch.from_numpy(s["pos"])
    cell = torch.from_numpy(s["cell"]) if s["pbc"] else None
    pbc = [True] * 3 if s["pbc"] else None
    ei, sh = O.neighbor_list(pos, cfg["cutoff"], cell, pbc, cfg.get("max_neighbors"))
    return O.energy_forces(w, cfg, tables, pos, torch.from_numpy(s["Z"]), ei,
                           sh if s["pbc"] else None, compute_stress=stress)


def _tables(cfg):
    t = configs.lmax2_tables()
    off, coeff = configs.gaussian_basis(cfg)
    return dict(t, gauss_offset=off, gauss_coeff=coeff)


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("shape,sysname,ff", [("tiny", "tiny", "grid"),
                                              ("uma-s-1", "fcc-small", "grid"),
                                              ("tiny", "tiny", "spectral"),
                                              ("uma-s-1", "fcc-small", "spectral")])
def test_configs_vs_oracle(shape, sysname, ff, precision):
    cfg = configs.model_config(shape, ff_type=ff)
    arrs = configs.random_bundle_arrays(cfg, seed=0)
    b = WeightBundle.from_arrays(arrs)
    s = configs.system(sysname)
    calc, E, Fo, V = engine_eval(b, s["pos"], s["Z"], s["cell"], [True] * 3 if s["pbc"] else None,
                                 stress=s["pbc"], precision=precision)
    r = _oracle(cfg, b.weights, _tables(cfg), s, s["pbc"])
    E_ref = float(r["energy"][0])
    assert abs(E - E_ref) <= E_REL * abs(E_ref), (E, E_ref)
    assert (Fo.float() - r["forces"]).abs().max() <= F_ABS
    if s["pbc"]:
        vol = abs(np.linalg.det(s["cell"].astype(np.float64)))
        assert (V.float() - r["virial"]).abs().max() / vol <= S_ABS


def test_batch_equals_single_and_trace_is_bit_exact():
    cfg = configs.model_config("tiny")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    calc = TTAtomCalculator(b)
    sysl = configs.screening_set(count=5, seed=7)
    out = calc.evaluate_batch(sysl)
    for k, s in enumerate(sysl):
        _, E, Fo, _ = engine_eval(b, s["pos"], s["Z"], calc=calc)
        assert abs(out["energy"][k] - E) <= 1e-5 * max(1.0, abs(E))
        assert np.abs(out["forces"][k] - Fo.numpy()).max() <= 1e-5
    s = sysl[0]
    _, E0, F0, _ = engine_eval(b, s["pos"], s["Z"], calc=calc)
    _, E1, F1, _ = engine_eval(b, s["pos"], s["Z"], calc=calc, trace=True)
    _, E2, F2, _ = engine_eval(b, s["pos"], s["Z"], calc=calc, trace=True)
    assert E0 == E1 == E2
    assert torch.equal(F0, F1) and torch.equal(F1, F2)



def test_traced_calculate_with_stress_is_bit_exact():
    """Calculator(trace=True) replays the captured step (virial included) and gives the eager
    results bit for bit, also after the positions move within the same topology."""
    from tt_atom.ase_compat import SimpleAtoms
    cfg = configs.model_config("uma-s-1")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    s = configs.fcc_alloy(reps=(3, 3, 3), seed=2)
    res = {}
    for trace in (False, True):
        calc = TTAtomCalculator(b, trace=trace)
        out = []
        for dx in (0.0, 0.001, 0.0):
            a = SimpleAtoms(s["Z"], s["pos"] + dx, s["cell"], True)
            calc.calculate(a, ("energy", "forces", "stress"))
            out.append((calc.results["energy"], calc.results["forces"].copy(),
                        calc.results["stress"].copy()))
        res[trace] = out
    for (e0, f0, s0), (e1, f1, s1) in zip(res[False], res[True]):
        assert e0 == e1 and np.array_equal(f0, f1) and np.array_equal(s0, s1)


def test_traced_step_survives_a_same_size_topology_change():
    """MD moves atoms across neighbour ranks every step: with the cap the edge count stays the
    same while the edge set changes. The calculator then copies the new topology into the
    workspace's own arrays and replays the captured step instead of capturing again; results
    equal a fresh eager evaluation bit for bit."""
    from tt_atom.ase_compat import SimpleAtoms
    cfg = configs.model_config("uma-s-1")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    s = configs.fcc_alloy(reps=(3, 3, 3), seed=2)
    rng = np.random.default_rng(5)
    calc = TTAtomCalculator(b, trace=True)
    a = SimpleAtoms(s["Z"], s["pos"], s["cell"], True)
    calc.calculate(a, ("energy", "forces", "stress"))
    step, src0 = calc._step, calc._ws.graph.src.clone()
    assert step is not None
    changed = 0
    for k in range(3):
        p = s["pos"] + rng.normal(0.0, 0.15, s["pos"].shape)
        a = SimpleAtoms(s["Z"], p, s["cell"], True)
        calc.calculate(a, ("energy", "forces", "stress"))
        assert calc._step is step                        # no new capture
        changed += int(not torch.equal(calc._ws.graph.src, src0))
        ref = TTAtomCalculator(b, trace=False)
        ref.calculate(SimpleAtoms(s["Z"], p, s["cell"], True), ("energy", "forces", "stress"))
        assert calc.results["energy"] == ref.results["energy"]
        assert np.array_equal(calc.results["forces"], ref.results["forces"])
        assert np.array_equal(calc.results["stress"], ref.results["stress"])
    assert changed > 0                                   # the topology did change


def test_calculator_api_and_errors():
    from tt_atom.ase_compat import SimpleAtoms
    cfg = configs.model_config("tiny")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    calc = TTAtomCalculator(b)
    s = configs.tiny_molecule()
    atoms = SimpleAtoms(s["Z"], s["pos"])
    atoms.calc = calc
    e = atoms.get_potential_energy()
    f = atoms.get_forces()
    assert np.isfinite(e) and f.shape == (24, 3)
    assert set(calc.results) >= {"energy", "free_energy", "energies", "forces"}
    sparse = SimpleAtoms([1, 1], [[0, 0, 0], [0, 0, 50.0]])
    sparse.calc = calc
    with pytest.raises(ValueError, match="no edges"):
        sparse.get_potential_energy()
    with pytest.raises(ValueError, match="task_name"):
        TTAtomCalculator(b, task_name="omol")
    # a bundle carrying its merge reference: batches must share its reduced composition and its
    # (charge, spin) (tt_atom/calculator.py:193-217)
    arrs = dict(configs.random_bundle_arrays(cfg, seed=0))
    m = configs.tiny_molecule()
    arrs.update({"ref@energy": np.array([0.0]), "ref@forces": np.zeros((24, 3)),
                 "ref@pos": m["pos"], "ref@atomic_numbers": np.asarray(m["Z"]),
                 "ref@charge": np.array([0.0]), "ref@spin": np.array([0.0])})
    calc_r = TTAtomCalculator(WeightBundle.from_arrays(arrs))
    out = calc_r.evaluate_batch([dict(pos=m["pos"], Z=m["Z"]), dict(pos=m["pos"] + 0.01, Z=m["Z"])])
    assert out["energy"].shape == (2,)
    with pytest.raises(ValueError, match="different reduced composition"):
        calc_r.evaluate_batch([dict(pos=m["pos"], Z=m["Z"]), dict(pos=m["pos"][:23], Z=m["Z"][:23])])
    with pytest.raises(ValueError, match=r"\(charge, spin\)"):
        calc_r.evaluate_batch([dict(pos=m["pos"], Z=m["Z"], charge=1.0)])


def test_calculator_by_name_loads_the_cached_bundle(tmp_path):
    """`tt_atom.Calculator(atoms, "uma-s-1", ...)` finds the merged bundle of the atoms'
    (reduced composition, charge, spin, task) in the cache layout and gives the same results as
    a calculator built on that bundle directly."""
    import tt_atom
    from tt_atom import bundle_cache as BC
    from tt_atom.ase_compat import SimpleAtoms
    cfg = configs.model_config("tiny")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    m = configs.tiny_molecule()
    b.save(BC.bundle_path("uma-s-1", b.task, m["Z"], 0, 1, cache_dir=tmp_path))
    a = SimpleAtoms(m["Z"], m["pos"])
    calc = tt_atom.Calculator(a, "uma-s-1", task=b.task, cache_dir=tmp_path)
    assert a.calc is calc and a.info["spin"] == 1
    ref = SimpleAtoms(m["Z"], m["pos"], info=dict(charge=0, spin=1))
    ref.calc = TTAtomCalculator(b)
    assert a.get_potential_energy() == ref.get_potential_energy()
    assert np.array_equal(a.get_forces(), ref.get_forces())
