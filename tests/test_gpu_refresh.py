"""The device-resident neighbour-list refresh (atom_neighbor_refresh + sender CSR + species,
``graph.TopologyRefresh``) and the traced calculator path built on it, which rebuilds the list
inside the captured step: the refreshed arrays equal a fresh ``build_graph`` bit for bit; a new
edge count or a candidate overflow leaves the arrays untouched and says so; traced results equal
eager ones through same-size topology changes and through size changes (host fallback)."""
import dataclasses

import numpy as np
import pytest
import torch

from tt_atom import configs
from tt_atom.ase_compat import SimpleAtoms
from tt_atom.calculator import TTAtomCalculator
from tt_atom.graph import TopologyRefresh, build_graph
from tt_atom.weights import WeightBundle

pytestmark = pytest.mark.gpu

ARRAYS = ("src", "tgt", "img", "recv_ptr", "send_ptr", "send_eid", "zs", "zt")


def _own_copy(g):
    return dataclasses.replace(g, **{k: getattr(g, k).clone() for k in ARRAYS})


@pytest.mark.parametrize("periodic", [True, False])
def test_refresh_equals_a_fresh_build(periodic):
    rng = np.random.default_rng(3)
    if periodic:
        s = configs.fcc_alloy(reps=(10, 10, 5), seed=1)
        cell, pbc, cap = s["cell"], [True] * 3, 30
    else:
        s = configs.screening_set(count=40)[-1]          # one molecule, cap binding
        cell, pbc, cap = None, None, 30
    g0 = build_graph(s["pos"], s["Z"], 6.0, cell, pbc, max_neighbors=cap)
    mine = _own_copy(g0)
    ref = TopologyRefresh(mine)
    same = 0
    for k in range(4):
        p = (s["pos"] + rng.normal(0.0, 0.05, s["pos"].shape)).astype(np.float32)
        g1 = build_graph(p, s["Z"], 6.0, cell, pbc, max_neighbors=cap)
        before = {k2: getattr(mine, k2).clone() for k2 in ARRAYS}
        ref.launch(torch.from_numpy(p).cuda())
        torch.cuda.synchronize()
        st = ref.status.cpu().tolist()
        if g1.E == mine.E:
            assert st[0] == TopologyRefresh.OK and st[1] == g1.E
            for k2 in ARRAYS:
                assert torch.equal(getattr(mine, k2), getattr(g1, k2)), k2
            same += 1
        else:
            assert st[0] == TopologyRefresh.SIZE_CHANGED and st[1] == g1.E
            for k2 in ("src", "tgt", "img", "recv_ptr"):
                assert torch.equal(getattr(mine, k2), before[k2]), k2
    assert same >= 1


def test_refresh_reports_candidate_overflow_and_keeps_arrays():
    s = configs.fcc_alloy(reps=(4, 4, 4), seed=1)
    g0 = build_graph(s["pos"], s["Z"], 6.0, s["cell"], [True] * 3, max_neighbors=30)
    mine = _own_copy(g0)
    mine.max_cand = 8                     # fcc has 78 candidates within 6 A
    ref = TopologyRefresh(mine, headroom=0)
    src = mine.src.clone()
    ref.launch(torch.from_numpy(s["pos"]).cuda())
    torch.cuda.synchronize()
    st = ref.status.cpu().tolist()
    assert st[0] == TopologyRefresh.OVERFLOW and st[2] >= 78
    assert torch.equal(mine.src, src)


def test_traced_calculator_refreshes_on_the_device_and_falls_back():
    cfg = configs.model_config("uma-s-1")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    s = configs.fcc_alloy(reps=(3, 3, 3), seed=2)
    rng = np.random.default_rng(11)
    traced = TTAtomCalculator(b, trace=True)
    eager = TTAtomCalculator(b, trace=False)
    used_fast = 0
    for k in range(5):
        p = s["pos"] + rng.normal(0.0, 0.1, s["pos"].shape)
        for c in (traced, eager):
            c.calculate(SimpleAtoms(s["Z"], p, s["cell"], True), ("energy", "forces", "stress"))
        used_fast += int(getattr(traced, "_full_step", None) is not None)
        assert traced.results["energy"] == eager.results["energy"]
        assert np.array_equal(traced.results["forces"], eager.results["forces"])
        assert np.array_equal(traced.results["stress"], eager.results["stress"])
    assert used_fast >= 3
    # an uncapped molecule whose edge count changes: the traced path falls back and stays exact
    m = configs.tiny_molecule(seed=0)
    traced = TTAtomCalculator(b, trace=True, max_neighbors=None)
    eager = TTAtomCalculator(b, trace=False, max_neighbors=None)
    for scale in (1.0, 1.0, 1.15, 1.15, 0.9):
        p = m["pos"] * scale
        for c in (traced, eager):
            c.calculate(SimpleAtoms(m["Z"], p), ("energy", "forces"))
        assert traced.results["energy"] == eager.results["energy"]
        assert np.array_equal(traced.results["forces"], eager.results["forces"])


def _random_cell(rng, n, skew):
    a = np.diag(rng.uniform(5.0, 14.0, 3))
    if skew:
        a[1, 0], a[2, 0], a[2, 1] = rng.uniform(-2.5, 2.5, 3)
    frac = rng.uniform(-0.3, 1.3, (n, 3))         # atoms outside the cell too
    return (frac @ a).astype(np.float32), a.astype(np.float32)


@pytest.mark.parametrize("seed", range(6))
def test_cell_list_equals_all_pairs(seed):
    """The cell-list candidates give the all-pairs edge list bit for bit: orthogonal and
    triclinic cells, cells narrower than the cutoff (several images per axis), atoms outside
    the cell, with and without the cap."""
    rng = np.random.default_rng(seed)
    n = int(rng.integers(20, 400))
    pos, cell = _random_cell(rng, n, skew=seed % 2 == 1)
    Z = np.ones(n, np.int64)
    for cap in (None, 12):
        a = build_graph(pos, Z, 6.0, cell, [True] * 3, max_neighbors=cap, use_cells=True)
        b = build_graph(pos, Z, 6.0, cell, [True] * 3, max_neighbors=cap, use_cells=False)
        assert a.cell_grid is not None and b.cell_grid is None
        assert a.E == b.E
        for k in ("src", "tgt", "img", "recv_ptr"):
            assert torch.equal(getattr(a, k), getattr(b, k)), (seed, cap, k)


@pytest.mark.parametrize("name", ["fcc2000", "sio2", "fe65k"])
def test_cell_list_on_the_benchmark_cells(name):
    if name == "fcc2000":
        s, cap = configs.fcc_alloy(reps=(10, 10, 5), seed=1), 30
    elif name == "sio2":
        s, cap = configs.amorphous_sio2(), 20
    else:
        s, cap = configs.bcc_iron(reps=(12, 12, 12)), 30
    a = build_graph(s["pos"], s["Z"], 6.0, s["cell"], [True] * 3, max_neighbors=cap)
    b = build_graph(s["pos"], s["Z"], 6.0, s["cell"], [True] * 3, max_neighbors=cap,
                    use_cells=False)
    assert a.E == b.E == cap * len(s["Z"])
    for k in ("src", "tgt", "img", "recv_ptr", "send_ptr", "send_eid"):
        assert torch.equal(getattr(a, k), getattr(b, k)), k


def test_traced_orb_calculator_refreshes_on_the_device():
    from tt_atom.orb import OrbCalculator
    cfg = configs.orb_config("orb-v3")
    w = configs.orb_random_weights(cfg, seed=0)
    s = configs.amorphous_sio2(n_si=40, n_o=80, seed=2)
    rng = np.random.default_rng(4)
    traced = OrbCalculator(w, cfg=cfg, trace=True)
    eager = OrbCalculator(w, cfg=cfg, trace=False)
    used = 0
    for k in range(4):
        p = s["pos"] + rng.normal(0.0, 0.05, s["pos"].shape)
        for c in (traced, eager):
            c.calculate(SimpleAtoms(s["Z"], p, s["cell"], True), ("energy", "forces", "stress"))
        used += int(getattr(traced, "_full_step", None) is not None)
        assert traced.results["energy"] == eager.results["energy"]
        assert np.array_equal(traced.results["forces"], eager.results["forces"])
        assert np.array_equal(traced.results["stress"], eager.results["stress"])
    assert used >= 2


def test_traced_orb_calculator_falls_back_when_the_edge_count_changes():
    from tt_atom.orb import OrbCalculator
    cfg = configs.orb_config("orb-tiny")
    w = configs.orb_random_weights(cfg, seed=0)
    m = configs.tiny_molecule(seed=0)
    traced = OrbCalculator(w, cfg=cfg, trace=True, max_num_neighbors=None)
    eager = OrbCalculator(w, cfg=cfg, trace=False, max_num_neighbors=None)
    for scale in (1.0, 1.0, 1.2, 1.2, 0.9):
        for c in (traced, eager):
            c.calculate(SimpleAtoms(m["Z"], m["pos"] * scale), ("energy", "forces"))
        assert traced.results["energy"] == eager.results["energy"]
        assert np.array_equal(traced.results["forces"], eager.results["forces"])
