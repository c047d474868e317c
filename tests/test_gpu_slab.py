"""The slab-partitioned engine on one GPU (partitions in lock step) equals the unpartitioned
engine on the same cell: energy, forces and virial."""
import numpy as np
import pytest
import torch

from tt_atom import configs
from tt_atom.engine import UMAEngine
from tt_atom.graph import build_graph, csd_embedding
from tt_atom.slab import LockstepGroup, local_graph, plans_for, run_lockstep, slab_order
from tt_atom.weights import WeightBundle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape,nparts", [("tiny", 3), ("uma-s-1", 2)])
def test_slab_lockstep_matches_single(shape, nparts):
    cfg = configs.model_config(shape)
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    s = configs.fcc_alloy(reps=(6, 3, 3), seed=3)          # 21.3 A along x: slabs >= 7.1 A
    perm, ranges = slab_order(s["pos"], s["cell"], nparts)
    pos = torch.from_numpy(s["pos"][perm]).cuda()
    Z = s["Z"][perm]
    eng = UMAEngine(b.weights, cfg, b.tables(), precision="3xtf32")
    se = csd_embedding(b.weights, [0.0], [0.0], cfg["sphere_channels"])
    g = build_graph(pos, Z, cfg["cutoff"], s["cell"], [True] * 3,
                    max_neighbors=cfg["max_neighbors"])
    ref = eng.workspace(g, se)
    ref.pos.copy_(pos)
    eng.run(ref, ref.pos, forces=True, virial=True)
    plans = plans_for(g, ranges)
    wss = []
    for p in plans:
        ws = eng.workspace(local_graph(g, p), se)
        ws.pos.copy_(pos[p.global_ids.cuda()])       # owned atoms, then halo atoms
        wss.append(ws)
    run_lockstep(eng, wss, LockstepGroup(plans))
    E = sum(float(ws.energy[0]) for ws in wss)
    V = sum(ws.virial.double().cpu() for ws in wss)
    F = torch.zeros(g.N, 3, dtype=torch.float64)
    for p, ws in zip(plans, wss):
        F[p.global_ids[:p.n_own].cpu()] = ws.forces[:p.n_own].double().cpu()
    E_ref = float(ref.energy[0])
    assert abs(E - E_ref) <= 1e-5 * abs(E_ref)
    assert (F - ref.forces.double().cpu()).abs().max() <= 1e-4
    vol = abs(np.linalg.det(s["cell"].astype(np.float64)))
    assert (V - ref.virial.double().cpu()).abs().max() / vol <= 1e-5
