"""Receiver-chunked execution (edge stages over contiguous receiver chunks, recomputed in the
reverse pass) equals the unchunked engine on the same graph: energy, forces, virial."""
import numpy as np
import pytest
import torch

from tt_atom import configs
from tt_atom.engine import UMAEngine
from tt_atom.graph import build_graph, csd_embedding
from tt_atom.weights import WeightBundle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape,ff,nchunks", [("tiny", "grid", 7), ("uma-s-1", "grid", 3),
                                               ("uma-s-1", "spectral", 4), ("tiny", "grid", 1)])
def test_chunked_matches_unchunked(shape, ff, nchunks):
    cfg = configs.model_config(shape, ff_type=ff)
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    s = configs.fcc_alloy(reps=(4, 3, 3), seed=5)
    pos = torch.from_numpy(s["pos"]).cuda()
    eng = UMAEngine(b.weights, cfg, b.tables(), precision="3xtf32")
    se = csd_embedding(b.weights, [0.0], [0.0], cfg["sphere_channels"])
    g = build_graph(pos, s["Z"], cfg["cutoff"], s["cell"], [True] * 3,
                    max_neighbors=cfg["max_neighbors"])
    ref = eng.workspace(g, se)
    ref.pos.copy_(pos)
    eng.run(ref, ref.pos, forces=True, virial=True)
    max_in = int((g.recv_ptr[1:] - g.recv_ptr[:-1]).max())
    ws = eng.workspace(g, se, chunk_edges=-(-g.E // nchunks) + max_in)
    assert len(ws.chunks) >= min(nchunks, 2) or nchunks == 1
    assert sum(ch.e1 - ch.e0 for ch in ws.chunks) == g.E
    ws.pos.copy_(pos)
    for _ in range(2):            # twice: chunk buffers are reused, adjoints re-zeroed
        eng.run(ws, ws.pos, forces=True, virial=True)
    E_ref, E = float(ref.energy[0]), float(ws.energy[0])
    assert abs(E - E_ref) <= 1e-6 * abs(E_ref)
    assert (ws.forces - ref.forces).abs().max().item() <= 1e-5
    vol = abs(np.linalg.det(s["cell"].astype(np.float64)))
    assert (ws.virial - ref.virial).abs().max().item() / vol <= 1e-6
    assert ws.nbytes() < ref.nbytes()


def test_workspace_size_estimate_and_chunk_choice():
    cfg = configs.model_config("uma-s-1")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    s = configs.fcc_alloy(reps=(4, 3, 3), seed=5)
    eng = UMAEngine(b.weights, cfg, b.tables(), precision="3xtf32")
    se = csd_embedding(b.weights, [0.0], [0.0], cfg["sphere_channels"])
    g = build_graph(torch.from_numpy(s["pos"]).cuda(), s["Z"], cfg["cutoff"], s["cell"],
                    [True] * 3, max_neighbors=cfg["max_neighbors"])
    for k in (None, 2000):
        ws = eng.workspace(g, se, chunk_edges=k)
        est = eng.workspace_bytes(g.N, g.E, chunk_edges=k)
        assert 0.75 * ws.nbytes() <= est <= 1.25 * ws.nbytes()
        del ws
    full = eng.workspace_bytes(g.N, g.E)
    assert eng.choose_chunk_edges(g, budget_bytes=2 * full) is None
    # halfway between the chunked workspace's fixed part and one chunk of all edges
    budget = 0.5 * (eng.workspace_bytes(g.N, g.E, chunk_edges=0)
                    + eng.workspace_bytes(g.N, g.E, chunk_edges=g.E))
    k = eng.choose_chunk_edges(g, budget_bytes=budget)
    assert k is not None and 0 < k < g.E
    assert eng.workspace_bytes(g.N, g.E, chunk_edges=k) <= budget
    with pytest.raises(MemoryError):
        eng.choose_chunk_edges(g, budget_bytes=1e3)


def test_calculator_with_chunks_matches_default():
    from tt_atom.calculator import TTAtomCalculator
    cfg = configs.model_config("uma-s-1")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    s = configs.fcc_alloy(reps=(4, 3, 3), seed=5)
    args = (s["pos"], s["Z"], s["cell"], [True] * 3, [0.0], [0.0])
    E0, F0, V0 = TTAtomCalculator(b)._evaluate(*args, forces=True, stress=True)
    c = TTAtomCalculator(b, chunk_edges=1500)
    E1, F1, V1 = c._evaluate(*args, forces=True, stress=True)
    assert c._ws.chunks is not None and len(c._ws.chunks) > 1
    assert abs(float(E1[0] - E0[0])) <= 1e-6 * abs(float(E0[0]))
    assert (F1 - F0).abs().max().item() <= 1e-5
    assert (V1 - V0).abs().max().item() <= 1e-4
