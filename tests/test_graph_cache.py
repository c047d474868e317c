"""Host-side helpers (no GPU): the neighbour-list builder's caches (the image-shift table and
the per-system index tensors are reused for identical inputs and rebuilt when the cell, the
periodic axes, the cutoff or the system offsets change) and the single read-back of results."""
import numpy as np
import torch

from tt_atom import graph as G


def test_image_shift_cache_keys_on_cell_pbc_and_cutoff():
    cell = np.diag([7.1, 7.1, 7.1]).astype(np.float32)
    a = G._device_shifts(cell, [True] * 3, 6.0, "cpu")
    assert G._device_shifts(cell.copy(), [True] * 3, 6.0, "cpu") is a
    assert torch.equal(a, G.image_shifts(cell, [True] * 3, 6.0))
    b = G._device_shifts(cell * 1.01, [True] * 3, 6.0, "cpu")
    assert b is not a and not torch.equal(a, b)
    c = G._device_shifts(cell, [True, True, False], 6.0, "cpu")
    assert c.shape[0] < a.shape[0]
    d = G._device_shifts(cell, [True] * 3, 8.0, "cpu")     # two image layers per axis
    assert d.shape[0] == 125 and a.shape[0] == 27


def test_system_index_cache():
    sid, sp = G._device_sys([0, 3, 7], "cpu")
    assert sid.tolist() == [0, 0, 0, 1, 1, 1, 1] and sp.tolist() == [0, 3, 7]
    assert G._device_sys([0, 3, 7], "cpu")[0] is sid
    sid2, _ = G._device_sys([0, 4, 7], "cpu")
    assert sid2.tolist() == [0, 0, 0, 0, 1, 1, 1]


def test_to_host_returns_float64_copies_in_order():
    """One read-back for several result tensors: shapes and values kept, float64, None kept."""
    from tt_atom.engine import to_host
    a = torch.arange(3, dtype=torch.float32)
    b = torch.arange(6, dtype=torch.float32).reshape(2, 3) / 7
    c = torch.tensor([1.5], dtype=torch.float64)
    x, y, z, w = to_host(a, None, b, c)
    assert y is None and x.dtype == torch.float64 and z.shape == (2, 3)
    assert torch.equal(x, a.double()) and torch.equal(z, b.double()) and torch.equal(w, c)
    assert to_host(None, None) == [None, None]


def test_reduced_composition_and_bundle_reference():
    """The merged-bundle composition key (counts divided by their gcd) and the bundle's embedded
    reference system (``ref@`` entries; None without them)."""
    from tt_atom.weights import WeightBundle, reduced_composition
    assert reduced_composition([1, 1, 8]) == ((1, 2), (8, 1))
    assert reduced_composition([8, 1, 1, 1, 8, 1]) == ((1, 2), (8, 1))     # H4O2 ~ H2O
    assert reduced_composition([6, 1, 1, 1, 1]) != reduced_composition([6, 1, 1])
    cfg = b'{"task": "omol"}'
    arrs = {"config": np.frombuffer(cfg, dtype=np.uint8)}
    assert WeightBundle.from_arrays(arrs).reference is None
    arrs.update({"ref@energy": np.array([-1.5]), "ref@forces": np.zeros((3, 3)),
                 "ref@pos": np.zeros((3, 3)), "ref@atomic_numbers": np.array([8, 1, 1]),
                 "ref@charge": np.array([0.0]), "ref@spin": np.array([1.0])})
    ref = WeightBundle.from_arrays(arrs).reference
    assert ref["energy"] == -1.5 and ref["spin"] == 1.0 and ref["cell"] is None
    assert reduced_composition(ref["atomic_numbers"]) == ((1, 2), (8, 1))
