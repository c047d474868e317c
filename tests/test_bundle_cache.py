"""Bundle cache layout and the name-based entry points (no GPU: every case here stops before a
calculator is built)."""
import os

import numpy as np
import pytest

import tt_atom
from tt_atom import bundle_cache as BC
from tt_atom.ase_compat import SimpleAtoms


def test_bundle_path_layout_and_invariance(tmp_path):
    p = BC.bundle_path("uma-s-1", "omol", [8, 1, 1], 0, 1, cache_dir=tmp_path)
    assert p.parent == tmp_path
    assert p.name == f"uma-s-1_omol_{BC.composition_hash([1, 8, 1])}_c0_s1.npz"
    assert len(BC.composition_hash([8, 1, 1])) == 12
    # atom order and an integer scaling of the counts give the same bundle
    assert BC.bundle_path("uma-s-1", "omol", [1, 1, 8, 8, 1, 1], 0, 1, cache_dir=tmp_path) == p
    assert BC.bundle_path("uma-s-1", "omat", [8, 1, 1], 0, 1, cache_dir=tmp_path) != p
    assert BC.bundle_path("uma-s-1", "omol", [8, 1, 1], 1, 1, cache_dir=tmp_path) != p
    ck = BC.bundle_path("uma-s-1", "omol", [8, 1, 1], 0, 1, cache_dir=tmp_path,
                        checkpoint=str(tmp_path / "x.pt"))
    assert ck.name.startswith(p.name[:-4] + "_ckpt")
    assert BC.orb_weights_path("orb-v3-direct-omol", tmp_path).name == "direct-omol.npz"
    with pytest.raises(ValueError, match="unknown Orb checkpoint"):
        BC.orb_weights_path("orb-v9", tmp_path)


def test_default_cache_directories(monkeypatch, tmp_path):
    monkeypatch.delenv("TT_ATOM_CACHE", raising=False)
    home = os.path.expanduser("~")
    assert str(BC._uma_dir()) == os.path.join(home, ".cache", "tt_atom", "bundles")
    assert str(BC._orb_dir()) == os.path.join(home, ".cache", "tt_atom", "orb_weights")
    monkeypatch.setenv("TT_ATOM_CACHE", str(tmp_path))
    assert BC._uma_dir() == tmp_path and BC._orb_dir() == tmp_path / "orb_weights"


def test_infer_task_and_name_dispatch_errors(tmp_path):
    mol = SimpleAtoms([8, 1, 1], np.zeros((3, 3)))
    bulk = SimpleAtoms([29], np.zeros((1, 3)), cell=np.eye(3) * 3.6, pbc=True)
    assert BC.infer_task(mol) == "omol" and BC.infer_task(bulk) == "omat"
    with pytest.raises(ValueError, match="needs `atoms`"):
        tt_atom.Calculator(None, "uma-s-1", cache_dir=tmp_path)
    with pytest.raises(RuntimeError, match="no cached uma-s-1 bundle"):
        tt_atom.Calculator(mol, "uma-s-1", cache_dir=tmp_path)
    assert mol.info["charge"] == 0 and mol.info["spin"] == 1     # stamped for calculate
    with pytest.raises(ValueError, match="applies only to UMA"):
        tt_atom.Calculator(mol, "orb-v3-conservative-omol", task="omol", cache_dir=tmp_path)
    with pytest.raises(RuntimeError, match="no cached orb-v3-conservative-omol weights"):
        tt_atom.Calculator(mol, "orb-v3-conservative-omol", cache_dir=tmp_path)
    with pytest.raises(ValueError, match="unknown model"):
        tt_atom.Calculator(mol, "schnet")
