"""The spectral feed-forward (uma-s-1's atomwise block) pinned to the reference's own module
(tests/golden/ref_run_spectral.npz: tt_atom/spectral.py:41-188 ``SpectralAtomwise``, its flat
block-diagonal path and its per-degree path, run on the CPU through ``tests/golden/ttnn_cpu.py``
on seeded node features and random-init weights). The oracle's ``spectral_ff`` must match both;
the GPU engine's spectral blocks are checked against the oracle end to end
(tests/test_gpu_parity.py, tests/test_gpu_headline.py)."""
import pytest
import torch

from oracle import uma as O
from tt_atom import configs

CASES = {"tiny": ("tiny", "blocks.1.atom_wise"), "uma_s1": ("uma-s-1", "blocks.3.atom_wise")}


@pytest.mark.parametrize("fused", ["1", "0"])
@pytest.mark.parametrize("name", list(CASES))
def test_oracle_spectral_ff_matches_reference(fx, name, fused):
    d = fx("ref_run_spectral.npz").d
    shape, prefix = CASES[name]
    cfg = configs.model_config(shape, ff_type="spectral")
    w = configs.random_weights(cfg, seed=0)
    out = O.spectral_ff(torch.from_numpy(d[f"{name}@x"]), w, prefix, 2)
    ref = torch.from_numpy(d[f"{name}@out_fused{fused}"])
    assert (out - ref).abs().max() <= 1e-5 * max(1.0, float(ref.abs().max()))
