"""The gate fused into the so2_2 GEMM (``atom_gemm_gated``: the tensor-core kernel forms the
gated operand from the so2_1 output while converting A) against the standalone gate kernel
followed by the GEMM: the same results bit for bit, for both tensor-core precisions, in a full
energy / force / stress step and at the kernel level (ragged row counts)."""
import ctypes

import numpy as np
import pytest
import torch

from tt_atom import _lib as L
from tt_atom import configs
from tt_atom.calculator import TTAtomCalculator
from tt_atom.weights import WeightBundle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("precision", ["3xtf32", "3xf16"])
def test_fused_gate_step_is_bit_identical(precision):
    cfg = configs.model_config("uma-s-1")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    s = configs.fcc_alloy(reps=(3, 3, 3), seed=2)
    out = {}
    for fused in (True, False):
        calc = TTAtomCalculator(b, precision=precision)
        calc.engine.fuse_gate = fused
        E, F, V = calc._evaluate(s["pos"], s["Z"], s["cell"], [True] * 3, [0.0], [0.0],
                                 forces=True, stress=True)
        out[fused] = (E, F, V)
    for a, c in zip(out[True], out[False]):
        assert torch.equal(a, c)


@pytest.mark.parametrize("M", [1, 130, 1000])
def test_gemm_gated_kernel_matches_gate_then_gemm(M):
    from tt_atom.engine import UMAEngine
    cfg = configs.model_config("uma-s-1")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    eng = UMAEngine(b.weights, cfg, b.tables(), device="cuda", precision="3xtf32")
    H, C = eng.H, eng.C
    g = torch.Generator(device="cuda").manual_seed(M)
    Y = torch.randn(M, 11 * H, device="cuda", generator=g) * 3.0
    blk = eng.blocks[1]
    s = L.stream_ptr()
    fused = torch.full((M, 9 * C), float("nan"), device="cuda")
    eng._scratch = torch.empty(1 << 22, device="cuda")
    L.call("atom_gemm_gated", Y.data_ptr(), 11 * H, M, blk["so2_2g"].struct, H,
           fused.data_ptr(), 9 * C, 2, eng._scratch.data_ptr(), eng._scratch.numel(), s)
    Gt = torch.empty(M, 9 * H, device="cuda")
    L.call("atom_gate_fwd", Y.data_ptr(), M, H, Gt.data_ptr(), s)
    ref = torch.empty(M, 9 * C, device="cuda")
    eng._gemm(Gt, 9 * H, M, blk["so2_2"], ref, 9 * C, stream=s)
    torch.cuda.synchronize()
    assert torch.equal(fused, ref)


def test_gemm_gated_rejects_what_it_cannot_do():
    cfg = configs.model_config("uma-s-1")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    from tt_atom.engine import UMAEngine
    eng = UMAEngine(b.weights, cfg, b.tables(), device="cuda", precision="fp32")
    H = eng.H
    Y = torch.zeros(4, 11 * H, device="cuda")
    out = torch.zeros(4, 9 * eng.C, device="cuda")
    rc = L.lib().atom_gemm_gated(Y.data_ptr(), 11 * H, 4, eng.blocks[0]["so2_2g"].struct, H,
                                 out.data_ptr(), 9 * eng.C, 0, None, 0, L.stream_ptr())
    assert rc == L.ATOM_ERR_UNSUPPORTED
    # groups addressing the gating columns are refused
    rc = L.lib().atom_gemm_gated(Y.data_ptr(), 11 * H, 4, eng.blocks[0]["so2_2"].struct, H,
                                 out.data_ptr(), 9 * eng.C, 2, None, 0, L.stream_ptr())
    assert rc == 1
