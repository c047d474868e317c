"""A bounded device-side wait that expired must surface as an exception, never as results.

The tensor-core GEMM bounds every mbarrier wait; on expiry it records a code in a device flag and
its later CTAs return at entry, so the outputs of that step are incomplete. Every host read-back
(``engine.to_host``) reads the flag back with the results (``atom_device_error_take``) and the
end of the GPU-resident relax / MD loops reads it (``atom_device_error``); both raise. The CPU test fakes the library's answer; the GPU test makes the
GEMM's own bounded wait run out on a barrier that nothing arrives on (a short budget, no fault)
and checks that the calculator raises once and then recovers."""
import ctypes

import numpy as np
import pytest
import torch

from tt_atom import _lib
from tt_atom import engine as engine_mod


class _FakeLib:
    """Stands in for libatomb200.so: the error code is ``code`` once, then 0 (both the
    synchronous read and the stream-ordered take into a buffer)."""

    def __init__(self, code):
        self.code = code

    def atom_device_error(self, code_ptr, stream):
        ctypes.cast(code_ptr, ctypes.POINTER(ctypes.c_int))[0] = self.code
        self.code = 0
        return 0

    def atom_device_error_take(self, code_ptr, stream):
        return self.atom_device_error(code_ptr, stream)

    def atom_last_error(self, buf, n):
        return 0


def test_expired_wait_code_raises_on_readback(monkeypatch):
    fake = _FakeLib(4)
    monkeypatch.setattr(_lib, "_lib", fake)
    monkeypatch.setattr(_lib, "stream_ptr", lambda stream=None: None)
    t = torch.ones(3)
    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))
    with pytest.raises(RuntimeError, match="bounded device-side wait"):
        engine_mod.to_host(t)
    # the flag was cleared by the read: the next read-back returns the values
    (out,) = engine_mod.to_host(t)
    assert out.dtype == torch.float64 and torch.equal(out, t.double())


def test_clean_code_returns_results(monkeypatch):
    monkeypatch.setattr(_lib, "_lib", _FakeLib(0))
    monkeypatch.setattr(_lib, "stream_ptr", lambda stream=None: None)
    monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))
    a, b = engine_mod.to_host(torch.arange(4.0), None)
    assert b is None and a.tolist() == [0.0, 1.0, 2.0, 3.0]


@pytest.mark.gpu
def test_expired_wait_makes_calculator_raise_then_recover():
    from tt_atom import configs
    from tt_atom.ase_compat import SimpleAtoms
    from tt_atom.calculator import TTAtomCalculator
    from tt_atom.weights import WeightBundle
    cfg = configs.model_config("tiny")
    calc = TTAtomCalculator(WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0)),
                            precision="3xtf32")
    s = configs.system("tiny")
    atoms = SimpleAtoms(s["Z"], s["pos"])
    calc.calculate(atoms)
    e0, f0 = calc.results["energy"], calc.results["forces"].copy()
    s_ptr = _lib.stream_ptr()
    # ~1 ms of SM clock: the wait gives up, records its code and the kernel returns
    _lib.call("atom_wait_selftest", 2_000_000, s_ptr)
    with pytest.raises(RuntimeError, match="bounded device-side wait"):
        calc.calculate(atoms)
    calc.calculate(atoms)
    assert calc.results["energy"] == e0
    assert np.array_equal(calc.results["forces"], f0)
    code = ctypes.c_int(-1)
    _lib.call("atom_device_error", ctypes.byref(code), s_ptr)
    assert code.value == 0


@pytest.mark.gpu
def test_expired_ring_wait_is_reported_and_cleared():
    """The streamed edge kernels' bounded wait (a barrier whose bytes never arrive) gives up,
    records ATOM_EDGE_WAIT_CODE, and the context stays usable."""
    s_ptr = _lib.stream_ptr()
    code = ctypes.c_int(-1)
    _lib.call("atom_device_error", ctypes.byref(code), s_ptr)
    _lib.call("atom_ring_wait_selftest", 2_000_000, s_ptr)
    _lib.call("atom_device_error", ctypes.byref(code), s_ptr)
    assert code.value == 8
    _lib.call("atom_device_error", ctypes.byref(code), s_ptr)
    assert code.value == 0
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum()) == 8.0


def test_ring_wait_selftest_rejects_bad_budget():
    with pytest.raises(_lib.AtomError):
        _lib.call("atom_ring_wait_selftest", 0, None)
