"""Relaxation and MD loops on analytic potentials (CPU): FIRE reaches the minimum, NVE
conserves energy, Langevin thermalises to its temperature, masses and units."""
import math

import pytest
import torch

from tt_atom import dynamics as D


def harmonic(k, x0):
    def f(pos):
        d = pos - x0
        return 0.5 * k * (d * d).sum(), -k * d
    return f


def test_fire_reaches_minimum():
    g = torch.Generator().manual_seed(0)
    x0 = torch.randn(20, 3, generator=g, dtype=torch.float64)
    pos = x0 + 0.5 * torch.randn(20, 3, generator=g, dtype=torch.float64)
    res = D.fire(harmonic(3.0, x0), pos, fmax=1e-4, steps=2000)
    assert res["converged"] and res["fmax"] < 1e-4
    assert (pos - x0).abs().max() < 1e-4
    # the step cap holds on the first step
    pos2 = x0 + 10.0
    D.fire(harmonic(3.0, x0), pos2, fmax=1e-9, steps=1)
    assert (pos2 - (x0 + 10.0)).norm() <= 0.2 + 1e-12


def test_nve_conserves_energy():
    g = torch.Generator().manual_seed(1)
    x0 = torch.zeros(50, 3, dtype=torch.float64)
    pos = torch.randn(50, 3, generator=g, dtype=torch.float64) * 0.1
    m = torch.full((50,), 12.0, dtype=torch.float64)
    vel = torch.zeros(50, 3, dtype=torch.float64)
    f = harmonic(10.0, x0)
    E0 = float(f(pos)[0])
    res = D.langevin(f, pos, m, steps=500, dt_fs=0.5, friction_fs=0.0, vel=vel)
    E1 = res["energy"] + D.kinetic_energy(vel, m)
    assert abs(E1 - E0) <= 1e-3 * abs(E0)
    # period of one oscillator in fs: 2 pi sqrt(m / k) in ASE time units
    assert 2 * math.pi * math.sqrt(12.0 / 10.0) / D.FS == pytest.approx(70.07, rel=1e-3)


def test_langevin_thermalises():
    g = torch.Generator().manual_seed(2)
    n = 4000
    pos = torch.zeros(n, 3, dtype=torch.float64)
    m = torch.full((n,), 20.0, dtype=torch.float64)
    res = D.langevin(harmonic(5.0, torch.zeros(n, 3, dtype=torch.float64)), pos, m, steps=400,
                     dt_fs=2.0, temp=500.0, friction_fs=0.05, generator=g)
    assert D.temperature(res["vel"], m) == pytest.approx(500.0, rel=0.05)


def test_masses_and_units():
    m = D.masses_of([1, 6, 8, 26, 79])
    assert m.tolist() == pytest.approx([1.008, 12.011, 15.999, 55.845, 196.97])
    with pytest.raises(ValueError):
        D.masses_of([0])
    assert D.FS == pytest.approx(0.0982269475, rel=1e-9)
    assert D.KB == pytest.approx(8.617333262e-05, rel=1e-9)
