"""Geometry relaxation (FIRE) and Langevin / NVE molecular dynamics with the whole state on the
GPU.

The reference runs ASE's optimiser and integrator around its calculator
(tt_atom/simulate.py:15-74: ``FIRE`` and ``Langevin``). Here the loops are plain tensor updates
on the device around a force callback, so a run never copies positions or forces to the host
except for the scalars a stopping test needs; with the UMA calculator the force call rebuilds
the neighbour list on the GPU and replays the captured CUDA graph of the step while the edge
set is unchanged (re-capturing when it changes).

Units are ASE's: eV, Angstrom, atomic mass units; times in femtoseconds at the interface and in
ASE's internal unit (Angstrom sqrt(amu / eV) = 10.1805 fs) inside.

* ``fire``: FIRE of Bitzek et al., Phys. Rev. Lett. 97, 170201 (2006), with ASE's default
  parameters and conventions (unit masses, a step-length cap ``maxstep`` on the whole
  displacement vector, convergence when the largest per-atom force is below ``fmax``, checked
  before every step).
* ``langevin``: BAOAB splitting (Leimkuhler & Matthews, Appl. Math. Res. Express 2013) with
  friction ``friction`` (1/fs); ``friction = 0`` is velocity Verlet (NVE). The random kicks come
  from a seeded torch generator on the device, so trajectories are reproducible for a seed but
  are not ASE's (ASE's Langevin draws from numpy's global generator with another splitting).
"""
from __future__ import annotations

import math

import torch

_E, _AMU = 1.602176634e-19, 1.66053906660e-27             # C, kg (CODATA 2018)
FS = 1e-15 * math.sqrt(_E / _AMU) / 1e-10                    # one fs in Angstrom sqrt(amu/eV)
KB = 1.380649e-23 / _E                                       # Boltzmann constant, eV / K

# Standard atomic weights (IUPAC, conventional values), Z = 1 .. 86; index 0 unused.
MASSES = [0.0,
          1.008, 4.0026, 6.94, 9.0122, 10.81, 12.011, 14.007, 15.999, 18.998, 20.180,
          22.990, 24.305, 26.982, 28.085, 30.974, 32.06, 35.45, 39.948, 39.098, 40.078,
          44.956, 47.867, 50.942, 51.996, 54.938, 55.845, 58.933, 58.693, 63.546, 65.38,
          69.723, 72.630, 74.922, 78.971, 79.904, 83.798, 85.468, 87.62, 88.906, 91.224,
          92.906, 95.95, 97.0, 101.07, 102.91, 106.42, 107.87, 112.41, 114.82, 118.71,
          121.76, 127.60, 126.90, 131.29, 132.91, 137.33, 138.91, 140.12, 140.91, 144.24,
          145.0, 150.36, 151.96, 157.25, 158.93, 162.50, 164.93, 167.26, 168.93, 173.05,
          174.97, 178.49, 180.95, 183.84, 186.21, 190.23, 192.22, 195.08, 196.97, 200.59,
          204.38, 207.2, 208.98, 209.0, 210.0, 222.0]


def masses_of(Z, device=None, dtype=torch.float64):
    Z = torch.as_tensor(Z, dtype=torch.long)
    if int(Z.max()) >= len(MASSES) or int(Z.min()) < 1:
        raise ValueError("atomic masses are tabulated for Z = 1 .. 86; pass masses explicitly")
    return torch.tensor(MASSES, dtype=dtype)[Z].to(device)


def fire(force_fn, pos, fmax=0.05, steps=200, dt=0.1, maxstep=0.2, dtmax=1.0, nmin=5,
         finc=1.1, fdec=0.5, astart=0.1, fa=0.99, callback=None):
    """Relax ``pos`` [N, 3] (a tensor on any device, updated in place) with FIRE.

    ``force_fn(pos) -> (energy scalar tensor, forces [N, 3])``. Returns
    ``dict(energy, forces, fmax, nsteps, converged)`` of the final state."""
    v = torch.zeros_like(pos)
    a, n_pos, n = astart, 0, 0
    E, F = force_fn(pos)
    F = F.to(pos.dtype)
    while True:
        fm = float(F.norm(dim=1).max()) if F.numel() else 0.0
        if fm < fmax or n >= steps:
            break
        if n > 0:
            vf = float((F * v).sum())
            if vf > 0.0:
                v.mul_(1.0 - a).add_(a * F / F.norm() * v.norm())
                if n_pos > nmin:
                    dt = min(dt * finc, dtmax)
                    a *= fa
                n_pos += 1
            else:
                v.zero_()
                a = astart
                dt *= fdec
                n_pos = 0
        v.add_(dt * F)
        dr = dt * v
        norm = float(dr.norm())
        if norm > maxstep:
            dr.mul_(maxstep / norm)
        pos.add_(dr)
        n += 1
        E, F = force_fn(pos)
        F = F.to(pos.dtype)
        if callback is not None:
            callback(n, E, F)
    return dict(energy=float(E), forces=F, fmax=fm, nsteps=n, converged=fm < fmax)


def maxwell_boltzmann(masses, temp, generator=None):
    """Velocities [N, 3] (ASE units) drawn at temperature ``temp`` (K)."""
    sd = torch.sqrt(KB * temp / masses).unsqueeze(1)
    return sd * torch.randn(masses.shape[0], 3, dtype=masses.dtype, device=masses.device,
                            generator=generator)


def langevin(force_fn, pos, masses, steps, dt_fs=1.0, temp=300.0, friction_fs=0.01,
             vel=None, generator=None, callback=None):
    """``steps`` BAOAB steps of Langevin dynamics (NVE velocity Verlet for ``friction_fs = 0``)
    on ``pos`` [N, 3] and ``vel`` (updated in place; drawn at ``temp`` when None).

    Returns ``dict(energy, forces, vel, nsteps)`` of the final state."""
    dt = dt_fs * FS
    m = masses.to(pos.dtype).unsqueeze(1)
    if vel is None:
        vel = maxwell_boltzmann(masses.to(pos.dtype), temp, generator)
    c1 = math.exp(-friction_fs / FS * dt)
    c2 = math.sqrt(max(0.0, 1.0 - c1 * c1))
    sd = torch.sqrt(KB * temp / m)
    E, F = force_fn(pos)
    F = F.to(pos.dtype)
    for n in range(1, steps + 1):
        vel.add_(0.5 * dt * F / m)                       # B
        pos.add_(0.5 * dt * vel)                         # A
        if friction_fs > 0.0:                            # O
            noise = torch.randn(vel.shape, dtype=vel.dtype, device=vel.device,
                                generator=generator)
            vel.mul_(c1).add_(c2 * sd * noise)
        pos.add_(0.5 * dt * vel)                         # A
        E, F = force_fn(pos)
        F = F.to(pos.dtype)
        vel.add_(0.5 * dt * F / m)                       # B
        if callback is not None:
            callback(n, E, F, vel)
    return dict(energy=float(E), forces=F, vel=vel, nsteps=steps)


def kinetic_energy(vel, masses):
    return 0.5 * float((masses.to(vel.dtype).unsqueeze(1) * vel * vel).sum())


def temperature(vel, masses):
    return 2.0 * kinetic_energy(vel, masses) / (3.0 * vel.shape[0] * KB)
