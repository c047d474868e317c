"""Relax / MD loops shared by single-structure use and ``MultiCardSim`` workers
(the reference's tt_atom/simulate.py:15-74: ``relax_atoms`` and ``md_atoms``, same signatures
and result keys).

With ASE installed and ``native=False`` they run ASE's FIRE optimiser and Langevin integrator
around the calculator, as the reference does. Otherwise (ASE absent, or ``native=True``) they
run the GPU-resident loops of ``tt_atom.dynamics``: positions, velocities and forces stay on
the device, each force call rebuilds the neighbour list on the GPU (periodic positions are
wrapped into the cell for it) and replays the captured CUDA graph of the step while the edge
set is unchanged.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib as _L
from . import dynamics as D
from .ase_compat import HAVE_ASE


def _native_forces(atoms):
    """(force_fn, pos) for the atoms' tt_atom calculator (UMA or Orb): force_fn(pos) returns
    the energy and forces [N, 3] that ``calculate`` reports, as device tensors."""
    calc = atoms.calc
    if calc is None or not hasattr(calc, "_evaluate"):
        raise RuntimeError("the native loops need a tt_atom calculator attached to the atoms")
    dev = calc.device
    Z = np.asarray(atoms.get_atomic_numbers(), dtype=np.int64)
    pbc = np.asarray(atoms.get_pbc(), dtype=bool)
    periodic = bool(pbc.any())
    cell = np.asarray(atoms.get_cell(), dtype=np.float32) if periodic else None
    charge = float(atoms.info.get("charge", 0.0))
    spin = float(atoms.info.get("spin", 0.0))
    pos = torch.tensor(np.asarray(atoms.get_positions()), dtype=torch.float64, device=dev)
    if periodic:
        cell_t = torch.tensor(cell, dtype=torch.float64, device=dev)
        inv = torch.linalg.inv(cell_t)
        wrap_mask = torch.tensor(pbc, device=dev)
    if hasattr(calc, "_device_energy_forces"):          # Orb: its own normaliser and ZBL term
        def orb_force_fn(p):
            q = p
            if periodic:
                frac = p @ inv
                frac = torch.where(wrap_mask, frac - torch.floor(frac), frac)
                q = frac @ cell_t
            return calc._device_energy_forces(q.float(), Z, cell, pbc if periodic else None,
                                              charge, spin)
        return orb_force_fn, pos
    ref = 0.0
    if getattr(calc, "elem_refs", None) is not None:
        ref = float(calc.elem_refs[torch.as_tensor(Z)].sum())
    scale, mean = float(calc.scale_rmsd), float(calc.scale_mean)

    def force_fn(p):
        q = p
        if periodic:
            frac = p @ inv
            frac = torch.where(wrap_mask, frac - torch.floor(frac), frac)
            q = frac @ cell_t
        E, F, _ = calc._evaluate(q.float(), Z, cell, pbc if periodic else None, [charge], [spin],
                                 forces=True, stress=False, trace=True, device_out=True)
        return scale * E[0].double() + mean + ref, scale * F.double()
    return force_fn, pos


def relax_atoms(atoms, *, fmax=0.05, steps=200, logfile=None, native=None):
    """FIRE relaxation in place; returns dict(energy, forces, fmax, nsteps, converged)."""
    if native is None:
        native = not HAVE_ASE
    if not native:
        from ase.optimize import FIRE
        opt = FIRE(atoms, logfile=logfile)
        opt.run(fmax=fmax, steps=steps)
        E = float(atoms.get_potential_energy())
        F = np.asarray(atoms.get_forces(), dtype=np.float64)
        fm = float((F ** 2).sum(1).max() ** 0.5)
        return dict(energy=E, forces=F, fmax=fm, nsteps=int(opt.nsteps), converged=fm <= fmax)
    force_fn, pos = _native_forces(atoms)
    log = None
    if logfile is not None:
        def log(n, E, F):
            print(f"  FIRE {n:4d}  E={float(E):.6f}  fmax={float(F.norm(dim=1).max()):.4f}")
    res = D.fire(force_fn, pos, fmax=fmax, steps=steps, callback=log)
    _L.check_device()
    atoms.set_positions(pos.cpu().numpy())
    F = res["forces"].cpu().numpy()
    return dict(energy=res["energy"], forces=F, fmax=res["fmax"], nsteps=res["nsteps"],
                converged=res["fmax"] <= fmax)


def md_atoms(atoms, *, steps=100, dt=1.0, temp=300.0, logfile=None, seed=None, native=None,
             friction=0.01, masses=None):
    """Langevin MD in place (velocities drawn at ``temp`` first; ``dt`` in fs, ``friction`` in
    1/fs); returns dict(energy, forces, nsteps, temp, dt)."""
    if native is None:
        native = not HAVE_ASE
    if not native:
        from ase import units
        from ase.md.langevin import Langevin
        from ase.md.velocitydistribution import MaxwellBoltzmannDistribution
        if seed is not None:
            np.random.seed(seed)
            MaxwellBoltzmannDistribution(atoms, temperature_K=temp,
                                         rng=np.random.default_rng(seed))
        else:
            MaxwellBoltzmannDistribution(atoms, temperature_K=temp)
        dyn = Langevin(atoms, timestep=dt * units.fs, temperature_K=temp,
                       friction=friction / units.fs, logfile=logfile)
        dyn.run(steps)
        E = float(atoms.get_potential_energy())
        F = np.asarray(atoms.get_forces(), dtype=np.float64)
        return dict(energy=E, forces=F, nsteps=int(dyn.nsteps), temp=float(temp), dt=float(dt))
    force_fn, pos = _native_forces(atoms)
    m = (D.masses_of(atoms.get_atomic_numbers(), device=pos.device) if masses is None
         else torch.as_tensor(masses, dtype=torch.float64, device=pos.device))
    gen = torch.Generator(device=pos.device)
    gen.manual_seed(0 if seed is None else int(seed))
    if seed is None:
        gen.seed()
    log = None
    if logfile is not None:
        def log(n, E, F, v):
            if n % max(1, steps // 10) == 0:
                print(f"  step {n:4d}  E={float(E):.5f}  T={D.temperature(v, m):.1f} K")
    res = D.langevin(force_fn, pos, m, steps, dt_fs=dt, temp=temp, friction_fs=friction,
                     generator=gen, callback=log)
    _L.check_device()
    atoms.set_positions(pos.cpu().numpy())
    return dict(energy=res["energy"], forces=res["forces"].cpu().numpy(), nsteps=steps,
                temp=float(temp), dt=float(dt))
