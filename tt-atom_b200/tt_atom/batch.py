"""Multi-GPU throughput pools: one spawned worker process per GPU pulling independent systems
from a shared queue (tt_atom/batch.py:23-64,218-402 in the reference). No collectives: each
system runs the single-GPU path inside exactly one worker, so per-system results equal the
single-GPU results bit for bit.
"""
from __future__ import annotations

import multiprocessing as mp
import os

import numpy as np


def _pin_worker(device_id):
    """Make ``device_id`` this worker's only visible GPU and keep host threads to one."""
    os.environ["CUDA_VISIBLE_DEVICES"] = str(device_id)
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    import torch
    torch.set_num_threads(1)


class _WorkerPool:
    def __init__(self, target, args_per_device):
        self.ctx = mp.get_context("spawn")
        self.in_q = self.ctx.Queue()
        self.out_q = self.ctx.Queue()
        self.procs = [self.ctx.Process(target=target, args=(*a, self.in_q, self.out_q),
                                       daemon=True) for a in args_per_device]
        for p in self.procs:
            p.start()
        for _ in self.procs:
            msg = self.out_q.get()
            if msg[0] != "ready":
                self.close()
                raise RuntimeError(f"worker failed to start: {msg}")

    def close(self):
        for _ in self.procs:
            self.in_q.put(None)
        for p in self.procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def _energy_worker(device_id, weights_path, in_q, out_q):
    # the family comes from the bundle's config (tt_atom/batch.py:218-230): UMA bundles give the
    # eSCN-MD energy, Orb bundles the Orb energy with its normaliser and ZBL term
    try:
        _pin_worker(device_id)
        from .calculator import TTAtomCalculator
        from .weights import WeightBundle
        bundle = WeightBundle.load(weights_path)
        if "latent_dim" in bundle.config:
            from .ase_compat import SimpleAtoms
            from .orb import OrbCalculator
            orb = OrbCalculator(bundle, device_id=0)
        else:
            orb = None
            calc = TTAtomCalculator(bundle, device_id=0)
    except Exception as e:  # noqa: BLE001
        out_q.put(("error", f"{type(e).__name__}: {e}"))
        return
    out_q.put(("ready", device_id))
    while True:
        job = in_q.get()
        if job is None:
            break
        idx, pos, Z = job
        try:
            if orb is not None:
                a = SimpleAtoms(Z, pos)
                orb.calculate(a, ("energy",))
                out_q.put((idx, float(orb.results["energy"]), orb._ws.graph.E))
                continue
            E, _, _ = calc._evaluate(pos, Z, None, None, [0.0], [0.0], forces=False)
            g = calc._ws.graph
            out_q.put((idx, calc.scale_rmsd * float(E[0]) + calc.scale_mean, g.E))
        except Exception as e:  # noqa: BLE001
            out_q.put((idx, float("nan"), 0))


class MultiCard(_WorkerPool):
    """Energies of independent systems over several GPUs (tt_atom/batch.py:218-243)."""

    def __init__(self, weights_path, device_ids=(0, 1, 2, 3), *, fast=False, bucketing=False):
        super().__init__(_energy_worker, [(d, weights_path) for d in device_ids])

    def energies(self, systems):
        for i, (pos, Z) in enumerate(systems):
            self.in_q.put((i, np.asarray(pos, np.float32), np.asarray(Z, np.int64)))
        out, total = [None] * len(systems), 0
        for _ in systems:
            idx, en, E = self.out_q.get()
            out[idx] = en
            total += E
        return out, total


def _sim_worker(device_id, model, task, trace, sim_params, cache_dir, in_q, out_q):
    try:
        _pin_worker(device_id)
        from . import Calculator
        from .ase_compat import HAVE_ASE, SimpleAtoms
    except Exception as e:  # noqa: BLE001
        out_q.put(("error", f"{type(e).__name__}: {e}"))
        return
    mode = sim_params["mode"]
    # one calculator per bundle: a bundle path or an Orb checkpoint serves every structure; a
    # UMA model name needs the merged bundle of each (reduced composition, charge, spin)
    # (tt_atom/batch.py:262-295)
    import os
    from .weights import reduced_composition
    per_system = not os.path.exists(str(model)) and str(model).lower().startswith("uma")
    calcs = {}
    out_q.put(("ready", device_id))
    while True:
        job = in_q.get()
        if job is None:
            break
        idx, d = job
        try:
            if d.get("fail"):
                raise RuntimeError(d["fail"])
            if HAVE_ASE:
                from ase import Atoms
                atoms = Atoms(numbers=d["Z"], positions=d["pos"], cell=d.get("cell"),
                              pbc=d.get("pbc", False))
            else:
                atoms = SimpleAtoms(d["Z"], d["pos"], d.get("cell"), d.get("pbc", False))
            atoms.info.update(charge=d.get("charge", 0.0), spin=d.get("spin", 0.0))
            key = ((reduced_composition(np.asarray(d["Z"]).tolist()), atoms.info["charge"],
                    atoms.info["spin"]) if per_system else "all")
            if key not in calcs:
                calcs[key] = Calculator(atoms if per_system else None, model, task=task,
                                        device_id=0, trace=trace, cache_dir=cache_dir)
            atoms.calc = calcs[key]
            if mode == "energy":
                res = dict(energy=float(atoms.get_potential_energy()),
                           forces=np.asarray(atoms.get_forces(), dtype=np.float64),
                           fmax=None, nsteps=0, converged=None)
            else:
                # ASE's optimiser / integrator when ASE is installed, else the GPU-resident
                # loops of tt_atom.dynamics
                from .simulate import md_atoms, relax_atoms
                if mode == "relax":
                    res = relax_atoms(atoms, fmax=sim_params["fmax"], steps=sim_params["steps"])
                else:
                    res = md_atoms(atoms, steps=sim_params["steps"], dt=sim_params["dt"],
                                   temp=sim_params["temp"], seed=sim_params.get("seed"))
            out_q.put((idx, dict(ok=True, pos=atoms.get_positions(), Z=d["Z"],
                                 energy=res["energy"], forces=res["forces"], fmax=res.get("fmax"),
                                 nsteps=res.get("nsteps"), converged=res.get("converged"))))
        except Exception as e:  # noqa: BLE001 - ship the error back, keep the worker
            import traceback
            out_q.put((idx, dict(ok=False, error=f"{type(e).__name__}: {e}",
                                 tb=traceback.format_exc())))


class MultiCardSim(_WorkerPool):
    """Relax / MD / single point of independent structures over several GPUs
    (tt_atom/batch.py:338-380): same constructor, ``run`` returns per-system result dicts in
    input order, ``{ok: False, error, tb}`` for a failed system."""

    def __init__(self, model, device_ids=(0, 1, 2, 3), *, task=None, refenv=None,
                 cache_dir=None, fast=False, trace=False, sim_params=None):
        if sim_params is None or sim_params.get("mode") not in ("relax", "md", "energy"):
            raise ValueError("sim_params must be a dict with mode 'relax', 'md', or 'energy'")
        self.sim_params = sim_params
        super().__init__(_sim_worker,
                         [(d, model, task, trace, sim_params, cache_dir) for d in device_ids])

    def run(self, systems):
        for i, s in enumerate(systems):
            self.in_q.put(_to_system_dict(s, i))
        out = [None] * len(systems)
        for _ in systems:
            idx, res = self.out_q.get()
            out[idx] = res
        return out


def _to_system_dict(system, idx):
    """ASE Atoms / (pos, Z) / dict -> the worker message (tt_atom/batch.py:383-402)."""
    if isinstance(system, dict) and "pos" in system and "Z" in system:
        return idx, system
    if isinstance(system, tuple) and len(system) == 2:
        return idx, dict(pos=np.asarray(system[0], np.float32), Z=np.asarray(system[1], np.int64))
    pbc = system.get_pbc()
    return idx, dict(pos=np.asarray(system.get_positions(), np.float32),
                     Z=np.asarray(system.get_atomic_numbers(), np.int64),
                     charge=float(system.info.get("charge", 0.0)),
                     spin=float(system.info.get("spin", 0.0)),
                     cell=np.asarray(system.get_cell()) if np.asarray(pbc).any() else None,
                     pbc=bool(np.asarray(pbc).any()))
