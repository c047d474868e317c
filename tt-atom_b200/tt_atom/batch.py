"""Multi-GPU throughput pools over independent systems: ``MultiCard`` (energies) and
``MultiCardSim`` (relax / MD / single point), the reference's entry points of
tt_atom/batch.py:218-243 and 338-380 (same constructors, result lists in input order, the
``{ok: False, error, tb}`` record for a system that failed).

Design. One spawned process per GPU, each with that GPU as its only visible device. Each
worker has its own inbox, and the pool hands it the next system only when it has returned the
previous one, so faster GPUs take more systems and the pool always knows which system each
worker holds. Results come back on one shared outbox. While waiting, the pool checks that the
workers are alive: a worker that exits (a crash, an out-of-memory kill, ``os._exit``) has its
system reported as failed and is retired, and the remaining systems go to the other workers.
No collectives: each system runs the single-GPU path inside exactly one worker, so per-system
results equal the single-GPU results bit for bit.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import queue
import traceback

import numpy as np

_STOP = "stop"
_POLL_S = 0.5


def _isolate_device(device_id):
    """Make ``device_id`` this worker's only visible GPU; one host thread for torch."""
    os.environ["CUDA_VISIBLE_DEVICES"] = str(device_id)
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    import torch
    torch.set_num_threads(1)


def _serve(slot, device_id, make_handler, make_args, inbox, outbox):
    """Worker main loop: build the handler once, then answer ("job", idx, payload) messages
    with ("done", slot, idx, result) until ("stop",). A handler exception is the handler's to
    turn into a result; one that escapes is shipped back as a failed record."""
    try:
        _isolate_device(device_id)
        handler = make_handler(*make_args)
    except BaseException as e:  # noqa: BLE001 - report the start-up failure, then exit
        outbox.put(("failed", slot, f"{type(e).__name__}: {e}", traceback.format_exc()))
        return
    outbox.put(("up", slot, None, None))
    while True:
        msg = inbox.get()
        if msg[0] == _STOP:
            break
        _, idx, payload = msg
        try:
            result = handler(payload)
        except Exception as e:  # noqa: BLE001
            result = _failure(e)
        outbox.put(("done", slot, idx, result))


def _failure(e):
    return dict(ok=False, error=f"{type(e).__name__}: {e}", tb=traceback.format_exc())


class _DevicePool:
    """One worker process per device id; ``map`` runs a list of payloads through them."""

    def __init__(self, make_handler, make_args, device_ids, lost=None):
        # ``lost(idx, why)`` is the result recorded for a payload whose worker died
        self._lost = lost or (lambda idx, why: dict(ok=False, error=why, tb=""))
        ctx = mp.get_context("spawn")
        self._outbox = ctx.Queue()
        self._inbox, self._proc, self._dev = [], [], list(device_ids)
        for slot, dev in enumerate(self._dev):
            q = ctx.Queue()
            p = ctx.Process(target=_serve, args=(slot, dev, make_handler, make_args, q,
                                                 self._outbox), daemon=True)
            p.start()
            self._inbox.append(q)
            self._proc.append(p)
        self._live = set()
        waiting = set(range(len(self._dev)))
        problems = []
        while waiting:
            try:
                kind, slot, a, b = self._outbox.get(timeout=_POLL_S)
            except queue.Empty:
                for slot in list(waiting):
                    if not self._proc[slot].is_alive():
                        waiting.discard(slot)
                        problems.append(f"device {self._dev[slot]}: worker exited with code "
                                        f"{self._proc[slot].exitcode} during start-up")
                continue
            waiting.discard(slot)
            if kind == "up":
                self._live.add(slot)
            else:
                problems.append(f"device {self._dev[slot]}: {a}")
        if problems:
            self.close()
            raise RuntimeError("worker failed to start: " + "; ".join(problems))

    def map(self, payloads):
        results = [None] * len(payloads)
        todo = list(range(len(payloads)))[::-1]     # pop() hands them out in input order
        holding = {}                                # slot -> payload index in flight

        def hand_out(slot):
            if todo:
                idx = todo.pop()
                holding[slot] = idx
                self._inbox[slot].put(("job", idx, payloads[idx]))

        for slot in sorted(self._live):
            hand_out(slot)
        while holding:
            try:
                kind, slot, idx, res = self._outbox.get(timeout=_POLL_S)
            except queue.Empty:
                self._reap(holding, results, hand_out=None)
                if not self._live and todo:
                    for idx in todo:
                        results[idx] = self._lost(idx, "no live worker left in the pool")
                    todo.clear()
                continue
            if kind != "done" or holding.get(slot) != idx:
                continue
            del holding[slot]
            results[idx] = res
            hand_out(slot)
        for idx in todo:        # every worker died with systems still queued
            results[idx] = self._lost(idx, "no live worker left in the pool")
        return results

    def _reap(self, holding, results, hand_out):
        for slot in list(self._live):
            p = self._proc[slot]
            if p.is_alive():
                continue
            self._live.discard(slot)
            if slot in holding:
                idx = holding.pop(slot)
                results[idx] = self._lost(
                    idx, f"WorkerDied: the worker on device {self._dev[slot]} exited with code "
                         f"{p.exitcode} while running this system")

    @property
    def live_devices(self):
        return [self._dev[s] for s in sorted(self._live)]

    def close(self):
        for slot, p in enumerate(self._proc):
            if p.is_alive():
                self._inbox[slot].put((_STOP,))
        for p in self._proc:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
                p.join(timeout=5)
        self._live.clear()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


# ------------------------------------------------------------------------------ handlers
class _EnergyHandler:
    """Raw-model energy of one (pos, Z) system; the family comes from the bundle's config
    (tt_atom/batch.py:218-230): UMA bundles give the eSCN-MD energy with its normaliser, Orb
    bundles the Orb energy with its normaliser and ZBL term. Returns (energy, edge count);
    a failed system gives (nan, 0), as the reference's energy workers do."""

    def __init__(self, weights_path):
        from .weights import WeightBundle
        bundle = WeightBundle.load(weights_path)
        self.orb = self.uma = None
        if "latent_dim" in bundle.config:
            from .orb import OrbCalculator
            self.orb = OrbCalculator(bundle, device_id=0)
        else:
            from .calculator import TTAtomCalculator
            self.uma = TTAtomCalculator(bundle, device_id=0)

    def __call__(self, payload):
        pos, Z = payload
        try:
            if self.orb is not None:
                from .ase_compat import SimpleAtoms
                self.orb.calculate(SimpleAtoms(Z, pos), ("energy",))
                return float(self.orb.results["energy"]), self.orb._ws.graph.E
            c = self.uma
            E, _, _ = c._evaluate(pos, Z, None, None, [0.0], [0.0], forces=False)
            return c.scale_rmsd * float(E[0]) + c.scale_mean, c._ws.graph.E
        except Exception:  # noqa: BLE001
            return float("nan"), 0


class _SimHandler:
    """Relax / MD / single point of one system message (see ``_system_message``). A bundle
    path or an Orb checkpoint serves every structure with one calculator; a UMA model name needs
    the merged bundle of each (reduced composition, charge, spin), so calculators are cached by
    that key (tt_atom/batch.py:262-295)."""

    def __init__(self, model, task, trace, sim_params, cache_dir):
        self.model, self.task, self.trace = model, task, trace
        self.params, self.cache_dir = sim_params, cache_dir
        self.per_composition = (not os.path.exists(str(model))
                                and str(model).lower().startswith("uma"))
        self.calcs = {}

    def _atoms(self, d):
        from .ase_compat import HAVE_ASE, SimpleAtoms
        if HAVE_ASE:
            from ase import Atoms
            a = Atoms(numbers=d["Z"], positions=d["pos"], cell=d.get("cell"),
                      pbc=d.get("pbc", False))
        else:
            a = SimpleAtoms(d["Z"], d["pos"], d.get("cell"), d.get("pbc", False))
        a.info.update(charge=d.get("charge", 0.0), spin=d.get("spin", 0.0))
        return a

    def _calculator(self, atoms):
        from . import Calculator
        from .weights import reduced_composition
        key = "shared"
        if self.per_composition:
            key = (reduced_composition(np.asarray(atoms.get_atomic_numbers()).tolist()),
                   atoms.info["charge"], atoms.info["spin"])
        if key not in self.calcs:
            self.calcs[key] = Calculator(atoms if self.per_composition else None, self.model,
                                         task=self.task, device_id=0, trace=self.trace,
                                         cache_dir=self.cache_dir)
        return self.calcs[key]

    def __call__(self, d):
        try:
            atoms = self._atoms(d)
            atoms.calc = self._calculator(atoms)
            mode, p = self.params["mode"], self.params
            if mode == "energy":
                res = dict(energy=float(atoms.get_potential_energy()),
                           forces=np.asarray(atoms.get_forces(), dtype=np.float64),
                           fmax=None, nsteps=0, converged=None)
            elif mode == "relax":
                from .simulate import relax_atoms
                res = relax_atoms(atoms, fmax=p["fmax"], steps=p["steps"])
            else:
                from .simulate import md_atoms
                res = md_atoms(atoms, steps=p["steps"], dt=p["dt"], temp=p["temp"],
                               seed=p.get("seed"))
        except Exception as e:  # noqa: BLE001 - one bad system must not stop the pool
            return _failure(e)
        return dict(ok=True, pos=atoms.get_positions(), Z=d["Z"], energy=res["energy"],
                    forces=res["forces"], fmax=res.get("fmax"), nsteps=res.get("nsteps"),
                    converged=res.get("converged"))


def _system_message(system):
    """What a worker receives for one system: a dict with pos (float32), Z (int64) and, when
    the input carries them, charge, spin, cell and pbc. Accepts the dict form itself, a
    (positions, atomic numbers) pair, or anything with ASE's Atoms accessors."""
    if isinstance(system, dict):
        if "pos" not in system or "Z" not in system:
            raise ValueError("a system dict needs 'pos' and 'Z'")
        return system
    if isinstance(system, (tuple, list)) and len(system) == 2:
        pos, Z = system
        return {"pos": np.asarray(pos, np.float32), "Z": np.asarray(Z, np.int64)}
    periodic = bool(np.any(system.get_pbc()))
    msg = {"pos": np.asarray(system.get_positions(), np.float32),
           "Z": np.asarray(system.get_atomic_numbers(), np.int64),
           "pbc": periodic, "cell": np.asarray(system.get_cell()) if periodic else None}
    for k in ("charge", "spin"):
        msg[k] = float(system.info.get(k, 0.0))
    return msg


# ------------------------------------------------------------------------- public pools
class MultiCard(_DevicePool):
    """Energies of independent systems over several GPUs (tt_atom/batch.py:218-243)."""

    def __init__(self, weights_path, device_ids=(0, 1, 2, 3), *, fast=False, bucketing=False):
        super().__init__(_EnergyHandler, (weights_path,), device_ids,
                         lost=lambda idx, why: (float("nan"), 0))

    def energies(self, systems):
        """(energies in input order, total edge count); nan for a system that failed."""
        out = self.map([(np.asarray(p, np.float32), np.asarray(z, np.int64))
                        for p, z in systems])
        return [e for e, _ in out], sum(n for _, n in out)


class MultiCardSim(_DevicePool):
    """Relax / MD / single point of independent structures over several GPUs
    (tt_atom/batch.py:338-380): same constructor, ``run`` returns per-system result dicts in
    input order, ``{ok: False, error, tb}`` for a system that failed (including one whose worker
    died under it; the pool goes on with the workers that are left)."""

    def __init__(self, model, device_ids=(0, 1, 2, 3), *, task=None, refenv=None,
                 cache_dir=None, fast=False, trace=False, sim_params=None):
        if sim_params is None or sim_params.get("mode") not in ("relax", "md", "energy"):
            raise ValueError("sim_params must be a dict with mode 'relax', 'md', or 'energy'")
        self.sim_params = sim_params
        super().__init__(_SimHandler, (model, task, trace, sim_params, cache_dir), device_ids)

    def run(self, systems):
        return self.map([_system_message(s) for s in systems])
