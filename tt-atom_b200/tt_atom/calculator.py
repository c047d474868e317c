"""``TTAtomCalculator``: the ASE calculator over the GPU engine (drop-in for the reference's
tt_atom/calculator.py:23-277 and tt_atom/ase_base.py:18-54).

Same constructor and methods (``calculate``, ``evaluate_batch``, ``close``), same results keys
(energy, free_energy, energies, forces, stress), same energy normaliser
(``E = rmsd * E_raw + mean + sum refs[Z]``, ``F = rmsd * F_raw``, stress = rmsd * virial / V as
Voigt-6) and the same errors (no edges -> ValueError; task mismatch -> ValueError). ``device`` /
``device_id`` name a CUDA device. ``trace=True`` captures the step in a CUDA graph per topology
and replays it while the neighbour list (and image shifts) are unchanged. ``precision``:
"3xtf32" (default; tcgen05 tensor cores with fp32-level accuracy), "fp32" (FMA pipe) or "tf32"
(one tensor-core pass, looser).
"""
from __future__ import annotations

import numpy as np
import torch

from .ase_compat import _AseCalculator, all_changes, atoms_volume, voigt_6
from .engine import CapturedStep, UMAEngine, to_host, upload_positions
from .graph import build_graph, csd_embedding
from .weights import WeightBundle, reduced_composition


def _fields(system):
    """positions, Z, charge, spin, cell, pbc of an ASE Atoms / dict / (pos, Z) tuple
    (tt_atom/disjoint.py:30-56)."""
    if hasattr(system, "get_positions"):
        pbc = np.asarray(system.get_pbc())
        cell = np.asarray(system.get_cell(), dtype=np.float32) if pbc.any() else None
        return (np.asarray(system.get_positions(), dtype=np.float32),
                np.asarray(system.get_atomic_numbers(), dtype=np.int64),
                float(system.info.get("charge", 0.0)), float(system.info.get("spin", 0.0)),
                cell, pbc if pbc.any() else None)
    if isinstance(system, dict):
        return (np.asarray(system["pos"], dtype=np.float32), np.asarray(system["Z"], np.int64),
                float(system.get("charge", 0.0)), float(system.get("spin", 0.0)),
                system.get("cell"), system.get("pbc"))
    pos, Z = system
    return np.asarray(pos, np.float32), np.asarray(Z, np.int64), 0.0, 0.0, None, None


class TTAtomCalculator(_AseCalculator):
    implemented_properties = ["energy", "energies", "free_energy", "forces", "stress"]

    def __init__(self, bundle, task_name=None, device=None, device_id=0, gamma=0.0, fast=False,
                 trace=False, precision="3xtf32", max_neighbors="config", chunk_edges="auto",
                 **kwargs):
        super().__init__(**kwargs)
        # receiver-chunked edge stages: "auto" (only when the whole workspace would not fit in
        # free device memory), None (never) or a chunk size in edges
        self.chunk_edges = chunk_edges
        if isinstance(bundle, str):
            bundle = WeightBundle.load(bundle)
        if gamma != 0.0:
            raise ValueError("only the roll gauge gamma = 0 is implemented (energy and forces "
                             "do not depend on it)")
        self.bundle = bundle
        self.cfg = bundle.config
        self.C = self.cfg["sphere_channels"]
        self.trace = trace
        self.fast = fast
        if task_name is not None and task_name != bundle.task:
            raise ValueError(
                f"task_name={task_name!r} does not match this bundle's task {bundle.task!r}. "
                f"UMA's MoLE routing bakes the task into the merged bundle; export a bundle for "
                f"{task_name!r} to use that task.")
        self.task = self.task_name = bundle.task
        self.max_neighbors = (self.cfg.get("max_neighbors") if max_neighbors == "config"
                              else max_neighbors)
        if device is None:
            device = torch.device("cuda", device_id)
        self.device = torch.device(device)
        w = bundle.weights
        self._w = w
        self.engine = UMAEngine(w, self.cfg, bundle.tables(), device=self.device,
                                precision=precision)
        self.scale_rmsd = bundle.scale_rmsd
        self.scale_mean = bundle.scale_mean
        self.elem_refs = bundle.elem_refs
        self._ws = None
        self._ws_key = None
        self._step = None

    # ------------------------------------------------------------------------------ core
    @classmethod
    def from_uma(cls, model="uma-s-1", task_name="omol", atoms=None, charge=0, spin=1,
                 refenv=None, checkpoint=None, cache_dir=None, device=None, device_id=0,
                 fast=False, trace=False, **kwargs):
        """A calculator for ``atoms`` from the cached merged bundle of its (reduced composition,
        charge, spin, task) (tt_atom/calculator.py:68-114). Charge / spin already on the atoms
        win over the arguments, and the resolved values are stamped back onto the atoms so that
        ``calculate`` reads what the bundle was merged for. A cache miss raises: building the
        bundle needs the reference environment, which this build does not include."""
        from . import bundle_cache as BC
        if atoms is None:
            raise ValueError(
                "from_uma needs `atoms` to determine the composition — MoLE bakes one bundle per "
                "reduced composition/charge/spin/task, so there is no way to pick (or build) a "
                "bundle without the structure. Pass the Atoms you want to run.")
        charge = atoms.info.get("charge", charge)
        spin = atoms.info.get("spin", spin)
        atoms.info.setdefault("charge", charge)
        atoms.info.setdefault("spin", spin)
        path = BC.cached(BC.bundle_path(model, task_name, atoms.get_atomic_numbers(), charge,
                                        spin, cache_dir=cache_dir, checkpoint=checkpoint),
                         f"{model} bundle (task {task_name}, charge {int(charge)}, spin "
                         f"{int(spin)})")
        return cls(WeightBundle.load(path), task_name=task_name, device=device,
                   device_id=device_id, fast=fast, trace=trace, **kwargs)

    def _graph(self, pos, Z, cell, pbc, sys_ptr=None):
        return build_graph(pos, Z, self.cfg["cutoff"], cell, pbc,
                           max_neighbors=self.max_neighbors, sys_ptr=sys_ptr, device=self.device)

    def _evaluate(self, pos, Z, cell, pbc, charges, spins, sys_ptr=None, forces=True,
                  stress=False, trace=False, device_out=False, graph=None):
        """Raw (unnormalised) per-system energies [nsys], forces [N, 3], virial [3, 3]|None,
        as float64 host tensors, or (``device_out``) as float32 device tensors that the next
        call overwrites (``pos`` may then be a device tensor too: nothing crosses to the host
        but the neighbour-list size)."""
        fast = None
        if trace and graph is None and sys_ptr is None:
            fast = self._device_refresh_step(pos, Z, cell, pbc, charges, spins, forces, stress,
                                             device_out)
            if fast is not None:
                return fast
        g = graph if graph is not None else self._graph(pos, Z, cell, pbc, sys_ptr)
        if g.E == 0:
            raise ValueError("no edges within cutoff — system too sparse for this model")
        se = csd_embedding(self._w, charges, spins, self.C, dataset=self.task)
        key = (g.N, g.E, bool(stress), bool(forces))
        if self._ws is not None and self._ws.fits(g) and self._ws.chunks is None:
            # same sizes: the (possibly unchanged) topology is copied into the workspace's own
            # arrays, asynchronously, instead of comparing it first; the captured step stays
            # valid and is replayed on them
            keep = self._ws_key == key
            self._ws.rebind(g, se)
        elif self._ws is not None and self._ws.fits(g):
            # chunked: the chunk plans are host-side launch parameters of a captured step, so it
            # is kept only while the topology is unchanged
            keep = (self._ws_key == key and g.same_topology(self._ws.graph)
                    and self._se is not None and torch.equal(self._se, se))
            if not keep:
                self._ws.rebind(g, se)
        else:
            keep = False
            self._ws = self._step = self._full_step = None   # free the old buffers first
            chunk = self.chunk_edges
            if chunk == "auto":
                chunk = self.engine.choose_chunk_edges(g)
            self._ws = self.engine.workspace(g, se, chunk_edges=chunk)
        self._ws_key, self._se = key, se
        if not keep:
            self._step = None
        ws = self._ws
        upload_positions(ws, pos)
        if trace:
            if self._step is None:
                self._step = CapturedStep(self.engine, ws, forces=forces, virial=stress)
            self._step()
        else:
            self.engine.run(ws, ws.pos, forces=forces, virial=stress)
        # the next traced call on this system (same atoms, cell, charge and spin) may rebuild
        # its neighbour list on the device inside the captured step
        self._refresh_key = None
        if trace and sys_ptr is None and graph is None and ws.chunks is None and g.nsys == 1:
            self._refresh_key = self._system_key(Z, cell, pbc, charges, spins, forces, stress)
        if device_out:
            return ws.energy, ws.forces if forces else None, ws.virial if stress else None
        E, F, V = to_host(ws.energy, ws.forces if forces else None,
                          ws.virial if stress else None)
        return E, F, V

    def _system_key(self, Z, cell, pbc, charges, spins, forces, stress):
        Z = np.asarray(Z, dtype=np.int64)
        return (Z.shape[0], Z.tobytes(), None if cell is None else
                np.asarray(cell, np.float32).tobytes(),
                None if pbc is None else tuple(np.broadcast_to(np.asarray(pbc, bool), 3)),
                tuple(float(c) for c in charges), tuple(float(v) for v in spins), bool(forces),
                bool(stress))

    def _device_refresh_step(self, pos, Z, cell, pbc, charges, spins, forces, stress,
                             device_out):
        """Traced evaluation of the same system as the previous call with new positions: one
        captured graph rebuilds the neighbour list on the device into the workspace's arrays
        and runs the step; one read-back returns the results and the refresh status. None
        when this path does not apply or the refresh could not keep the edge count (the caller
        then rebuilds the graph on the host side and re-captures)."""
        from .graph import TopologyRefresh
        ws = self._ws
        if (ws is None or getattr(self, "_refresh_key", None) is None or
                self._refresh_key != self._system_key(Z, cell, pbc, charges, spins, forces,
                                                      stress)):
            return None
        full = getattr(self, "_full_step", None)
        if full is None or full[0] is not ws:
            refresh = TopologyRefresh(ws.graph)
            upload_positions(ws, pos)
            step = CapturedStep(self.engine, ws, forces=forces, virial=stress,
                                prelude=lambda st: refresh.launch(ws.pos, st))
            self._full_step = full = (ws, refresh, step)
        else:
            upload_positions(ws, pos)
        _, refresh, step = full
        step()
        if device_out:
            if int(refresh.status[0]) != TopologyRefresh.OK:
                self._refresh_key = self._full_step = None
                return None
            return ws.energy, ws.forces if forces else None, ws.virial if stress else None
        E, F, V, st = to_host(ws.energy, ws.forces if forces else None,
                              ws.virial if stress else None, refresh.status[:1])
        if int(st[0]) != TopologyRefresh.OK:
            # another edge count (or candidate overflow): the step ran on the old topology
            self._refresh_key = self._full_step = None
            return None
        return E, F, V

    # ------------------------------------------------------------------------------- ASE
    def calculate(self, atoms=None, properties=("energy", "forces"), system_changes=all_changes):
        super().calculate(atoms, properties, system_changes)
        pos, Z, charge, spin, cell, pbc = _fields(atoms)
        want_stress = cell is not None and ("stress" in properties or bool(np.all(pbc)))
        E, F, V = self._evaluate(pos, Z, cell, pbc, [charge], [spin], forces=True,
                                 stress=want_stress, trace=self.trace)
        e = self.scale_rmsd * float(E[0]) + self.scale_mean
        if self.elem_refs is not None:
            e += float(self.elem_refs[torch.as_tensor(Z)].sum())
        F = (self.scale_rmsd * F).numpy()
        n = len(Z)
        self.results["energy"] = e
        self.results["free_energy"] = e
        self.results["energies"] = np.full(n, e / n, dtype=np.float64)
        self.results["forces"] = F.astype(np.float64)
        if V is not None:
            self.results["stress"] = voigt_6(self.scale_rmsd * V.numpy() / atoms_volume(atoms))

    def evaluate_batch(self, systems, properties=("energy", "forces"), trace=False):
        """Disjoint-union batch of aperiodic systems in one device pass
        (tt_atom/calculator.py:168-236). Returns dict(energy [K], forces list or None)."""
        if len(systems) == 0:
            raise ValueError("empty batch")
        # a merged bundle bakes the expert routing for one reduced composition and one (charge,
        # spin): with its reference system embedded, every batched system is checked against it
        # (tt_atom/calculator.py:193-217; same errors)
        ref = self.bundle.reference if hasattr(self.bundle, "reference") else None
        if ref is not None:
            want_comp = reduced_composition(ref["atomic_numbers"])
            want_cs = (float(ref["charge"]), float(ref["spin"]))
            for k, system in enumerate(systems):
                _, Z_k, chg_k, spin_k, _, _ = _fields(system)
                if reduced_composition(np.asarray(Z_k).tolist()) != want_comp:
                    raise ValueError(
                        f"batched system {k} has a different reduced composition than this "
                        "bundle. A merged uma-s-1 bundle bakes the MoLE routing for one reduced "
                        "composition, so every system in a batch must share it (e.g. conformers "
                        "/ an MD ensemble of one molecule); evaluate other compositions with "
                        "their own bundle.")
                if (chg_k, spin_k) != want_cs:
                    raise ValueError(
                        f"batched system {k} has (charge, spin)=({chg_k}, {spin_k}) but this "
                        f"bundle was merged for {want_cs}. The MoLE routing bakes one "
                        "charge/spin; every system in a batch must share it.")
        pos_all, Z_all, chg, spn, ptr_ = [], [], [], [], [0]
        for k, s in enumerate(systems):
            pos, Z, c, sp, cell, pbc = _fields(s)
            if cell is not None:
                raise ValueError("evaluate_batch takes aperiodic systems")
            pos_all.append(pos)
            Z_all.append(Z)
            chg.append(c)
            spn.append(sp)
            ptr_.append(ptr_[-1] + len(Z))
        want_forces = "forces" in properties
        pos = np.concatenate(pos_all)
        Z = np.concatenate(Z_all)
        g = self._graph(pos, Z, None, None, ptr_)
        cnt = torch.diff(g.recv_ptr.long().cpu())
        for k in range(len(systems)):
            if int(cnt[ptr_[k]:ptr_[k + 1]].sum()) == 0:
                raise ValueError(f"system {k} has no edges within cutoff — too sparse for this model")
        E, F, _ = self._evaluate(pos, Z, None, None, chg, spn, sys_ptr=ptr_, forces=want_forces,
                                 trace=trace, graph=g)
        energies, forces_out = [], []
        for k in range(len(systems)):
            ek = self.scale_rmsd * float(E[k]) + self.scale_mean
            if self.elem_refs is not None:
                ek += float(self.elem_refs[torch.as_tensor(Z_all[k])].sum())
            energies.append(ek)
            if want_forces:
                forces_out.append((self.scale_rmsd * F[ptr_[k]:ptr_[k + 1]]).numpy())
        return dict(energy=np.array(energies), forces=forces_out if want_forces else None)

    def close(self):
        self._ws = None
        self._step = None
        self._full_step = None
        self._refresh_key = None
