"""``tt-atom run``: structures in, single point / relax / MD out, on one GPU or fanned out over
several (the reference's command of tt_atom/cli.py:179-256).

    python -m tt_atom.cli run STRUCTURE [STRUCTURE ...] [--model uma-s-1|BUNDLE.npz]
        [--task T] [--charge Q] [--spin S] [--relax | --md] [--devices 0,1,...] [--trace]
        [--fmax F] [--steps N] [--dt FS] [--temp K] [--seed S] [--out PATH]

Same options and behaviour as the reference's ``run``: one structure (or no ``--devices``) runs
the structures one after another on ``--device-id``; with ``--devices`` and several structures
they are fanned out over the listed GPUs through ``MultiCardSim`` (one worker process per GPU,
no collectives). A structure that fails is reported and the command exits 1, after writing the
others' results. ``--model`` (an addition) takes a model name, as the reference's fixed
"uma-s-1", or the path of an exported weight bundle.

Structures are read with ASE when it is installed; without it, extended XYZ files
(``Lattice="..."`` and ``pbc="..."`` in the comment line, species symbols or atomic numbers in the
first column) are read and written by this module.
"""
from __future__ import annotations

import argparse
import pathlib
import re
import sys

import numpy as np

from .ase_compat import HAVE_ASE, SimpleAtoms

_SYMBOLS = (
    "X H He Li Be B C N O F Ne Na Mg Al Si P S Cl Ar K Ca Sc Ti V Cr Mn Fe Co Ni Cu Zn Ga Ge As "
    "Se Br Kr Rb Sr Y Zr Nb Mo Tc Ru Rh Pd Ag Cd In Sn Sb Te I Xe Cs Ba La Ce Pr Nd Pm Sm Eu Gd "
    "Tb Dy Ho Er Tm Yb Lu Hf Ta W Re Os Ir Pt Au Hg Tl Pb Bi Po At Rn Fr Ra Ac Th Pa U Np Pu Am "
    "Cm Bk Cf Es Fm Md No Lr Rf Db Sg Bh Hs Mt Ds Rg Cn Nh Fl Mc Lv Ts Og").split()
_NUMBER = {s: z for z, s in enumerate(_SYMBOLS)}


# ----------------------------------------------------------------------------- structure I/O
def read_xyz(path):
    """One structure from an (extended) XYZ file as a ``SimpleAtoms``."""
    lines = pathlib.Path(path).read_text().splitlines()
    n = int(lines[0].split()[0])
    comment = lines[1] if len(lines) > 1 else ""
    Z, pos = [], []
    for ln in lines[2:2 + n]:
        f = ln.split()
        Z.append(int(f[0]) if f[0].isdigit() else _NUMBER[f[0]])
        pos.append([float(v) for v in f[1:4]])
    if len(Z) != n:
        raise ValueError(f"{path}: expected {n} atoms, found {len(Z)}")
    cell, pbc = None, False
    m = re.search(r'Lattice="([^"]+)"', comment)
    if m:
        cell = np.array([float(v) for v in m.group(1).split()]).reshape(3, 3)
        p = re.search(r'pbc="([^"]+)"', comment)
        pbc = [v.upper() in ("T", "TRUE", "1") for v in p.group(1).split()] if p else True
    return SimpleAtoms(Z, pos, cell, pbc)


def write_xyz(path, Z, pos, cell=None, pbc=False, energy=None, forces=None):
    """Extended XYZ with the lattice, pbc, energy and per-atom forces."""
    pbc = np.broadcast_to(np.asarray(pbc, dtype=bool), (3,))
    head = []
    if cell is not None and pbc.any():
        head.append('Lattice="' + " ".join(f"{v:.8f}" for v in np.asarray(cell).ravel()) + '"')
    head.append('pbc="' + " ".join("T" if b else "F" for b in pbc) + '"')
    head.append("Properties=species:S:1:pos:R:3" + (":forces:R:3" if forces is not None else ""))
    if energy is not None:
        head.append(f"energy={float(energy):.10f}")
    out = [str(len(Z)), " ".join(head)]
    for k, (z, p) in enumerate(zip(Z, np.asarray(pos))):
        row = f"{_SYMBOLS[int(z)]} {p[0]:.8f} {p[1]:.8f} {p[2]:.8f}"
        if forces is not None:
            f = np.asarray(forces)[k]
            row += f" {f[0]:.8f} {f[1]:.8f} {f[2]:.8f}"
        out.append(row)
    pathlib.Path(path).write_text("\n".join(out) + "\n")


def read_structures(paths):
    if HAVE_ASE:
        from ase.io import read
        return [read(p) for p in paths]
    return [read_xyz(p) for p in paths]


def _write(path, Z, pos, cell, pbc, energy, forces):
    if HAVE_ASE:
        from ase import Atoms
        from ase.calculators.singlepoint import SinglePointCalculator
        from ase.io import write
        a = Atoms(numbers=Z, positions=pos, cell=cell, pbc=pbc)
        a.calc = SinglePointCalculator(a, energy=float(energy),
                                       forces=np.asarray(forces, dtype=float))
        write(str(path), a)
    else:
        write_xyz(path, Z, pos, cell, pbc, energy, forces)


# ---------------------------------------------------------------------------------- run
def parse_devices(text):
    try:
        ids = tuple(int(p) for p in str(text).split(",") if p.strip())
    except ValueError as e:
        raise SystemExit(f"--devices expects a comma-separated list of GPU ids (e.g. 0,1,2): {e}")
    if not ids:
        raise SystemExit("--devices lists no GPU")
    if len(set(ids)) != len(ids):
        raise SystemExit(f"--devices lists a GPU twice: {text}")
    return ids


def _mode(args):
    return "relax" if args.relax else ("md" if args.md else "energy")


def _fmax(forces):
    return float(np.max(np.linalg.norm(np.asarray(forces, dtype=float), axis=1)))


def _summary(i, name, res, mode):
    line = f"  [{i}] {name}: E={res['energy']:.6f} eV"
    if mode == "energy":
        return line + f", fmax={_fmax(res['forces']):.4f}"
    line += f", steps={res.get('nsteps')}"
    if mode == "relax":
        line += f", fmax={res['fmax']:.4f}, converged={res['converged']}"
    return line


def _out_path(args, i, many):
    out = pathlib.Path(args.out)
    if not many:
        return out
    folder = out.parent if out.suffix else out
    folder.mkdir(parents=True, exist_ok=True)
    return folder / f"{pathlib.Path(args.structures[i]).stem}_{i}{out.suffix or '.xyz'}"


def _report(args, structures, results):
    mode, many = _mode(args), len(structures) > 1
    for i, (src, res) in enumerate(zip(structures, results)):
        if not res.get("ok"):
            print(f"  [{i}] FAILED: {res.get('error', '?')}")
            if res.get("tb"):
                print(res["tb"])
            continue
        print(_summary(i, pathlib.Path(args.structures[i]).name, res, mode))
        if args.out:
            p = _out_path(args, i, many)
            periodic = bool(np.any(src.get_pbc()))
            _write(p, res["Z"], res["pos"], src.get_cell() if periodic else None,
                   src.get_pbc(), res["energy"], res["forces"])
            print(f"      wrote {p}")
    bad = sum(not r.get("ok") for r in results)
    if bad:
        print(f"  {bad}/{len(results)} structure(s) FAILED; results written for the rest; "
              "exiting 1.")
    return 1 if bad else 0


def _single_gpu(args, structures):
    """Structures one after another on one GPU, each through the public Calculator."""
    import traceback

    from . import Calculator
    from .simulate import md_atoms, relax_atoms
    mode, results = _mode(args), []
    for atoms in structures:
        try:
            calc = Calculator(atoms, args.model, task=args.task, charge=args.charge,
                              spin=args.spin, refenv=args.refenv, device_id=args.device_id,
                              trace=args.trace)
            atoms.calc = calc
            if mode == "energy":
                res = dict(energy=float(atoms.get_potential_energy()),
                           forces=np.asarray(atoms.get_forces(), dtype=np.float64))
            elif mode == "relax":
                res = relax_atoms(atoms, fmax=args.fmax, steps=args.steps)
            else:
                res = md_atoms(atoms, steps=args.steps, dt=args.dt, temp=args.temp,
                               seed=args.seed)
            results.append(dict(res, ok=True, pos=atoms.get_positions(),
                                Z=atoms.get_atomic_numbers()))
            calc.close()
        except Exception as e:  # noqa: BLE001 - report it, go on with the next structure
            results.append(dict(ok=False, error=f"{type(e).__name__}: {e}",
                                tb=traceback.format_exc()))
    return results


def _fan_out(args, structures, devices):
    """Independent structures over several GPUs (MultiCardSim, no collectives)."""
    from .batch import MultiCardSim
    mode = _mode(args)
    params = dict(mode=mode, fmax=args.fmax, steps=args.steps, dt=args.dt, temp=args.temp,
                  seed=args.seed)
    print(f"multi-GPU: {len(structures)} structure(s) over {len(devices)} GPU(s) "
          f"({','.join(map(str, devices))}), mode={mode}")
    with MultiCardSim(args.model, device_ids=devices, task=args.task, refenv=args.refenv,
                      trace=args.trace, sim_params=params) as pool:
        return pool.run(structures)


def cmd_run(args):
    structures = read_structures(args.structures)
    for a in structures:
        a.info.setdefault("charge", args.charge)
        a.info.setdefault("spin", args.spin)
    devices = parse_devices(args.devices) if args.devices else (args.device_id,)
    fan_out = args.devices is not None and (len(devices) > 1 or len(structures) > 1)
    results = _fan_out(args, structures, devices) if fan_out else _single_gpu(args, structures)
    return _report(args, structures, results)


def build_parser():
    ap = argparse.ArgumentParser(prog="tt-atom", description="tt-atom on B200 GPUs")
    ap.add_argument("--device-id", type=int, default=0)
    ap.add_argument("--fast", action="store_true", help="accepted; no effect on this GPU build")
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("run", help="structures -> single point / relax / md")
    p.add_argument("structures", nargs="+", help="structure file(s); several fan out over "
                                                 "--devices")
    p.add_argument("--uma-s-1", action="store_true", help=argparse.SUPPRESS)
    p.add_argument("--model", default="uma-s-1",
                   help="model name (uma-s-1, an orb-v3 checkpoint) or a weight bundle path")
    p.add_argument("--task", default=None)
    p.add_argument("--charge", type=float, default=0.0)
    p.add_argument("--spin", type=float, default=1.0)
    p.add_argument("--refenv", default=None)
    p.add_argument("--trace", action="store_true", help="replay the step as a CUDA graph")
    p.add_argument("--devices", default=None, help="comma-separated GPU ids for the fan-out")
    p.add_argument("--seed", type=int, default=None, help="MD velocity seed")
    g = p.add_mutually_exclusive_group()
    g.add_argument("--relax", action="store_true", help="FIRE relaxation")
    g.add_argument("--md", action="store_true", help="Langevin MD")
    p.add_argument("--fmax", type=float, default=0.05)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--dt", type=float, default=1.0)
    p.add_argument("--temp", type=float, default=300.0)
    p.add_argument("--out", help="final geometry file (one structure) or folder (several)")
    p.set_defaults(func=cmd_run)
    return ap


def main(argv=None):
    args = build_parser().parse_args(argv)
    return args.func(args)


if __name__ == "__main__":
    sys.exit(main())
