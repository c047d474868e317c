"""tt_atom (B200 build): the eSCN-MD (UMA) and Orb-v3 energy + force + stress path on sm_100a.

Drop-in surface of the reference package for this path:
  Calculator                     family dispatch by bundle or model name (tt_atom/auto.py:40)
  TTAtomCalculator               UMA ASE calculator, evaluate_batch, from_uma (calculator.py:23)
  orb.OrbCalculator              Orb ASE calculator, evaluate_batch, from_checkpoint
                                 (tt_atom/orb_calculator.py:26)
  MultiCard, MultiCardSim        one process per GPU (tt_atom/batch.py:218,338)
  simulate.relax_atoms, md_atoms FIRE / Langevin, GPU-resident without ASE (simulate.py:15-74)
  radius_graph                   device neighbour list (tt_atom/geometry.py:48)
  bundle_cache                   the reference's bundle cache layout (bundle_cache.py)
"""
from .calculator import TTAtomCalculator
from .weights import WeightBundle

__version__ = "0.1.0"


def Calculator(atoms=None, model="uma-s-1", *, task=None, charge=0, spin=1, refenv=None,
               checkpoint=None, cache_dir=None, device=None, device_id=0, fast=False,
               trace=False, **kw):
    """Family dispatch of the reference (tt_atom/auto.py:40-89). ``model`` is either a model
    name, as in the reference ('uma-*': the cached merged bundle for the atoms' composition,
    charge, spin and task; 'orb-v3-*': the cached checkpoint weights; see ``bundle_cache``), or
    the path of an exported ``.npz`` weight bundle, whose config selects the family (UMA /
    eSCN-MD -> ``TTAtomCalculator``, Orb -> ``OrbCalculator``). Building a missing bundle needs
    the reference environment (fairchem / orb-models), which this build does not provide."""
    path = checkpoint or model
    import os
    if not (isinstance(path, str) and os.path.exists(path)):
        # a model name, as in the reference: the bundle comes from the reference's cache layout
        from . import bundle_cache as BC
        m = str(model).lower()
        if m.startswith("uma"):
            if atoms is None:
                raise ValueError(
                    "a UMA model needs `atoms` to determine the composition — MoLE bakes one "
                    "bundle per reduced composition/charge/spin/task, so there is no bundle to "
                    "pick or build without the structure. Pass the Atoms you want to run.")
            calc = TTAtomCalculator.from_uma(
                model=model, task_name=task or BC.infer_task(atoms), atoms=atoms, charge=charge,
                spin=spin, refenv=refenv, checkpoint=checkpoint, cache_dir=cache_dir,
                device=device, device_id=device_id, fast=fast, trace=trace, **kw)
            atoms.calc = calc
            return calc
        if m.startswith("orb"):
            if task is not None:
                raise ValueError(
                    f"`task` applies only to UMA models; the Orb checkpoint {model!r} has no task "
                    "selector (the checkpoint itself fixes omat vs omol). Drop task=.")
            if checkpoint is not None:
                raise ValueError(
                    f"for Orb the model name is the checkpoint (model={model!r}); there is no "
                    "separate raw-checkpoint override to pass. Drop checkpoint=.")
            if atoms is not None:
                atoms.info.setdefault("charge", charge)
                atoms.info.setdefault("spin", spin)
            from .orb import OrbCalculator
            calc = OrbCalculator.from_checkpoint(checkpoint=model, refenv=refenv,
                                                 cache_dir=cache_dir, device=device,
                                                 device_id=device_id, trace=trace, **kw)
            if atoms is not None:
                atoms.calc = calc
            return calc
        raise ValueError(
            f"unknown model {model!r}: expected a UMA model (e.g. 'uma-s-1'), an Orb checkpoint "
            f"(one of {', '.join(BC.ORB_CHECKPOINTS)}) or the path of a weight bundle (.npz).")
    bundle = WeightBundle.load(path)
    if "latent_dim" in bundle.config:
        # Orb family: the checkpoint fixes omat vs omol, so there is no task selector
        if task is not None:
            raise ValueError(
                f"`task` applies only to UMA models; the Orb checkpoint {model!r} has no task "
                "selector (the checkpoint itself fixes omat vs omol). Drop task=.")
        from .orb import OrbCalculator
        if atoms is not None:
            atoms.info.setdefault("charge", charge)
            atoms.info.setdefault("spin", spin)
        calc = OrbCalculator(bundle, device=device, device_id=device_id, trace=trace, **kw)
        if atoms is not None:
            atoms.calc = calc
        return calc
    if "sphere_channels" not in bundle.config:
        raise ValueError(f"unknown model {model!r}: expected a UMA or an Orb weight bundle")
    if atoms is not None:
        atoms.info.setdefault("charge", charge)
        atoms.info.setdefault("spin", spin)
    calc = TTAtomCalculator(bundle, task_name=task, device=device, device_id=device_id,
                            fast=fast, trace=trace, **kw)
    if atoms is not None:
        atoms.calc = calc
    return calc


def __getattr__(name):
    if name in ("MultiCard", "MultiCardSim"):
        from . import batch
        return getattr(batch, name)
    if name == "radius_graph":
        from .graph import radius_graph
        return radius_graph
    raise AttributeError(name)
