"""tt_atom (B200 build): the eSCN-MD (UMA) energy + force + stress path on sm_100a.

Drop-in surface of the reference package for this path:
  Calculator, TTAtomCalculator   ASE calculators (tt_atom/auto.py:40, tt_atom/calculator.py:23)
  MultiCard, MultiCardSim        one process per GPU (tt_atom/batch.py:218,338)
  radius_graph                   device neighbour list (tt_atom/geometry.py:48)
"""
from .calculator import TTAtomCalculator
from .weights import WeightBundle

__version__ = "0.1.0"


def Calculator(atoms=None, model="uma-s-1", *, task=None, charge=0, spin=1, refenv=None,
               checkpoint=None, cache_dir=None, device=None, device_id=0, fast=False,
               trace=False, **kw):
    """Family dispatch of the reference (tt_atom/auto.py:40-89). ``model`` (or ``checkpoint``)
    is a path to an exported ``.npz`` weight bundle; its config selects the family: a UMA /
    eSCN-MD bundle gives a ``TTAtomCalculator``, an Orb bundle an ``OrbCalculator``. Building a
    bundle from a released checkpoint needs fairchem / orb-models and network access, which this
    build does not provide."""
    path = checkpoint or model
    import os
    if not (isinstance(path, str) and os.path.exists(path)):
        raise ValueError(
            f"model {model!r}: pass the path of an exported weight bundle (.npz); exporting a "
            "released uma checkpoint needs fairchem, which this build does not include")
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
