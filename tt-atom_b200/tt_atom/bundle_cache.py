"""Where exported weight bundles are cached, under the reference's cache layout, so bundles that
the reference's tools exported are found by name.

UMA: a merged bundle is valid for one (model, task, reduced composition, charge, spin), stored as
``{model}_{task}_{composition hash}_c{charge}_s{spin}[_ckpt{hash}].npz`` in ``$TT_ATOM_CACHE``
(default ``~/.cache/tt_atom/bundles``) (tt_atom/bundle_cache.py:25-80). Orb: one file per
checkpoint, ``{name without "orb-v3-"}.npz`` in ``$TT_ATOM_CACHE/orb_weights`` (default
``~/.cache/tt_atom/orb_weights``) (tt_atom/orb_weight_cache.py:19-35).

A cache hit is a plain load. Building a missing bundle needs the reference environment
(fairchem / orb-models and their checkpoints), which this build does not include: a miss raises
with the path it looked for.
"""
from __future__ import annotations

import hashlib
import os
import pathlib

import numpy as np

from .weights import reduced_composition

ORB_CHECKPOINTS = ("orb-v3-conservative-inf-omat", "orb-v3-direct-20-omat",
                   "orb-v3-conservative-omol", "orb-v3-direct-omol")


def _uma_dir(cache_dir=None):
    if cache_dir is not None:
        return pathlib.Path(cache_dir)
    env = os.environ.get("TT_ATOM_CACHE")
    return pathlib.Path(env) if env else pathlib.Path.home() / ".cache" / "tt_atom" / "bundles"


def _orb_dir(cache_dir=None):
    if cache_dir is not None:
        return pathlib.Path(cache_dir)
    env = os.environ.get("TT_ATOM_CACHE")
    root = pathlib.Path(env) if env else pathlib.Path.home() / ".cache" / "tt_atom"
    return root / "orb_weights"


def infer_task(atoms):
    """Default UMA task: 'omat' for a fully periodic cell, else 'omol'."""
    return "omat" if np.asarray(atoms.get_pbc()).all() else "omol"


def composition_hash(numbers):
    """First 12 hex digits of the SHA-1 of the reduced composition written as 'Z:count;...'."""
    key = ";".join(f"{z}:{c}" for z, c in reduced_composition(numbers))
    return hashlib.sha1(key.encode()).hexdigest()[:12]


def bundle_path(model, task, numbers, charge, spin, cache_dir=None, checkpoint=None):
    """Cache path of the merged UMA bundle for this system; an explicit raw checkpoint gets its
    own namespace (hash of its resolved path)."""
    suffix = ""
    if checkpoint is not None:
        ident = str(pathlib.Path(checkpoint).expanduser().resolve())
        suffix = f"_ckpt{hashlib.sha1(ident.encode()).hexdigest()[:12]}"
    name = (f"{model}_{task}_{composition_hash(numbers)}_c{int(charge)}_s{int(spin)}"
            f"{suffix}.npz")
    return _uma_dir(cache_dir) / name


def orb_weights_path(checkpoint, cache_dir=None):
    if checkpoint not in ORB_CHECKPOINTS:
        raise ValueError(f"unknown Orb checkpoint {checkpoint!r}; choose from {ORB_CHECKPOINTS}")
    return _orb_dir(cache_dir) / f"{checkpoint[len('orb-v3-'):]}.npz"


def cached(path, what):
    """``path`` when the bundle is there; otherwise a RuntimeError naming it."""
    path = pathlib.Path(path)
    if path.exists():
        return path
    raise RuntimeError(
        f"no cached {what} at {path}. Building it needs the reference environment (fairchem / "
        "orb-models and the released checkpoint), which this build does not include: export the "
        "bundle with the reference's tools into that path, or pass a bundle .npz directly.")
