"""Weight bundles: the reference's portable ``.npz`` format (tt_atom/bundle.py:18-37,
tt_atom/weights.py:19-136): an embedded JSON ``config``, ``w@``-prefixed weights, ``host@``
geometry tables and optional ``scale@`` energy normaliser entries. Read-compatible with bundles
the reference exports."""
from __future__ import annotations

import json
import math
import pathlib
from collections import Counter

import numpy as np
import torch


class WeightBundle:
    def __init__(self, npz):
        self._d = npz
        self.config = json.loads(bytes(npz["config"]).decode())

    @classmethod
    def load(cls, path):
        return cls(np.load(pathlib.Path(path)))

    @classmethod
    def from_arrays(cls, arrays):
        return cls(dict(arrays) if not hasattr(arrays, "files") else arrays)

    @property
    def files(self):
        return list(self._d.files) if hasattr(self._d, "files") else list(self._d.keys())

    def has(self, key):
        return key in self.files

    def _t(self, key):
        return torch.from_numpy(np.array(self._d[key], copy=True))

    @property
    def weights(self):
        return {k[2:]: self._t(k).float() for k in self.files if k.startswith("w@")}

    def buffer(self, name):
        return self._t(f"host@{name}").float()

    @property
    def task(self):
        return self.config.get("task", "omat")

    @property
    def scale_rmsd(self):
        return float(self._d["scale@rmsd"][0]) if self.has("scale@rmsd") else 1.0

    @property
    def scale_mean(self):
        return float(self._d["scale@mean"][0]) if self.has("scale@mean") else 0.0

    @property
    def elem_refs(self):
        return self._t("scale@elem_refs").double() if self.has("scale@elem_refs") else None

    @property
    def reference(self):
        """The system a merged bundle was made for and its energy / forces, from the bundle's
        ``ref@`` entries (tt_atom/weights.py:45-59), or None when it carries none (random-init
        bundles)."""
        if not self.has("ref@energy"):
            return None
        arr = lambda k: np.array(self._d[k], copy=True) if self.has(k) else None  # noqa: E731
        return dict(energy=float(self._d["ref@energy"][0]), forces=arr("ref@forces"),
                    pos=arr("ref@pos"), atomic_numbers=arr("ref@atomic_numbers"),
                    charge=float(self._d["ref@charge"][0]), spin=float(self._d["ref@spin"][0]),
                    cell=arr("ref@cell"), pbc=arr("ref@pbc"))

    def tables(self):
        """The fixed geometry tables the engine needs (to_m, grid projections, Gaussian basis)."""
        out = {k: self.buffer(k) for k in ("to_m", "to_grid_mat", "from_grid_mat",
                                           "gauss_offset", "gauss_coeff")}
        return out

    def save(self, path):
        np.savez(path, **{k: np.asarray(self._d[k]) for k in self.files})


def reduced_composition(numbers):
    """Sorted ((Z, count / gcd of all counts), ...): the composition key a merged bundle's expert
    routing depends on, so H2O and H4O2 share it (tt_atom/bundle_cache.py:45-52)."""
    counts = Counter(int(z) for z in numbers)
    g = 0
    for c in counts.values():
        g = math.gcd(g, c)
    return tuple(sorted((z, c // g) for z, c in counts.items()))


def random_bundle(cfg_name="uma-s-1", seed=0):
    """A random-init bundle of a named model shape (see ``tt_atom.configs``)."""
    from . import configs
    cfg = configs.model_config(cfg_name)
    return WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed))
