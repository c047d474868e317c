"""Weight bundles: the reference's portable ``.npz`` format (tt_atom/bundle.py:18-37,
tt_atom/weights.py:19-136): an embedded JSON ``config``, ``w@``-prefixed weights, ``host@``
geometry tables and optional ``scale@`` energy normaliser entries. Read-compatible with bundles
the reference exports."""
from __future__ import annotations

import json
import pathlib

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
        return None

    def tables(self):
        """The fixed geometry tables the engine needs (to_m, grid projections, Gaussian basis)."""
        out = {k: self.buffer(k) for k in ("to_m", "to_grid_mat", "from_grid_mat",
                                           "gauss_offset", "gauss_coeff")}
        return out

    def save(self, path):
        np.savez(path, **{k: np.asarray(self._d[k]) for k in self.files})


def random_bundle(cfg_name="uma-s-1", seed=0):
    """A random-init bundle of a named model shape (see ``tt_atom.configs``)."""
    from . import configs
    cfg = configs.model_config(cfg_name)
    return WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed))
