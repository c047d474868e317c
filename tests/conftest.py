"""Shared test set-up: import paths, the ``gpu`` marker and golden-fixture loaders."""
import json
import pathlib
import sys

import numpy as np
import pytest
import torch

REPO = pathlib.Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
for p in (str(REPO / "tt-atom_b200"), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


class Fixture:
    """Accessor over a golden npz: config, ``w@`` weights, ``host@`` tables, ``in@``/``out@``."""

    def __init__(self, name):
        self.d = np.load(GOLDEN / name)
        self.config = (json.loads(bytes(self.d["config"]).decode())
                       if "config" in self.d.files else {})

    def has(self, k):
        return k in self.d.files

    def t(self, key):
        return torch.from_numpy(np.ascontiguousarray(self.d[key]))

    def w(self):
        return {k[2:]: self.t(k).float() for k in self.d.files if k.startswith("w@")}

    def tables(self):
        out = {k[5:]: self.t(k).float() for k in self.d.files if k.startswith("host@")
               and k[5:] in ("to_m", "gauss_offset", "gauss_coeff", "to_grid_mat", "from_grid_mat")}
        w = self.w()
        for l in range(3):
            out[f"Jd_{l}"] = w[f"Jd_{l}"]
        return out


@pytest.fixture(scope="session")
def fx():
    cache = {}

    def get(name):
        if name not in cache:
            cache[name] = Fixture(name)
        return cache[name]
    return get


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
