"""Regenerate ``lmax2_tables.npz``: the fixed lmax=mmax=2 geometry tables of the eSCN-MD model.

These are model constants, not learned weights: the e3nn Wigner ``J`` matrices ``Jd_0..2``, the
m-primed coefficient permutation ``to_m`` and the SO(3) grid projections ``to_grid_mat`` /
``from_grid_mat`` (6x7 sphere points x 9 coefficients). Real weight bundles carry their own copy
(tt_atom/weights.py:19-136 in the reference reads them as ``host@`` / ``w@Jd_*`` keys); the
random-init bundles used for synthetic benchmarks take them from this file.

The values are read out of the reference's committed golden fixture
(tests/data/golden_tiny.npz, produced by fairchem's eSCNMDBackbone), so that this framework uses
exactly the tables the reference's parity tests were generated with. The table ships inside
the package (tt-atom_b200/tt_atom/data/lmax2_tables.npz); this generator is test
infrastructure and lives beside the other fixture generators. Usage:

    python tests/golden/make_tables.py <reference_root>
"""
import pathlib
import sys

import numpy as np


def main(ref_root):
    z = np.load(pathlib.Path(ref_root) / "tests" / "data" / "golden_tiny.npz")
    out = {f"Jd_{l}": z[f"w@Jd_{l}"].astype(np.float32) for l in range(3)}
    for k in ("to_m", "to_grid_mat", "from_grid_mat"):
        out[k] = z[f"host@{k}"].astype(np.float32)
    dst = (pathlib.Path(__file__).resolve().parents[2] / "tt-atom_b200" / "tt_atom" / "data"
           / "lmax2_tables.npz")
    np.savez(dst, **out)
    print("wrote", dst, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_tables.py <reference_root>")
    main(sys.argv[1])
