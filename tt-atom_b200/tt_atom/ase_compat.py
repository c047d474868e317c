"""ASE calculator base: ASE's own ``Calculator`` when ASE is installed, else a minimal stand-in
with the same ``results`` / ``calculate`` / ``get_*`` surface (duck-typed ``Atoms``: positions,
numbers, cell, pbc, info, volume)."""
from __future__ import annotations

import numpy as np

try:  # pragma: no cover - depends on the environment
    from ase.calculators.calculator import Calculator as _AseCalculator
    from ase.calculators.calculator import all_changes
    HAVE_ASE = True
except ImportError:  # ASE is optional
    HAVE_ASE = False
    all_changes = ("positions", "numbers", "cell", "pbc")

    class _AseCalculator:
        implemented_properties: list = []

        def __init__(self, **kwargs):
            self.results = {}
            self.atoms = None

        def calculate(self, atoms=None, properties=("energy",), system_changes=all_changes):
            self.atoms = atoms
            self.results = {}

        def get_property(self, name, atoms):
            self.calculate(atoms, (name,))
            return self.results[name]

        def get_potential_energy(self, atoms=None, force_consistent=False):
            return self.get_property("energy", atoms)

        def get_forces(self, atoms=None):
            return self.get_property("forces", atoms)

        def get_stress(self, atoms=None):
            return self.get_property("stress", atoms)


def voigt_6(s):
    """3x3 -> Voigt (xx, yy, zz, yz, xz, xy), symmetrised, as ASE's full_3x3_to_voigt_6_stress."""
    s = np.asarray(s, dtype=np.float64)
    return np.array([s[0, 0], s[1, 1], s[2, 2], 0.5 * (s[1, 2] + s[2, 1]),
                     0.5 * (s[0, 2] + s[2, 0]), 0.5 * (s[0, 1] + s[1, 0])])


def atoms_volume(atoms):
    if hasattr(atoms, "get_volume"):
        return float(atoms.get_volume())
    return float(abs(np.linalg.det(np.asarray(atoms.get_cell(), dtype=np.float64))))


class SimpleAtoms:
    """Minimal ``Atoms`` stand-in (positions, numbers, cell, pbc, info) for environments
    without ASE."""

    def __init__(self, numbers, positions, cell=None, pbc=False, info=None):
        self.numbers = np.asarray(numbers, dtype=np.int64)
        self.positions = np.asarray(positions, dtype=np.float64)
        self.cell = np.zeros((3, 3)) if cell is None else np.asarray(cell, dtype=np.float64)
        self.pbc = np.array([bool(pbc)] * 3) if np.isscalar(pbc) else np.asarray(pbc, dtype=bool)
        self.info = dict(info or {})
        self.calc = None

    def __len__(self):
        return len(self.numbers)

    def get_positions(self):
        return self.positions.copy()

    def set_positions(self, p):
        self.positions = np.asarray(p, dtype=np.float64)

    def get_atomic_numbers(self):
        return self.numbers.copy()

    def get_cell(self):
        return self.cell.copy()

    def get_pbc(self):
        return self.pbc.copy()

    def get_volume(self):
        return float(abs(np.linalg.det(self.cell)))

    def get_potential_energy(self):
        return self.calc.get_potential_energy(self)

    def get_forces(self):
        return self.calc.get_forces(self)

    def get_stress(self):
        return self.calc.get_stress(self)
