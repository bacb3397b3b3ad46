"""Minimal ASE-compatible ``Atoms`` / ``Calculator`` stand-ins.

The calculator is a drop-in for ASE code: when ``ase`` is importable it
subclasses ``ase.calculators.calculator.Calculator`` and works with
``ase.Atoms``.  When ASE is absent (as on the build and GPU images), these
small classes provide the subset of the API the calculator and its users
need: positions, numbers, cell, pbc, ``calc`` and the ``get_*`` accessors.
"""

from __future__ import annotations

import numpy as np

try:  # pragma: no cover - exercised only where ASE is installed
    from ase.calculators.calculator import Calculator as _ASECalculator
    from ase.calculators.calculator import all_changes as _ase_all_changes

    HAVE_ASE = True
except Exception:  # noqa: BLE001
    _ASECalculator = None
    _ase_all_changes = None
    HAVE_ASE = False


class Cell:
    def __init__(self, array):
        self.array = np.zeros((3, 3)) if array is None else np.array(array, dtype=np.float64).reshape(3, 3)

    @property
    def rank(self) -> int:
        """Number of non-zero cell vectors (ASE's definition)."""
        return int(self.array.any(1).sum())

    def __array__(self, dtype=None, copy=None):
        return self.array.astype(dtype) if dtype is not None else self.array

    def volume(self) -> float:
        return abs(float(np.linalg.det(self.array)))


class Atoms:
    """Tiny subset of ``ase.Atoms``."""

    def __init__(self, numbers=None, positions=None, cell=None, pbc=False, symbols=None):
        self.numbers = np.asarray(numbers, dtype=np.int64)
        self.positions = np.array(positions, dtype=np.float64).reshape(-1, 3)
        self.cell = Cell(cell)
        p = np.asarray(pbc, dtype=bool)
        self.pbc = np.repeat(p, 3) if p.ndim == 0 else p.copy()
        self.calc = None

    def __len__(self) -> int:
        return len(self.numbers)

    def copy(self) -> "Atoms":
        a = Atoms(self.numbers.copy(), self.positions.copy(), self.cell.array.copy(), self.pbc.copy())
        return a

    def get_positions(self) -> np.ndarray:
        return self.positions.copy()

    def set_positions(self, pos) -> None:
        self.positions = np.array(pos, dtype=np.float64).reshape(-1, 3)

    def get_atomic_numbers(self) -> np.ndarray:
        return self.numbers.copy()

    def get_cell(self) -> np.ndarray:
        return self.cell.array.copy()

    def set_cell(self, cell, scale_atoms: bool = False) -> None:
        new = np.array(cell, dtype=np.float64).reshape(3, 3)
        if scale_atoms and self.cell.rank == 3:
            frac = self.positions @ np.linalg.inv(self.cell.array)
            self.positions = frac @ new
        self.cell = Cell(new)

    def get_volume(self) -> float:
        return self.cell.volume()

    def _calc(self):
        if self.calc is None:
            raise RuntimeError("Atoms object has no calculator.")
        return self.calc

    def get_potential_energy(self) -> float:
        return self._calc().get_potential_energy(self)

    def get_forces(self) -> np.ndarray:
        return self._calc().get_forces(self)

    def get_stress(self) -> np.ndarray:
        return self._calc().get_stress(self)

    def get_potential_energies(self) -> np.ndarray:
        return self._calc().get_property("energies", self)


all_changes = _ase_all_changes or ["positions", "numbers", "cell", "pbc", "initial_charges", "initial_magmoms"]


class _MiniCalculator:
    """Subset of ``ase.calculators.calculator.Calculator`` semantics."""

    implemented_properties: list[str] = []

    def __init__(self, **kwargs):
        self.results: dict = {}
        self.atoms = None
        self.parameters = dict(kwargs)

    def _changed(self, atoms) -> bool:
        if self.atoms is None:
            return True
        a = self.atoms
        return (
            len(a) != len(atoms)
            or not np.array_equal(a.numbers, atoms.numbers)
            or not np.array_equal(a.positions, atoms.positions)
            or not np.array_equal(np.asarray(a.cell), np.asarray(atoms.cell))
            or not np.array_equal(a.pbc, atoms.pbc)
        )

    def calculate(self, atoms=None, properties=None, system_changes=all_changes):
        if atoms is not None:
            self.atoms = atoms.copy()

    def get_property(self, name, atoms=None, allow_calculation=True):
        if name not in self.implemented_properties:
            raise NotImplementedError(f"{name} property not implemented")
        if atoms is None:
            atoms = self.atoms
        if self._changed(atoms):
            self.results = {}
        if name not in self.results:
            if not allow_calculation:
                return None
            self.calculate(atoms, [name], all_changes)
        if name not in self.results:
            raise NotImplementedError(f"{name} not present in this calculation")
        r = self.results[name]
        return r.copy() if isinstance(r, np.ndarray) else r

    def get_potential_energy(self, atoms=None, force_consistent=False):
        return self.get_property("free_energy" if force_consistent else "energy", atoms)

    def get_forces(self, atoms=None):
        return self.get_property("forces", atoms)

    def get_stress(self, atoms=None):
        return self.get_property("stress", atoms)


Calculator = _ASECalculator if HAVE_ASE else _MiniCalculator
