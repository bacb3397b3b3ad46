"""Host logic of MACECalculator.calculate_batch: how structures become one system."""

import numpy as np
import pytest

from mace_mlx_b200.atoms import Atoms
from mace_mlx_b200.calculators import batch_layout
from mace_mlx_b200.structures import diamond_si


def test_molecules_concatenate_into_graphs():
    a = Atoms([6, 1, 1], [[0, 0, 0], [1.1, 0, 0], [-1.1, 0, 0]])
    b = Atoms([8], [[5, 5, 5]])
    c = Atoms([7, 7], [[0, 0, 0], [0, 0, 1.1]])
    lay = batch_layout([a, b, c])
    np.testing.assert_array_equal(lay["graph_ptr"], [0, 3, 4, 6])
    np.testing.assert_array_equal(lay["numbers"], [6, 1, 1, 8, 7, 7])
    np.testing.assert_array_equal(lay["positions"][3], [5, 5, 5])
    assert lay["cell"] is None and not lay["pbc"].any()
    assert lay["graph_ptr"].dtype == np.int32


def test_periodic_batch_shares_one_cell():
    sts = [diamond_si(2, 0.05, s) for s in (1, 2)]
    atoms = [Atoms(s.numbers, s.positions, s.cell, True) for s in sts]
    lay = batch_layout(atoms)
    np.testing.assert_array_equal(lay["cell"], sts[0].cell)
    assert lay["pbc"].all() and lay["positions"].shape == (128, 3)
    other = diamond_si(3, 0.05, 3)
    with pytest.raises(ValueError, match="another cell"):
        batch_layout(atoms + [Atoms(other.numbers, other.positions, other.cell, True)])
    with pytest.raises(ValueError, match="pbc"):
        batch_layout([atoms[0], Atoms([6], [[0, 0, 0]])])
    with pytest.raises(ValueError, match="at least one"):
        batch_layout([])
