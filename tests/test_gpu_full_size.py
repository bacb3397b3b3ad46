"""BASELINE configurations 2 and 3 at their full sizes, through properties that
do not need the float64 oracle to run at that size.

* c2 (large arch, periodic LiPSO box of 8000 atoms, with stress): rotating
  the box and its atoms rotates forces and stress and leaves energies alone;
  moving a quarter of the atoms by lattice vectors (unwrapped positions, other
  periodic images in the neighbour list) changes nothing; per-atom energies
  sum to the energy and forces to zero.  The same model is compared with the
  oracle on a 300-atom box in ``test_gpu_parity.py``.
* c3 (MACE-OFF-like model, 512 molecules, 20 300 atoms in one batched step):
  every molecule's energy, per-atom energies and forces equal those of the
  molecule evaluated alone, and three molecules are compared with the oracle.

The c3 comparisons use ``helpers.assert_parity`` (BASELINE tolerances plus
relative bounds).  The c2 comparisons set two float32 runs against each other
with their inputs rounded differently (rotated, or moved by up to 51 A), so they
use the BASELINE absolute tolerances (energy 1e-5 eV/atom, forces 1e-4 eV/A,
stress 1e-6 eV/A^3) with a relative bound of 1e-3 of each quantity's scale."""

import numpy as np
import pytest
import torch

from helpers import assert_parity, run_gpu, species_of
from mace_mlx_b200.model import MACEModel
from mace_mlx_b200.spec import ModelSpec
from mace_mlx_b200.structures import Structure, lipso_box, molecule_batch
from mace_mlx_b200.weights import random_config, random_weights
from oracle.model import OracleMACE
from oracle.nl import neighbour_list

pytestmark = pytest.mark.gpu


def assert_baseline(a: dict, b: dict, n_atoms: int):
    de = abs(float(a["energy"][0]) - float(b["energy"][0]))
    assert de / n_atoms < 1e-5, f"energy/atom {de / n_atoms:.3e}"
    dn = np.abs(a["node_energy"] - b["node_energy"]).max()
    assert dn < 1e-3 * np.abs(b["node_energy"]).max(), f"node energy {dn:.3e}"
    df = np.abs(a["forces"] - b["forces"]).max()
    assert df < 1e-4 and df < 1e-3 * np.abs(b["forces"]).max(), f"forces {df:.3e}"
    ds = np.abs(a["stress"] - b["stress"]).max()
    assert ds < 1e-6 and ds < 1e-3 * np.abs(b["stress"]).max(), f"stress {ds:.3e}"


def _voigt_to_matrix(v):
    xx, yy, zz, yz, xz, xy = v
    return np.array([[xx, xy, xz], [xy, yy, yz], [xz, yz, zz]])


def _matrix_to_voigt(m):
    return m[[0, 1, 2, 1, 0, 0], [0, 1, 2, 2, 2, 1]]


@pytest.fixture(scope="module")
def c2_model():
    config = random_config("large", z_table=[3, 8, 15, 16], avg_num_neighbors=50.0)
    m = MACEModel(config=config, weights=random_weights(ModelSpec.from_config(config), seed=2), device=0)
    yield m
    m.close()


@pytest.fixture(scope="module")
def c2_result(c2_model):
    st = lipso_box(8000, 2)
    res, edges, _ = run_gpu(c2_model, st, virial=True)
    return st, res, edges.n_edges


def test_c2_full_size_invariants(c2_model, c2_result):
    st, res, n_edges = c2_result
    assert n_edges > 8000 * 20
    assert c2_model.error_flag() == 0
    np.testing.assert_allclose(res["node_energy"].sum(), res["energy"][0], rtol=1e-6)
    # forces are sums of pair terms with opposite signs: they cancel to rounding
    assert np.abs(res["forces"].sum(0)).max() < 2e-3
    assert np.abs(res["forces"]).max() > 1e-2  # a non-trivial field


def test_c2_full_size_rotation_equivariance(c2_model, c2_result):
    st, res, _ = c2_result
    rng = np.random.default_rng(7)
    q, r = np.linalg.qr(rng.standard_normal((3, 3)))
    R = q * np.sign(np.diag(r))
    if np.linalg.det(R) < 0:
        R[:, 0] = -R[:, 0]
    rot = Structure(st.positions @ R.T, st.numbers.copy(), st.cell @ R.T, st.pbc.copy())
    out, _, _ = run_gpu(c2_model, rot, virial=True)
    back = {
        "energy": out["energy"],
        "node_energy": out["node_energy"],
        "forces": out["forces"] @ R,  # F' = F R^T
        "stress": _matrix_to_voigt(R.T @ _voigt_to_matrix(out["stress"]) @ R),
    }
    assert_baseline(back, res, len(st))


def test_c2_full_size_periodic_images(c2_model, c2_result):
    st, res, n_edges = c2_result
    rng = np.random.default_rng(8)
    moved = rng.random(len(st)) < 0.25
    k = rng.integers(-1, 2, size=(int(moved.sum()), 3))
    pos = st.positions.copy()
    pos[moved] += k @ st.cell
    out, edges, _ = run_gpu(c2_model, Structure(pos, st.numbers.copy(), st.cell.copy(), st.pbc.copy()), virial=True)
    assert edges.n_edges == n_edges
    assert_baseline(out, res, len(st))


@pytest.fixture(scope="module")
def c3_case():
    config = random_config("medium", hidden_irreps="96x0e + 96x1o", r_max=5.0, z_table=[1, 6, 7, 8],
                           avg_num_neighbors=12.0)
    weights = random_weights(ModelSpec.from_config(config), seed=3)
    m = MACEModel(config=config, weights=weights, device=0)
    yield config, weights, m, molecule_batch(512, 3)
    m.close()


def _molecule(st: Structure, g: int) -> Structure:
    sel = st.batch == g
    return Structure(st.positions[sel].copy(), st.numbers[sel].copy())


def test_c3_full_size_batch_equals_molecules_alone(c3_case):
    config, weights, m, st = c3_case
    assert st.num_graphs == 512 and len(st) > 20000
    res, _, _ = run_gpu(m, st, virial=False)
    assert res["energy"].shape == (512,)
    assert m.error_flag() == 0
    for g in range(st.num_graphs):
        sel = st.batch == g
        alone, _, _ = run_gpu(m, _molecule(st, g), virial=False)
        part = {"energy": res["energy"][g:g + 1], "node_energy": res["node_energy"][sel], "forces": res["forces"][sel]}
        assert_parity(part, alone, int(sel.sum()))
    for g in (0, 255, 511):
        mol = _molecule(st, g)
        i, j, S = neighbour_list(mol.positions, mol.cell, mol.pbc, config["r_max"])
        ref = OracleMACE(config, weights).compute(mol.positions, species_of(mol.numbers, config["z_table"]),
                                                  i, j, S)
        sel = st.batch == g
        part = {"energy": res["energy"][g:g + 1], "node_energy": res["node_energy"][sel], "forces": res["forces"][sel]}
        assert_parity(part, ref, len(mol))
    torch.cuda.synchronize()
