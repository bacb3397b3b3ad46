"""GPU neighbour list against the numpy oracle: the edge set must be bit-exact
(as sets of (sender, receiver, shift)), sorted by (receiver, sender, S), with a
consistent CSR row pointer and reverse-edge map."""

import dataclasses

import numpy as np
import pytest
import torch

from helpers import graph_ptr_of, make_case
from mace_mlx_b200.model import MACEModel
from mace_mlx_b200.structures import Structure, diamond_si, lipso_box, molecule_batch
from oracle.nl import min_gap_to_cutoff, neighbour_list

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    config, weights, _ = make_case("small")
    return MACEModel(config=config, weights=weights, device=0)


def gpu_nl(model, st, r_cut, cap=None):
    dev = model.device
    gp = torch.as_tensor(graph_ptr_of(st), device=dev)
    pos = torch.tensor(st.positions, dtype=torch.float64, device=dev)
    periodic = bool(np.any(st.pbc))
    cell = torch.tensor(st.cell, dtype=torch.float64, device=dev) if periodic else None
    return model.neighbour_list(pos, cell, st.pbc, gp, r_cut)


def check_edges(model, st, r_cut):
    e = gpu_nl(model, st, r_cut)
    s, r, S = e.numpy()
    i, j, So = neighbour_list(st.positions, st.cell, st.pbc, r_cut, batch=st.batch)
    if len(i):
        assert min_gap_to_cutoff(st.positions, st.cell, i, j, So, r_cut) > 1e-9
    assert set(zip(s.tolist(), r.tolist(), map(tuple, S.tolist()))) == \
        set(zip(i.tolist(), j.tolist(), map(tuple, So.tolist())))
    assert len(s) == len(i)
    # sorted by (receiver, sender, S) and CSR over receivers
    key = np.lexsort((S[:, 2], S[:, 1], S[:, 0], s, r))
    np.testing.assert_array_equal(key, np.arange(len(s)))
    rp = e.row_ptr.cpu().numpy()
    np.testing.assert_array_equal(rp, np.concatenate([[0], np.cumsum(np.bincount(r, minlength=len(st)))]))
    rev = e.rev[: e.n_edges].cpu().numpy()
    if len(s):
        np.testing.assert_array_equal(s[rev], r)
        np.testing.assert_array_equal(r[rev], s)
        np.testing.assert_array_equal(S[rev], -S)
    return e


@pytest.mark.parametrize("reps,sigma,seed,r_cut", [(3, 0.01, 0, 6.0), (5, 0.05, 1, 6.0), (5, 0.05, 1, 6.5)])
def test_diamond_configs(model, reps, sigma, seed, r_cut):
    check_edges(model, diamond_si(reps, sigma, seed), r_cut)


def test_small_cell_with_self_images(model):
    st = diamond_si(1, 0.02, 5)  # 5.43 A cell, cutoff 6 A: every atom sees its own images
    e = check_edges(model, st, 6.0)
    s, r, S = e.numpy()
    assert np.any(s == r)


def test_triclinic_and_wrapped_positions(model):
    st = diamond_si(2, 0.05, 6)
    cell = st.cell.copy()
    cell[1, 0] = 3.1
    cell[2, 1] = -2.2
    frac = st.positions @ np.linalg.inv(st.cell)
    pos = frac @ cell
    pos[::3] += cell[0] * 2 - cell[2]  # atoms far outside the cell
    check_edges(model, Structure(pos, st.numbers, cell, np.ones(3, bool)), 6.0)


def test_slab_mixed_pbc(model):
    st = diamond_si(2, 0.05, 7)
    st = Structure(st.positions, st.numbers, st.cell, np.array([True, True, False]))
    check_edges(model, st, 6.0)


def test_molecule_batch_no_cross_graph_edges(model):
    st = molecule_batch(6, 3)
    e = check_edges(model, st, 5.0)
    s, r, _ = e.numpy()
    assert np.all(st.batch[s] == st.batch[r])


def test_lipso_box_subset(model):
    st = lipso_box(600, 2)
    check_edges(model, st, 6.0)


def test_isolated_atoms_have_no_edges(model):
    st = Structure(np.array([[0.0, 0, 0], [10.0, 0, 0], [0, 20.0, 0]]), np.array([14, 14, 14]))
    e = check_edges(model, st, 5.0)
    assert e.n_edges == 0


def test_capacity_overflow_is_retried(model):
    st = diamond_si(3, 0.01, 0)
    dev = model.device
    gp = torch.as_tensor(graph_ptr_of(st), device=dev)
    pos = torch.tensor(st.positions, dtype=torch.float64, device=dev)
    cell = torch.tensor(st.cell, dtype=torch.float64, device=dev)
    from mace_mlx_b200.model import EdgeSet

    i32 = dict(dtype=torch.int32, device=dev)
    tiny = EdgeSet(torch.empty(16, **i32), torch.empty(16, **i32), torch.empty(16, 3, **i32),
                   torch.empty(len(st) + 1, **i32), torch.empty(16, **i32), 0)
    e = model.neighbour_list(pos, cell, st.pbc, gp, 6.0, tiny)
    i, _, _ = neighbour_list(st.positions, st.cell, st.pbc, 6.0)
    assert e.n_edges == len(i)


def _sheared(st: Structure, shear: float) -> Structure:
    M = np.eye(3)
    M[1, 0] = shear
    M[2, 1] = 0.5 * shear
    return dataclasses.replace(st, positions=st.positions @ M, cell=st.cell @ M)


@pytest.mark.parametrize("case", ["periodic", "periodic_r65", "triclinic", "wrapped", "open_cluster", "slab",
                                  "wire"])
def test_cell_list_against_oracle(model, monkeypatch, case):
    """Cell lists forced on (threshold 1 atom): bit-exact edge set against the oracle."""
    monkeypatch.setenv("MACE_B200_NL_CELL_MIN", "1")
    st, r = diamond_si(5, 0.05, 11), 6.0
    if case == "periodic_r65":
        r = 6.5
    elif case == "triclinic":
        st = _sheared(st, 0.3)
    elif case == "wrapped":
        rng = np.random.default_rng(5)
        k = rng.integers(-2, 3, size=(len(st), 3))
        st = dataclasses.replace(st, positions=st.positions + k @ st.cell)
    elif case == "open_cluster":
        st = dataclasses.replace(st, pbc=np.zeros(3, dtype=bool))
    elif case == "slab":  # periodic in x, y; open in z (a domain of a split along z)
        st = dataclasses.replace(_sheared(st, 0.2), pbc=np.array([True, True, False]))
    elif case == "wire":
        st = dataclasses.replace(st, pbc=np.array([True, False, False]))
    check_edges(model, st, r)


@pytest.mark.parametrize("pbc", [(True, True, True), (False, False, False), (True, True, False)])
def test_cell_list_equals_all_pairs_on_large_systems(model, monkeypatch, pbc):
    """4096 atoms (cell lists by default) against the all-pairs kernels, array for array."""
    st = dataclasses.replace(diamond_si(8, 0.05, 12), pbc=np.array(pbc))
    a = gpu_nl(model, st, 6.0)
    monkeypatch.setenv("MACE_B200_NL_ALL_PAIRS", "1")
    b = gpu_nl(model, st, 6.0)
    assert a.n_edges == b.n_edges > 30 * len(st) * (1 if pbc[0] else 0.5)
    for x, y in zip(a.numpy(), b.numpy()):
        np.testing.assert_array_equal(x, y)
    np.testing.assert_array_equal(a.row_ptr.cpu().numpy(), b.row_ptr.cpu().numpy())
    np.testing.assert_array_equal(a.rev[: a.n_edges].cpu().numpy(), b.rev[: b.n_edges].cpu().numpy())
