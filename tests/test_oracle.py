"""The CPU oracle itself: known answers and physical invariants.

Ports of the reference's own specification tests (paths in the reference):
Bessel values by formula (tests/test_radial.py:36-52), envelope boundary values
(:79-122), SH l=1 ordering and component norm (tests/test_spherical_harmonics.py:
84-160), zero vector (:276-286), forces by finite differences, sum of forces,
translation invariance (tests/test_forces.py:39-226), stress symmetry, stress by
finite differences, and stress-path forces == energy-path forces
(tests/test_stress.py:118-256)."""

import math

import numpy as np
import pytest
import torch

from helpers import make_case
from mace_mlx_b200.structures import diamond_si
from oracle.model import OracleMACE
from oracle.nl import neighbour_list

torch.set_num_threads(4)


@pytest.fixture(scope="module")
def small_case():
    config, weights, st = make_case("small", diamond_si(2, 0.05, 3), seed=3)
    orc = OracleMACE(config, weights)
    i, j, S = neighbour_list(st.positions, st.cell, st.pbc, 6.0)
    return orc, st, (i, j, S)


def test_bessel_known_values():
    config, weights, _ = make_case("small")
    orc = OracleMACE(config, weights)
    r = torch.tensor([[1.0], [2.0], [3.0]], dtype=torch.float64)
    b = orc.radial(r).numpy()
    pref = math.sqrt(2.0 / 6.0)
    p = 5
    for i, x in enumerate([1.0, 2.0, 3.0]):
        u = x / 6.0
        env = 1 - (p + 1) * (p + 2) / 2 * u ** p + p * (p + 2) * u ** (p + 1) - p * (p + 1) / 2 * u ** (p + 2)
        for n in range(8):
            w = (n + 1) * math.pi / 6.0
            # the converted layout stores the Bessel frequencies in float32
            assert b[i, n] == pytest.approx(pref * math.sin(w * x) / x * env, rel=1e-6, abs=1e-6)


def test_envelope_boundaries():
    config, weights, _ = make_case("small")
    orc = OracleMACE(config, weights)
    r = torch.tensor([[1e-9], [6.0], [7.0], [100.0]], dtype=torch.float64)
    b = orc.radial(r).numpy()
    assert np.all(b[1:] == 0.0)
    assert np.all(np.isfinite(b))


def test_sh_l1_and_component_norm():
    config, weights, _ = make_case("small")
    orc = OracleMACE(config, weights)
    rng = np.random.default_rng(0)
    v = rng.normal(size=(200, 3))
    Y = orc.spherical_harmonics(torch.tensor(v)).numpy()
    u = v / np.linalg.norm(v, axis=1, keepdims=True)
    np.testing.assert_allclose(Y[:, 0], 1.0)
    np.testing.assert_allclose(Y[:, 1:4], math.sqrt(3) * u, atol=1e-12)  # e3nn basis: (x, y, z)
    for l in range(4):
        np.testing.assert_allclose((Y[:, l * l:(l + 1) ** 2] ** 2).sum(1), 2 * l + 1, rtol=1e-10)
    Y0 = orc.spherical_harmonics(torch.zeros(1, 3, dtype=torch.float64)).numpy()
    assert np.all(np.isfinite(Y0))


def test_neighbour_list_closed_under_reversal(small_case):
    orc, st, (i, j, S) = small_case
    fwd = set(zip(i.tolist(), j.tolist(), map(tuple, S.tolist())))
    rev = set(zip(j.tolist(), i.tolist(), map(tuple, (-S).tolist())))
    assert fwd == rev
    v = st.positions[j] - st.positions[i] + S @ st.cell
    assert np.all(np.linalg.norm(v, axis=1) < 6.0)
    assert not np.any((i == j) & np.all(S == 0, axis=1))


def test_forces_sum_to_zero_and_match_finite_differences(small_case):
    orc, st, (i, j, S) = small_case
    sp = st.numbers - 1
    out = orc.compute(st.positions, sp, i, j, S, st.cell)
    np.testing.assert_allclose(out["forces"].sum(0), 0.0, atol=1e-12)
    h = 1e-5
    for a, c in [(0, 0), (5, 1), (17, 2)]:
        p = st.positions.copy()
        p[a, c] += h
        ep = orc.compute(p, sp, i, j, S, st.cell)["energy"][0]
        p[a, c] -= 2 * h
        em = orc.compute(p, sp, i, j, S, st.cell)["energy"][0]
        assert -(ep - em) / (2 * h) == pytest.approx(out["forces"][a, c], rel=1e-5, abs=1e-9)


def test_translation_and_rotation_invariance(small_case):
    orc, st, (i, j, S) = small_case
    sp = st.numbers - 1
    base = orc.compute(st.positions, sp, i, j, S, st.cell)
    shifted = orc.compute(st.positions + np.array([0.3, -1.1, 2.2]), sp, i, j, S, st.cell)
    assert shifted["energy"][0] == pytest.approx(base["energy"][0], abs=1e-10)
    np.testing.assert_allclose(shifted["forces"], base["forces"], atol=1e-10)
    th = 0.7
    R = np.array([[math.cos(th), -math.sin(th), 0], [math.sin(th), math.cos(th), 0], [0, 0, 1]])
    rot = orc.compute(st.positions @ R.T, sp, i, j, S, st.cell @ R.T)
    assert rot["energy"][0] == pytest.approx(base["energy"][0], abs=1e-10)
    np.testing.assert_allclose(rot["forces"], base["forces"] @ R.T, atol=1e-10)


def test_stress_symmetric_finite_difference_and_force_path(small_case):
    orc, st, (i, j, S) = small_case
    sp = st.numbers - 1
    out = orc.compute(st.positions, sp, i, j, S, st.cell, stress=True)
    ref = orc.compute(st.positions, sp, i, j, S, st.cell)
    np.testing.assert_allclose(out["forces"], ref["forces"], atol=1e-12)
    # finite-difference stress: sigma_xx = dE/de_xx / V
    eps = 1e-5
    vol = abs(np.linalg.det(st.cell))
    for a, (r, c) in enumerate([(0, 0), (1, 1), (2, 2), (1, 2), (0, 2), (0, 1)]):
        e = np.zeros((3, 3))
        e[r, c] = e[c, r] = eps if r != c else eps
        f = np.eye(3) + (e if r == c else e / 2)
        ep = orc.compute(st.positions @ f, sp, i, j, S, st.cell @ f)["energy"][0]
        fm = np.eye(3) - (e if r == c else e / 2)
        em = orc.compute(st.positions @ fm, sp, i, j, S, st.cell @ fm)["energy"][0]
        fd = (ep - em) / (2 * eps) / vol
        assert fd == pytest.approx(out["stress"][a], rel=1e-4, abs=1e-9)
