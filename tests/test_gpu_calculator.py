"""The ASE-facing calculator (reference calculators.py behaviour) on the GPU."""

import warnings

import numpy as np
import pytest

from helpers import assert_parity
from mace_mlx_b200.atoms import Atoms
from mace_mlx_b200.calculators import MACECalculator, mace_mp, mace_off
from mace_mlx_b200.structures import diamond_si
from mace_mlx_b200.weights import write_random_model
from oracle.model import OracleMACE
from oracle.nl import neighbour_list

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    return str(write_random_model(tmp_path_factory.mktemp("m") / "medium", "medium", seed=21,
                                  z_table=list(range(1, 90)), avg_num_neighbors=40.0))


def test_energy_forces_stress_match_oracle(model_dir):
    st = diamond_si(2, 0.05, 21)
    atoms = Atoms(st.numbers, st.positions, st.cell, True)
    calc = MACECalculator(model_path=model_dir, device="cuda", skin=0.0)
    atoms.calc = calc
    e = atoms.get_potential_energy()
    f = atoms.get_forces()
    s = atoms.get_stress()
    from mace_mlx_b200.weights import load_model_dir

    config, weights = load_model_dir(model_dir)
    i, j, S = neighbour_list(st.positions, st.cell, st.pbc, 6.0)
    ref = OracleMACE(config, weights).compute(st.positions, st.numbers - 1, i, j, S, st.cell, stress=True)
    gpu = {"energy": np.array([e]), "forces": f.astype(np.float64), "stress": s,
           "node_energy": calc.results["node_energy"]}
    assert_parity(gpu, ref, len(st), stress=True)
    assert set(calc.results) >= {"energy", "free_energy", "forces", "stress", "node_energy", "energies"}


def test_skin_cache_rebuild_rule(model_dir):
    st = diamond_si(2, 0.05, 22)
    atoms = Atoms(st.numbers, st.positions, st.cell, True)
    calc = MACECalculator(model_path=model_dir, skin=0.5)
    calc.calculate(atoms, ["energy", "forces"])
    nl0 = calc._nl_cache
    atoms.positions = atoms.positions + 0.1  # 0.17 A < skin / 2: cached list reused
    calc.calculate(atoms, ["energy", "forces"])
    assert calc._nl_cache is nl0
    f_cached = calc.results["forces"].copy()
    # the cached (r_max + skin) list gives the same physics as a fresh list
    fresh = MACECalculator(model_path=model_dir, skin=0.0)
    fresh.calculate(atoms, ["energy", "forces"])
    np.testing.assert_allclose(f_cached, fresh.results["forces"], atol=1e-5 * np.abs(f_cached).max() + 1e-8)
    p = atoms.positions.copy()
    p[0] += 0.3  # > skin / 2: rebuilt
    atoms.positions = p
    calc.calculate(atoms, ["energy", "forces"])
    assert calc._nl_cache is not None


def test_sticky_stress_and_molecules_without_stress(model_dir):
    st = diamond_si(2, 0.05, 23)
    atoms = Atoms(st.numbers, st.positions, st.cell, True)
    calc = MACECalculator(model_path=model_dir)
    calc.calculate(atoms, ["stress"])
    assert "stress" in calc.results
    calc.calculate(atoms, ["energy"])
    assert "stress" in calc.results  # sticky after an explicit stress request
    mol = Atoms([6, 8, 1], [[0, 0, 0], [1.2, 0, 0], [-0.6, 0.9, 0]])
    calc2 = MACECalculator(model_path=model_dir)
    calc2.calculate(mol, ["energy", "forces", "stress"])
    assert "stress" not in calc2.results
    assert calc2.results["forces"].shape == (3, 3)
    assert abs(calc2.results["forces"].sum(0)).max() < 1e-5


def test_unsupported_species_message(model_dir):
    from mace_mlx_b200.weights import load_model_dir, write_model_dir

    config, weights = load_model_dir(model_dir)
    config = dict(config, z_table=list(range(1, 90)))
    calc = MACECalculator(model_path=model_dir)
    atoms = Atoms([14, 118], [[0, 0, 0], [2, 0, 0]])
    with pytest.raises(ValueError, match="Atomic number 118 .*not supported"):
        calc.calculate(atoms, ["energy"])


def test_api_errors(model_dir, tmp_path, monkeypatch):
    with pytest.raises(NotImplementedError, match="committee"):
        MACECalculator(model_paths=[model_dir, model_dir])
    with pytest.raises(ValueError, match="cpu"):
        MACECalculator(model_path=model_dir, device="cpu")
    with pytest.warns(UserWarning, match="float64"):
        MACECalculator(model_path=model_dir, default_dtype="float64")
    monkeypatch.setenv("MACE_MLX_CACHE_DIR", str(tmp_path))
    with pytest.raises(FileNotFoundError, match="converted-model cache"):
        mace_mp("small")
    with pytest.raises(FileNotFoundError):
        mace_off("medium")
    with pytest.raises(NotImplementedError):
        mace_mp(model_dir, return_raw_model=True)
    # a cached named model resolves through the cache layout <root>/<name>/v2
    import shutil

    shutil.copytree(model_dir, tmp_path / "small" / "v2")
    calc = mace_mp("small")
    assert calc.model.spec.C == 128


def test_calculate_batch_matches_one_structure_at_a_time(model_dir):
    """One batched step (structures as graphs of one system) equals separate steps,
    and each structure's energy and forces equal the float64 oracle on it alone:
    a periodic batch of perturbed replicas of one cell and a molecule batch."""
    from mace_mlx_b200.structures import molecule_batch
    from mace_mlx_b200.weights import load_model_dir

    config, weights = load_model_dir(model_dir)
    orc = OracleMACE(config, weights)
    calc = MACECalculator(model_path=model_dir, device="cuda", skin=0.0)
    sts = [diamond_si(2, 0.05, s) for s in (31, 32, 33)]
    periodic = [Atoms(s.numbers, s.positions, s.cell, True) for s in sts]
    mols = molecule_batch(3, 7)
    bounds = np.concatenate([[0], np.cumsum(np.bincount(mols.batch))])
    molecules = [Atoms(mols.numbers[a:b], mols.positions[a:b]) for a, b in zip(bounds[:-1], bounds[1:])]
    for batch in (periodic, molecules):
        got = calc.calculate_batch(batch)
        assert len(got) == len(batch)
        for atoms, r in zip(batch, got):
            calc.calculate(atoms, ["energy", "forces"])
            ref = calc.results
            assert abs(r["energy"] - ref["energy"]) <= 1e-6 * max(1.0, abs(ref["energy"])) + 1e-7 * len(atoms)
            np.testing.assert_allclose(r["forces"], ref["forces"], atol=1e-5 * max(1.0, np.abs(ref["forces"]).max()))
            np.testing.assert_allclose(r["node_energy"], ref["node_energy"], atol=1e-6)
            i, j, S = neighbour_list(atoms.positions, atoms.get_cell(), atoms.pbc, 6.0)
            want = orc.compute(atoms.positions, atoms.numbers - 1, i, j, S,
                               atoms.get_cell() if np.any(atoms.pbc) else None)
            mine = {"energy": np.array([r["energy"]]), "forces": np.asarray(r["forces"], np.float64),
                    "node_energy": np.asarray(r["node_energy"], np.float64)}
            assert_parity(mine, want, len(atoms))
    with pytest.raises(NotImplementedError):
        calc.calculate_batch(periodic, ["energy", "stress"])


def test_multi_head_calculator_selects_the_named_head(tmp_path):
    """``head=`` picks the head (calculators.py:128-137): the default is the first
    head; each head's energy, forces and stress match the oracle's masked
    multi-head readout for that head."""
    from mace_mlx_b200.spec import ModelSpec
    from mace_mlx_b200.weights import random_config, random_weights, write_model_dir

    cfg = random_config("medium", z_table=[14, 6], avg_num_neighbors=30.0, heads=["pt_head", "Default"],
                        atomic_energies=[[-5.1, -7.9], [-5.4, -8.1]], model_type="ScaleShiftMACE")
    cfg["scale"], cfg["shift"] = [0.8, 1.3], [0.3, -0.2]
    weights = random_weights(ModelSpec.from_config(cfg), 5)
    d = str(write_model_dir(tmp_path / "mh", cfg, weights))
    st = diamond_si(2, 0.05, 31)
    st.numbers[::4] = 6
    i, j, S = neighbour_list(st.positions, st.cell, st.pbc, cfg["r_max"])
    species = np.where(st.numbers == 14, 0, 1)
    energies = {}
    for head in (None, "pt_head", "Default"):
        calc = MACECalculator(model_path=d, device="cuda", head=head, skin=0.0)
        assert calc.model.head == (head or "pt_head")
        atoms = Atoms(st.numbers, st.positions, st.cell, True)
        atoms.calc = calc
        gpu = {"energy": np.array([atoms.get_potential_energy()]), "forces": atoms.get_forces().astype(np.float64),
               "stress": atoms.get_stress(), "node_energy": calc.results["node_energy"]}
        ref = OracleMACE(cfg, weights, head=head).compute(st.positions, species, i, j, S, st.cell, stress=True)
        assert_parity(gpu, ref, len(st), stress=True)
        energies[head] = float(gpu["energy"][0])
    assert energies[None] == energies["pt_head"]
    assert abs(energies["pt_head"] - energies["Default"]) > 1.0
