"""The oracle against the reference's OWN execution.

``tests/golden/ref_*.npz`` hold energies, per-atom energies, forces and
stresses computed by the unmodified reference package (mace-mlx 0.5.0, run on
the CPU through a torch stand-in of the MLX API, ``tests/golden/refshim``;
generator ``tests/golden/make_ref_fixtures.py``).  These tests pin
``oracle/model.py`` -- and through it every CPU-side parity statement -- to the
reference at the composed-model level, and check that the seeded case
generators still produce exactly the inputs the reference was given."""

import json

import numpy as np
import pytest
import torch

from golden.ref_cases import CASE_HEADS, CASES, NO_CUDA_PATH, digest_config, digest_weights
from oracle.model import OracleMACE
from oracle.nl import neighbour_list

torch.set_num_threads(min(8, torch.get_num_threads()))

# c1 (Si1000, 44k edges) takes minutes in the float64 oracle; its reference
# fixture is checked against the CUDA path in tests/test_gpu_ref_parity.py.
CPU_CASES = [c for c in CASES if c != "c1_medium_si1000"]


def load_fixture(golden_dir, name):
    with np.load(golden_dir / f"ref_{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("name", list(CASES))
def test_generators_reproduce_the_reference_inputs(golden_dir, name):
    fx = load_fixture(golden_dir, name)
    config, weights, st, stress = CASES[name]()
    assert str(fx["config_digest"]) == digest_config(config)
    assert str(fx["weights_digest"]) == digest_weights(weights)
    assert json.loads(str(fx["config_json"])) == json.loads(json.dumps(config, sort_keys=True))
    np.testing.assert_array_equal(fx["positions"], st.positions)
    np.testing.assert_array_equal(fx["numbers"], st.numbers)
    np.testing.assert_array_equal(fx["cell"], st.cell)
    assert bool(fx["stress_computed"]) == (stress and bool(np.any(st.pbc)))


@pytest.mark.parametrize("name", CPU_CASES)
def test_oracle_equals_the_reference_execution(golden_dir, name):
    fx = load_fixture(golden_dir, name)
    config, weights, st, _ = CASES[name]()
    i, j, S = neighbour_list(st.positions, st.cell, st.pbc, config["r_max"], batch=st.batch)
    assert len(i) == int(fx["n_edges"])
    lut = {int(z): k for k, z in enumerate(config["z_table"])}
    species = np.array([lut[int(z)] for z in st.numbers])
    periodic = bool(np.any(st.pbc))
    cell = fx["cell"].astype(np.float32).astype(np.float64) if periodic else None
    res = OracleMACE(config, weights, head=CASE_HEADS.get(name)).compute(fx["positions_f32"], species, i, j, S, cell,
                                              stress=bool(fx["stress_computed"]), batch=st.batch,
                                              num_graphs=st.num_graphs)

    def close(a, b, rtol):
        a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
        scale = max(np.abs(b).max(), 1e-12)
        assert np.abs(a - b).max() <= rtol * scale, (np.abs(a - b).max(), scale)

    # Both sides run in float64, but the reference rounds its coupling constants
    # to float32 in numpy before it builds arrays from them (3j symbols
    # tensor_product.py:255, SH recursion spherical_harmonics.py:40, U rows
    # symmetric_contraction.py:321, 421), while the oracle keeps them in float64.
    # That leaves ~1e-9 relative on the plain models and up to ~1e-7 on the
    # density-normalised ones, whose activations are ~40x larger; the bound
    # here is 1e-6 of each quantity's scale (the parity bounds are 1e-5..1e-4).
    close(res["energy"], fx["energy"], 1e-6)
    close(res["node_energy"], fx["node_energy"], 1e-6)
    close(res["forces"], fx["forces"], 1e-6)
    if bool(fx["stress_computed"]):
        close(res["stress"], fx["stress"], 1e-6)


@pytest.mark.parametrize("name", list(CASES))
def test_reference_float32_run_is_within_tolerance_of_its_float64_run(golden_dir, name):
    """The reference's own fp32 execution differs from its fp64 execution by
    far less than the parity tolerances, so the fp64 fixtures are the pin.
    The energy bound is 1e-6 eV/atom, or 1e-6 of the mean per-atom energy
    where that is larger (fp32 rounding grows with the magnitude: the random
    non-linear-block model on LiPSO-300 carries ~4 eV per atom)."""
    fx = load_fixture(golden_dir, name)
    n = len(fx["numbers"])
    e_scale = float(np.abs(fx["node_energy"]).mean())
    assert np.abs(fx["energy_f32"] - fx["energy"]).max() / n < max(1e-6, 1e-6 * e_scale)
    assert np.abs(fx["forces_f32"] - fx["forces"]).max() < 1e-4
    if bool(fx["stress_computed"]):
        assert np.abs(fx["stress_f32"] - fx["stress"]).max() < 1e-6


@pytest.mark.parametrize("name", NO_CUDA_PATH)
def test_cases_without_a_cuda_path_are_refused_when_packed(name):
    from mace_mlx_b200.pack import PackedModel
    from mace_mlx_b200.spec import ModelSpec, UnsupportedModel

    config, weights, _, _ = CASES[name]()
    with pytest.raises(UnsupportedModel, match="no CUDA path"):
        PackedModel(ModelSpec.from_config(config, head=CASE_HEADS.get(name)), weights)
