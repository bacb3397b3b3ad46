"""Coupling constants pinned to the reference's own tables (tests/golden, made by
tests/golden/make_golden.py from mace_mlx/clebsch_gordan.py and irreps.py)."""

import json
import math

import numpy as np
import pytest

from mace_mlx_b200 import cg
from mace_mlx_b200.irreps import Irrep, Irreps


@pytest.fixture(scope="module")
def gold(golden_dir):
    with np.load(golden_dir / "cg_golden.npz") as z:
        return {k: z[k] for k in z.files}


def test_wigner_3j_matches_reference(gold):
    n = 0
    for k, ref in gold.items():
        if not k.startswith("w3j_"):
            continue
        l1, l2, l3 = map(int, k.split("_")[1:])
        np.testing.assert_allclose(cg.wigner_3j(l1, l2, l3), ref, atol=1e-12, err_msg=k)
        n += 1
    assert n > 50


def test_w3j_unit_norm_and_selection_rule():
    for l1 in range(4):
        for l2 in range(4):
            for l3 in range(7):
                w = cg.wigner_3j(l1, l2, l3)
                if abs(l1 - l2) <= l3 <= l1 + l2:
                    assert abs(np.linalg.norm(w) - 1.0) < 1e-12
                else:
                    assert not np.any(w)


def test_sh_recursion_tensors_match_reference(gold):
    for l in range(2, 5):
        np.testing.assert_allclose(cg.so3_clebsch_gordan(l - 1, 1, l), gold[f"shcg_{l}"], atol=1e-12)
        np.testing.assert_allclose(cg.sh_coupling(l), gold[f"shcg_{l}"] * math.sqrt((2 * l + 1) / (3 * l)),
                                   atol=1e-12)


@pytest.mark.parametrize("lmax", [2, 3])
def test_U_matrices_match_reference(gold, lmax):
    coupling = " + ".join(f"1x{l}{'e' if l % 2 == 0 else 'o'}" for l in range(lmax + 1))
    for L in ("0e", "1o", "2e", "3o"):
        if int(L[0]) > lmax:
            continue
        for nu in (1, 2, 3):
            key = f"U_{lmax}_{L}_{nu}"
            U = cg.U_matrix_real(coupling, L, nu)
            assert tuple(U.shape) == tuple(gold[key + "_shape"]), key
            nz = np.argwhere(np.abs(U) > 1e-12)
            np.testing.assert_array_equal(nz, gold[key + "_idx"].astype(np.int64), err_msg=key)
            np.testing.assert_allclose(U[tuple(nz.T)], gold[key + "_val"], atol=1e-11, err_msg=key)


def test_irreps_match_reference(golden_dir):
    g = json.loads((golden_dir / "irreps_golden.json").read_text())
    for case in g["irreps"]:
        ir = Irreps(case["spec"])
        assert ir.dim == case["dim"]
        srt, perm, inv = ir.sort()
        assert list(srt) == list(Irreps(case["sorted"]))
        assert list(ir) == list(Irreps(case["repr"]))
        assert list(perm) == case["perm"]
        assert list(inv) == case["inv"]
        offs = ir.offsets()
        assert [[o, o + m.dim] for o, m in zip(offs, ir)] == case["slices"]
    for p in g["products"]:
        assert [str(x) for x in Irrep.parse(p["a"]).couple(Irrep.parse(p["b"]))] == p["out"]
