"""Generate the golden fixtures of this directory from the reference itself.

The reference package cannot be imported as a whole here (it needs MLX), but
its ``mace_mlx/irreps.py`` and ``mace_mlx/clebsch_gordan.py`` depend only on
numpy/scipy.  This script loads exactly those two files from the reference
checkout (the required ``--reference`` argument, or ``$MACE_MLX_REFERENCE``)
under a stub package and records their outputs:

* ``cg_golden.npz``: real Wigner 3j symbols for all l <= 4 triples, the
  spherical-harmonics recursion tensors ``so3_clebsch_gordan(l-1, 1, l)``, and
  the symmetric-contraction tensors ``U_matrix_real`` (as non-zero lists) for
  the coupling irreps of max_ell 2 and 3, outputs 0e/1o/2e/3o, nu = 1..3;
* ``irreps_golden.json``: parsing, dims, sort permutations and products of a
  set of irreps strings.

Run once where the reference is available:
``python tests/golden/make_golden.py --reference <path of the mace-mlx checkout>``.
The tests only read the fixtures.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load_reference(root: str):
    pkg = types.ModuleType("mace_mlx")
    pkg.__path__ = [os.path.join(root, "mace_mlx")]
    sys.modules["mace_mlx"] = pkg
    mods = {}
    for name in ("irreps", "clebsch_gordan"):
        spec = importlib.util.spec_from_file_location(f"mace_mlx.{name}", os.path.join(root, "mace_mlx", f"{name}.py"))
        m = importlib.util.module_from_spec(spec)
        sys.modules[f"mace_mlx.{name}"] = m
        spec.loader.exec_module(m)
        mods[name] = m
    return mods["irreps"], mods["clebsch_gordan"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MACE_MLX_REFERENCE"),
                    help="path of the mace-mlx checkout (required; or $MACE_MLX_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <path of the mace-mlx checkout> or set MACE_MLX_REFERENCE")
    rirr, rcg = load_reference(args.reference)
    out = {}
    for l1 in range(5):
        for l2 in range(5):
            for l3 in range(abs(l1 - l2), min(l1 + l2, 4) + 1):
                out[f"w3j_{l1}_{l2}_{l3}"] = rcg.wigner_3j(l1, l2, l3)
    for l in range(2, 5):
        out[f"shcg_{l}"] = rcg.so3_clebsch_gordan(l - 1, 1, l)
    for lmax in (2, 3):
        coupling = rirr.Irreps(" + ".join(f"1x{l}{'e' if l % 2 == 0 else 'o'}" for l in range(lmax + 1)))
        for L in ("0e", "1o", "2e", "3o"):
            if int(L[0]) > lmax:
                continue
            for nu in (1, 2, 3):
                U = rcg.U_matrix_real(coupling, rirr.Irreps(f"1x{L}"), nu)[-1]
                nz = np.argwhere(np.abs(U) > 1e-12)
                out[f"U_{lmax}_{L}_{nu}_shape"] = np.array(U.shape)
                out[f"U_{lmax}_{L}_{nu}_idx"] = nz.astype(np.int16)
                out[f"U_{lmax}_{L}_{nu}_val"] = U[tuple(nz.T)]
    np.savez_compressed(HERE / "cg_golden.npz", **out)

    cases = ["128x0e", "128x0e + 128x1o", "128x0e+128x1o+128x2e", "16x1o + 8x0e + 4x1e + 2x0o",
             "1x0e+1x1o+1x2e+1x3o", "96x0e + 96x1o", "3x2e + 1x1o + 2x2o + 5x0e"]
    irr = []
    for c in cases:
        ir = rirr.Irreps(c)
        srt = ir.sort()
        irr.append({
            "spec": c, "dim": ir.dim, "repr": repr(ir), "sorted": repr(srt.irreps), "perm": list(srt.p),
            "inv": list(srt.inv), "slices": [[s.start, s.stop] for s in ir.slices],
        })
    prods = []
    for a in ("0e", "1o", "2e", "3o", "1e", "2o"):
        for b in ("0e", "1o", "2e", "3o"):
            prods.append({"a": a, "b": b, "out": [repr(x) for x in rirr.Irrep(a) * rirr.Irrep(b)]})
    (HERE / "irreps_golden.json").write_text(json.dumps({"irreps": irr, "products": prods}, indent=1))
    print("wrote", HERE / "cg_golden.npz", "and", HERE / "irreps_golden.json")


if __name__ == "__main__":
    main()
