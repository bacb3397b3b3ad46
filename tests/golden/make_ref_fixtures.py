"""Run the UNMODIFIED reference package on the parity cases and record its outputs.

The reference (mace-mlx) is imported from its own checkout -- the path comes
from the required ``--reference`` argument or ``$MACE_MLX_REFERENCE`` -- on top
of ``refshim/``, a torch-CPU stand-in for the MLX API it is written against
(MLX is not installed here) plus stubs of the two ASE modules it imports at
module level.  For every case of ``ref_cases.py`` the script

1. writes the seeded config + weights as a converted-model directory and loads
   it with the reference's own ``mace_mlx.model.load_model`` (``model.py:664-720``);
2. builds the one-hot node attributes, int32 ``edge_index`` and float32 shifts
   exactly as ``MACEMLXCalculator.calculate`` does (``calculators.py:297-375``),
   with the ``"ijS"`` neighbour list of the test oracle (``oracle/nl.py``;
   matscipy/ASE are absent);
3. calls the calculator's own step functions: ``_compute_energy_forces_stress``
   for periodic cases (``calculators.py:489-570``, symmetric displacement) and
   ``_compute_energy_and_forces`` otherwise (``:431-483``).  A batch of several
   molecules calls the model with ``num_graphs`` > 1 through the same
   ``mx.value_and_grad`` construction, since the calculator always passes one
   graph (``calculators.py:406``).

It runs each case twice: with MLX's float32 held in float64 (the reference's
algorithm without rounding noise: keys ``energy``, ``forces``, ...) and in
float32 like MLX itself (keys ``*_f32``).  Outputs: ``ref_<case>.npz``.

Usage: ``python tests/golden/make_ref_fixtures.py --reference <path of the mace-mlx checkout> [case ...]``
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def _import_reference(ref_root: str):
    sys.path.insert(0, str(HERE / "refshim"))
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, ref_root)
    import mace_mlx.calculators as rcalc  # noqa: E402
    import mace_mlx.model as rmodel  # noqa: E402
    import mlx.core as mx  # noqa: E402  (the stand-in)

    assert "refshim" in mx.__file__, "refusing to run against a real MLX: this script targets the CPU stand-in"
    return rmodel, rcalc, mx


def _run_case(name: str, ref_root: str) -> dict:
    """One case in the current process (float mode fixed by REFSHIM_FLOAT)."""
    rmodel, rcalc, mx = _import_reference(ref_root)
    from oracle.nl import neighbour_list
    from ref_cases import CASE_HEADS, CASES, reference_inputs
    from mace_mlx_b200.weights import write_model_dir

    config, weights, st, stress = CASES[name]()
    with tempfile.TemporaryDirectory() as d:
        write_model_dir(d, config, weights)
        model = rmodel.load_model(d)
    if name in CASE_HEADS:  # as the calculator selects a head (calculators.py:128-137)
        model._head_idx = model.heads.index(CASE_HEADS[name])

    n = len(st)
    periodic = bool(np.any(st.pbc))
    i, j, S = neighbour_list(st.positions, st.cell, st.pbc, config["r_max"], batch=st.batch)
    z_to_idx = {int(z): k for k, z in enumerate(config["z_table"])}
    idx = np.array([z_to_idx[int(z)] for z in st.numbers], dtype=np.int32)
    node_attrs = np.zeros((n, len(config["z_table"])), dtype=np.float32)
    node_attrs[np.arange(n), idx] = 1.0
    pos32, cell32 = reference_inputs(st)

    positions_mx = mx.array(pos32.astype(np.float32))
    node_attrs_mx = mx.array(node_attrs, dtype=mx.float32)
    edge_index_mx = mx.array(np.stack([i, j]).astype(np.int32))
    shifts_mx = mx.array(S.astype(np.float32))
    cell_mx = mx.array(cell32.astype(np.float32)) if periodic else None

    calc = object.__new__(rcalc.MACEMLXCalculator)
    calc.model = model
    calc._use_compile = False
    calc._step_fn = calc._step_fn_raw = None
    calc._stress_step_fn = calc._stress_step_fn_raw = None
    calc._step_fn_head = calc._stress_step_fn_head = None

    out = {}
    if st.num_graphs > 1:
        batch_mx = mx.array(st.batch.astype(np.int32))
        G = st.num_graphs

        def energy_fn(pos):
            o = model(pos, node_attrs_mx, edge_index_mx, shifts_mx, cell_mx, batch_mx, G)
            return o["energy"].sum(), (o["energy"], o["node_energy"])

        (_, (energy, node_energy)), grad = mx.value_and_grad(energy_fn)(positions_mx)
        out["energy"] = np.array(energy)
        out["node_energy"] = np.array(node_energy)
        out["forces"] = -np.array(grad)
    else:
        batch_mx = mx.zeros(n, dtype=mx.int32)
        if stress and periodic:
            e, f, s, ne = calc._compute_energy_forces_stress(
                positions_mx, node_attrs_mx, edge_index_mx, shifts_mx, cell_mx, batch_mx, num_graphs=1)
            out["stress"] = np.array(s)
        else:
            e, f, ne = calc._compute_energy_and_forces(
                positions_mx, node_attrs_mx, edge_index_mx, shifts_mx, cell_mx, batch_mx, num_graphs=1)
        out["energy"] = np.array(e).reshape(1)
        out["forces"] = np.array(f)
        out["node_energy"] = np.array(ne)
    res = {k: np.asarray(v, dtype=np.float64) for k, v in out.items()}
    res["n_edges"] = np.array(len(i))
    return res


def _child(name: str, ref_root: str, mode: str, out_path: str):
    env = dict(os.environ, REFSHIM_FLOAT=mode)
    cmd = [sys.executable, __file__, "--reference", ref_root, "--child", name, "--child-out", out_path]
    subprocess.run(cmd, env=env, check=True)
    with np.load(out_path) as z:
        return {k: np.asarray(z[k]) for k in z.files}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MACE_MLX_REFERENCE"),
                    help="path of the mace-mlx checkout (required; or $MACE_MLX_REFERENCE)")
    ap.add_argument("--child", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--child-out", default=None, help=argparse.SUPPRESS)
    ap.add_argument("cases", nargs="*")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <path of the mace-mlx checkout> or set MACE_MLX_REFERENCE")
    sys.path.insert(0, str(HERE))
    sys.path.insert(0, str(ROOT))
    if args.child:
        np.savez(args.child_out, **_run_case(args.child, args.reference))
        return

    from ref_cases import CASES, digest_config, digest_weights, reference_inputs

    for name in args.cases or list(CASES):
        config, weights, st, stress = CASES[name]()
        with tempfile.TemporaryDirectory() as d:
            r64 = _child(name, args.reference, "float64", os.path.join(d, "r64.npz"))
            r32 = _child(name, args.reference, "float32", os.path.join(d, "r32.npz"))
        pos32, _ = reference_inputs(st)
        rec = {
            "positions": np.asarray(st.positions, dtype=np.float64),
            "positions_f32": pos32,
            "numbers": np.asarray(st.numbers, dtype=np.int32),
            "cell": np.asarray(st.cell, dtype=np.float64),
            "pbc": np.asarray(st.pbc, dtype=bool),
            "batch": np.asarray(st.batch if st.batch is not None else np.zeros(len(st)), dtype=np.int32),
            "num_graphs": np.array(st.num_graphs),
            "stress_computed": np.array("stress" in r64),
            "config_digest": np.array(digest_config(config)),
            "weights_digest": np.array(digest_weights(weights)),
            "config_json": np.array(json.dumps(config, sort_keys=True)),
        }
        rec.update(r64)
        for k, v in r32.items():
            if k != "n_edges":
                rec[f"{k}_f32"] = v
        np.savez_compressed(HERE / f"ref_{name}.npz", **rec)
        fmax = np.abs(r64["forces"]).max()
        d32 = np.abs(r64["forces"] - r32["forces"]).max()
        print(f"{name}: N={len(st)} E={int(r64['n_edges'])} energy={r64['energy'][:3]} |F|max={fmax:.4f} "
              f"fp32-vs-fp64 dF={d32:.2e}", flush=True)


if __name__ == "__main__":
    main()
