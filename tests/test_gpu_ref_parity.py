"""The CUDA step (through the C ABI) against the reference's OWN execution.

Every fixture of ``tests/golden/ref_*.npz`` was computed by the unmodified
reference package (mace-mlx 0.5.0) on the CPU, in float64 (keys ``energy``,
``forces``, ...) and in float32 like MLX itself (``*_f32``).  The CUDA path
must match both within the BASELINE tolerances: energy 1e-5 eV/atom, forces
1e-4 eV/A max-abs, stress 1e-6 eV/A^3, plus the relative bounds of
``helpers.assert_parity``; and its neighbour list must have exactly the
reference run's edge count.  The cases include BASELINE configs 0 and 1 at
their full sizes, three models of the mpa-0 family and a two-head model with
its second head selected.  The cases of ``NO_CUDA_PATH`` (blocks the oracle
restates but the CUDA path refuses) are left out here; ``test_ref_fixtures.py``
checks that packing them raises."""

import numpy as np
import pytest
import torch

from golden.ref_cases import CASE_HEADS, CASES, NO_CUDA_PATH, digest_weights
from helpers import assert_parity, run_gpu
from mace_mlx_b200.model import MACEModel

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", [c for c in CASES if c not in NO_CUDA_PATH])
def test_cuda_step_matches_reference_execution(golden_dir, name):
    with np.load(golden_dir / f"ref_{name}.npz") as z:
        fx = {k: z[k] for k in z.files}
    config, weights, st, _ = CASES[name]()
    assert str(fx["weights_digest"]) == digest_weights(weights)
    stress = bool(fx["stress_computed"])
    m = MACEModel(config=config, weights=weights, device=0, head=CASE_HEADS.get(name))
    gpu, edges, _ = run_gpu(m, st, virial=stress)
    assert edges.n_edges == int(fx["n_edges"])
    for suffix in ("", "_f32"):
        ref = {"energy": fx["energy" + suffix], "node_energy": fx["node_energy" + suffix],
               "forces": fx["forces" + suffix]}
        if stress:
            ref["stress"] = fx["stress" + suffix]
        assert_parity(gpu, ref, len(st), stress=stress)
    assert m.error_flag() == 0
    torch.cuda.synchronize()
