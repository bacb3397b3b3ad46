"""The parity cases whose energies, forces and stresses were computed by the
reference implementation itself (``make_ref_fixtures.py``).

Each case is fully determined by this file and the package's seeded
generators: a model config + seeded random-init weights
(``mace_mlx_b200.weights``) and a seeded structure
(``mace_mlx_b200.structures``).  The fixtures additionally store the exact
inputs the reference was given (positions rounded to float32 as the
reference's calculator does, ``calculators.py:370``) and digests of the config
and weights, so a drift of a generator is caught instead of silently compared.
"""

from __future__ import annotations

import hashlib
import json

import numpy as np

from mace_mlx_b200.spec import ModelSpec
from mace_mlx_b200.structures import Structure, diamond_si, lipso_box, molecule_batch
from mace_mlx_b200.weights import random_config, random_weights


def _case(arch, st, seed, stress, *, z_table=None, avg=40.0, r_max=6.0, edit=None, **cfg):
    z_table = z_table or list(range(1, 90))
    config = random_config(arch, z_table=z_table, avg_num_neighbors=avg, r_max=r_max, **cfg)
    if edit is not None:
        edit(config)
    weights = random_weights(ModelSpec.from_config(config), seed)
    return config, weights, st, stress


def _scale_shift(cfg):
    cfg["scale"], cfg["shift"] = 1.3, -0.2


def _scale_shift_per_head(cfg):
    cfg["scale"], cfg["shift"] = [0.8, 1.3], [0.3, -0.2]


def _mixed_si(seed, sigma=0.05):
    st = diamond_si(2, sigma, seed)
    st.numbers[::3] = 6
    return st


# the mpa-0 family's blocks: density normalisation, Agnesi transform, ZBL repulsion
MPA = dict(use_density_normalization=True, distance_transform={}, pair_repulsion={})

CASES = {
    # BASELINE config 0 at its full size: small arch, Si216, energy + forces + stress
    "c0_small_si216": lambda: _case("small", diamond_si(3, 0.01, 0), 0, True, avg=46.0),
    # the three architectures on a small periodic cell, with stress
    "si64_small": lambda: _case("small", diamond_si(2, 0.05, 11), 11, True),
    "si64_medium": lambda: _case("medium", diamond_si(2, 0.05, 11), 11, True),
    "si64_large": lambda: _case("large", diamond_si(2, 0.05, 11), 11, True),
    # four species, large arch (layer-1 conv with 1o and 2e sources), with stress
    "lipso300_large": lambda: _case("large", lipso_box(300, 2), 2, True, z_table=[3, 8, 15, 16], avg=50.0),
    # MACE-OFF-like batch of molecules: per-graph energies, no cell
    "mol8_off": lambda: _case("medium", molecule_batch(8, 3), 3, False, z_table=[1, 6, 7, 8], avg=12.0,
                              r_max=5.0, hidden_irreps="96x0e + 96x1o"),
    # non-residual first block, ScaleShiftMACE with E0, two species
    "nonres_scaleshift": lambda: _case("medium", _mixed_si(4), 4, True, z_table=[14, 6], avg=30.0,
                                       first_interaction_nonresidual=True, atomic_energies=[-5.4, -8.1],
                                       model_type="ScaleShiftMACE", edit=_scale_shift),
    # other max_ell / correlation orders
    "lmax2_corr3": lambda: _case("medium", diamond_si(2, 0.05, 5), 5, True, z_table=[14], max_ell=2, correlation=3),
    "lmax3_corr2": lambda: _case("medium", diamond_si(2, 0.05, 5), 5, True, z_table=[14], max_ell=3, correlation=2),
    "lmax1_corr1": lambda: _case("medium", diamond_si(2, 0.05, 5), 5, True, z_table=[14], max_ell=1, correlation=1),
    # mpa-0-shaped models (density-normalised blocks + Agnesi + ZBL): ScaleShiftMACE with a
    # non-residual first block on the LiPSO box (pairs inside the ZBL range), plain MACE on a
    # strongly rattled Si/C cell, and a molecule batch (C-H bonds inside the ZBL range)
    "mpa_lipso300": lambda: _case("medium", lipso_box(300, 2), 6, True, z_table=[3, 8, 15, 16], avg=50.0,
                                  first_interaction_nonresidual=True, atomic_energies=[-1.9, -4.9, -5.4, -4.1],
                                  model_type="ScaleShiftMACE", edit=_scale_shift, **MPA),
    "mpa_si64_mixed": lambda: _case("medium", _mixed_si(21, 0.15), 7, True, z_table=[6, 14], **MPA),
    "mpa_mol8": lambda: _case("medium", molecule_batch(8, 3), 8, False, z_table=[1, 6, 7, 8], avg=12.0, r_max=5.0,
                              first_interaction_nonresidual=True, **MPA),
    # a two-head model (multi-head fine-tuning layout): per-head E0, scale and shift, the
    # second head selected (CASE_HEADS), two species, with stress
    "mh2_medium_si64mixed": lambda: _case("medium", _mixed_si(9), 9, True, z_table=[14, 6], avg=30.0,
                                          heads=["pt_head", "Default"],
                                          atomic_energies=[[-5.1, -7.9], [-5.4, -8.1]],
                                          model_type="ScaleShiftMACE", edit=_scale_shift_per_head),
    # the species-agnostic product (one symmetric-contraction weight set), two species, with stress
    "agnostic_medium_si64mixed": lambda: _case("medium", _mixed_si(12), 12, True, z_table=[14, 6], avg=30.0,
                                               use_agnostic_product=True),
    # the mh-1 family's shape: non-linear interaction blocks (edge irreps up to 2e), the
    # agnostic product, the envelope on the radial-MLP output (apply_cutoff=False) and two
    # heads with the second one selected; two species, with stress
    "mh1_medium_si64mixed": lambda: _case("medium", _mixed_si(13), 13, True, z_table=[14, 6], avg=30.0,
                                          nonlinear_interaction=True, edge_irreps="128x0e + 128x1o + 128x2e",
                                          use_agnostic_product=True, apply_cutoff=False,
                                          heads=["pt_head", "Default"],
                                          atomic_energies=[[-5.1, -7.9], [-5.4, -8.1]],
                                          model_type="ScaleShiftMACE", edit=_scale_shift_per_head),
    # the non-linear block alone: large arch, edge irreps left to the block's input,
    # species-indexed product, envelope on the radial features; four species, with stress
    "nonlinear_large_lipso300": lambda: _case("large", lipso_box(300, 2), 15, True, z_table=[3, 8, 15, 16],
                                              avg=50.0, nonlinear_interaction=True),
    # apply_cutoff=False with the standard residual blocks
    "nocutoff_small_si64": lambda: _case("small", diamond_si(2, 0.05, 14), 14, True, z_table=[14],
                                         apply_cutoff=False),
    # BASELINE config 1 (the headline) at its full size: medium Si1000, energy + forces
    "c1_medium_si1000": lambda: _case("medium", diamond_si(5, 0.05, 1), 1, False, avg=44.0),
}


# cases whose blocks the oracle restates but the CUDA path refuses (pack.py raises
# UnsupportedModel): the mh-1 non-linear block
NO_CUDA_PATH = ("mh1_medium_si64mixed", "nonlinear_large_lipso300")

# the head each multi-head case selects (the reference calculator's ``head`` argument)
CASE_HEADS = {"mh2_medium_si64mixed": "Default", "mh1_medium_si64mixed": "Default"}


def digest_config(config: dict) -> str:
    return hashlib.sha256(json.dumps(config, sort_keys=True).encode()).hexdigest()[:16]


def digest_weights(weights: dict) -> str:
    h = hashlib.sha256()
    for k in sorted(weights):
        h.update(k.encode())
        h.update(np.ascontiguousarray(weights[k], dtype=np.float32).tobytes())
    return h.hexdigest()[:16]


def reference_inputs(st: Structure):
    """Positions and cell exactly as the reference's calculator hands them to
    the model: float32 (``calculators.py:370, 372-375``)."""
    pos = np.asarray(st.positions, dtype=np.float32).astype(np.float64)
    cell = np.asarray(st.cell, dtype=np.float32).astype(np.float64)
    return pos, cell
