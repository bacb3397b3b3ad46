"""Converted-model directories: ``config.json`` + ``weights.npz``.

The layout is the reference's (``model.py:664-720`` loads it; ``converter.py``
writes it from a torch checkpoint), so a directory converted for the reference
loads here unchanged.  ``write_random_model`` writes a seeded random-init model
in the same layout; "seed k" is defined by this project with numpy's
``default_rng(k)`` and the reference's initialisation scales:
N(0,1) for o3.Linear / FCTP weights (``linear.py:70``, ``tensor_product.py:286``),
N(0,1)/K for symmetric-contraction weights (``symmetric_contraction.py:240-252``),
and ``n*pi/r_max`` Bessel frequencies (``radial.py:37-58``).  The radial MLP and
the last readout are written the way ``converter.py`` writes a freshly
initialised e3nn model: ``N(0,1)/sqrt(fan_in)`` per layer with the SiLU
second-moment factor folded into every layer that follows an activation
(``converter.py:578-646``) and into ``readouts.{last}.linear_2``
(``converter.py:907-929``).  This keeps activations O(1) so that forces are
O(0.1-1) eV/A and the parity tolerances are meaningful.
"""

from __future__ import annotations

import json
import os
from pathlib import Path

import numpy as np

from .spec import ModelSpec

# 1 / sqrt(E[silu(x)^2]) for x ~ N(0, 1) (e3nn normalize2mom; reference utils.py:17)
SILU_NORM_FACTOR = 1.6791768074035645

ARCHS = {
    "small": "128x0e",
    "medium": "128x0e + 128x1o",
    "large": "128x0e + 128x1o + 128x2e",
}


def load_model_dir(model_dir: str | os.PathLike) -> tuple[dict, dict[str, np.ndarray]]:
    """Read a converted model directory; returns (config, flat weights)."""
    d = Path(model_dir)
    with open(d / "config.json") as f:
        config = json.load(f)
    with np.load(d / "weights.npz") as z:
        weights = {k: np.asarray(z[k]) for k in z.files}
    return config, weights


def check_weights(spec: ModelSpec, weights: dict[str, np.ndarray]) -> None:
    """Raise ``ValueError`` naming every missing or mis-shaped array."""
    want = spec.weight_shapes()
    errs = []
    for k, sh in want.items():
        if k not in weights:
            errs.append(f"missing {k}")
        elif tuple(weights[k].shape) != tuple(sh):
            if k == "atomic_energies_fn.atomic_energies" and weights[k].size == int(np.prod(sh)):
                continue
            errs.append(f"{k}: shape {tuple(weights[k].shape)} != expected {tuple(sh)}")
    if errs:
        raise ValueError("converted weights do not match config: " + "; ".join(errs[:8]))


def random_config(
    arch: str = "medium",
    *,
    r_max: float = 6.0,
    num_bessel: int = 8,
    num_polynomial_cutoff: int = 5,
    max_ell: int = 3,
    num_interactions: int = 2,
    correlation: int = 3,
    num_elements: int = 89,
    z_table: list[int] | None = None,
    avg_num_neighbors: float = 1.0,
    radial_MLP: list[int] | None = None,
    hidden_irreps: str | None = None,
    first_interaction_nonresidual: bool = False,
    atomic_energies: list[float] | None = None,
    model_type: str = "MACE",
    use_density_normalization: bool = False,
    distance_transform: dict | None = None,
    pair_repulsion: dict | None = None,
    heads: list[str] | None = None,
    use_agnostic_product: bool = False,
    nonlinear_interaction: bool = False,
    edge_irreps: str | None = None,
    apply_cutoff: bool = True,
) -> dict:
    """A converted-model config.  ``use_density_normalization``,
    ``distance_transform`` (Agnesi; ``{}`` for the defaults) and
    ``pair_repulsion`` (ZBL; ``{}`` for the defaults) give the mpa-0 family's
    blocks; ``heads`` (two or more names) a multi-head model, whose
    ``atomic_energies`` are then one row per head.  The converter's key
    layout is kept (``converter.py:167-300``).  ``nonlinear_interaction``
    selects the mh-1 family's non-linear interaction block (with
    ``edge_irreps``); ``apply_cutoff=False`` moves the envelope from the radial
    features to the radial-MLP output and the edge densities."""
    hidden = hidden_irreps or ARCHS[arch]
    if z_table is None:
        z_table = list(range(1, num_elements + 1))
    num_elements = len(z_table)
    if use_density_normalization:
        inter_cls = "RealAgnosticDensityInteractionBlock" if first_interaction_nonresidual else \
            "RealAgnosticDensityResidualInteractionBlock"
    else:
        inter_cls = "RealAgnosticInteractionBlock" if first_interaction_nonresidual else \
            "RealAgnosticResidualInteractionBlock"
    if nonlinear_interaction:
        inter_cls = "RealAgnosticResidualNonLinearInteractionBlock"
    extra = {}
    if edge_irreps is not None:
        extra["edge_irreps"] = str(edge_irreps)
    if not apply_cutoff:
        extra["apply_cutoff"] = False
    if use_density_normalization:
        extra["use_density_normalization"] = True
    if distance_transform is not None:
        from .elements import AGNESI_DEFAULTS, COVALENT_RADII

        dt = dict(AGNESI_DEFAULTS)
        dt.update(distance_transform)
        dt.setdefault("covalent_radii", list(COVALENT_RADII))
        extra["distance_transform"] = dt
    if pair_repulsion is not None:
        from .elements import ZBL_DEFAULTS

        pr = dict(ZBL_DEFAULTS)
        pr.update(pair_repulsion)
        extra["pair_repulsion"] = pr
    if use_agnostic_product:
        extra["use_agnostic_product"] = True
    if heads is not None and len(heads) > 1:
        extra["heads"] = [str(h) for h in heads]
        if atomic_energies is None:
            atomic_energies = [[0.0] * num_elements for _ in heads]
    return extra | {
        "r_max": float(r_max),
        "num_bessel": int(num_bessel),
        "num_polynomial_cutoff": int(num_polynomial_cutoff),
        "max_ell": int(max_ell),
        "num_interactions": int(num_interactions),
        "hidden_irreps": hidden,
        "correlation": int(correlation),
        "num_elements": int(num_elements),
        "atomic_energies": list(atomic_energies) if atomic_energies is not None else [0.0] * num_elements,
        "avg_num_neighbors": float(avg_num_neighbors),
        "radial_MLP": list(radial_MLP or [64, 64, 64]),
        "gate": "silu",
        "first_interaction_nonresidual": bool(first_interaction_nonresidual),
        "interaction_cls": inter_cls,
        "model_type": model_type,
        "scale": 1.0,
        "shift": 0.0,
        "z_table": [int(z) for z in z_table],
    }


def _nonlinear_block_array(key: str, shape, rng) -> np.ndarray | None:
    """Seeded values for the non-linear block's own arrays: torch's Linear
    scale (fan-in) for the radial MLPs, LayerNorm gains near one, small biases,
    and alpha / beta around the block's initial 20 / 0 with beta made non-zero
    so that the density term is exercised."""
    if key.endswith(".alpha"):
        return np.asarray(rng.uniform(8.0, 20.0), dtype=np.float32)
    if key.endswith(".beta"):
        return np.asarray(rng.uniform(0.3, 1.0), dtype=np.float32)
    if ".conv_tp_weights.layers." in key or ".density_fn.layers." in key:
        idx = int(key.rsplit(".layers.", 1)[1].split(".")[0])
        if idx % 3 == 0:  # Linear
            if key.endswith(".weight"):
                return (rng.standard_normal(shape) / np.sqrt(shape[1])).astype(np.float32)
            return (0.1 * rng.standard_normal(shape)).astype(np.float32)
        if key.endswith(".weight"):  # LayerNorm gain
            return (1.0 + 0.1 * rng.standard_normal(shape)).astype(np.float32)
        return (0.1 * rng.standard_normal(shape)).astype(np.float32)
    return None


def random_weights(spec: ModelSpec, seed: int) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    out: dict[str, np.ndarray] = {}
    nonlinear = {lay.index for lay in spec.layers if lay.nonlinear is not None}
    for key, shape in spec.weight_shapes().items():
        if key.startswith("interactions.") and int(key.split(".")[1]) in nonlinear:
            v = _nonlinear_block_array(key, shape, rng)
            if v is not None:
                out[key] = v
                continue
        if key == "atomic_energies_fn.atomic_energies":
            out[key] = np.asarray(spec.atomic_energies, dtype=np.float32)
        elif key.endswith("bessel_weights"):
            n = np.arange(1, shape[0] + 1, dtype=np.float64)
            out[key] = (n * np.pi / spec.r_max).astype(np.float32)
        elif ".conv_tp_weights.layers." in key:
            layer = int(key.rsplit(".layers.", 1)[1].split(".")[0]) // 2
            w = rng.standard_normal(shape) / np.sqrt(shape[1])
            if layer > 0:
                w = w * SILU_NORM_FACTOR
            out[key] = w.astype(np.float32)
        elif ".linear_2.weights." in key:
            out[key] = (rng.standard_normal(shape) * SILU_NORM_FACTOR).astype(np.float32)
        elif key.endswith(".density_fn.weight"):
            out[key] = (rng.standard_normal(shape) / np.sqrt(shape[1])).astype(np.float32)
        elif ".symmetric_contractions." in key:
            out[key] = (rng.standard_normal(shape) / shape[1]).astype(np.float32)
        else:
            out[key] = rng.standard_normal(shape).astype(np.float32)
    return out


def write_model_dir(out_dir: str | os.PathLike, config: dict, weights: dict[str, np.ndarray]) -> Path:
    d = Path(out_dir)
    d.mkdir(parents=True, exist_ok=True)
    with open(d / "config.json", "w") as f:
        json.dump(config, f, indent=1)
    np.savez(d / "weights.npz", **weights)
    return d


def write_random_model(out_dir, arch: str = "medium", seed: int = 0, **cfg_kw) -> Path:
    config = random_config(arch, **cfg_kw)
    spec = ModelSpec.from_config(config)
    return write_model_dir(out_dir, config, random_weights(spec, seed))
