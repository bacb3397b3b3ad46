"""Shared helpers of the test suite: synthetic cases, layout conversion, and the
comparison of the CUDA path (through the C ABI) with the CPU oracle."""

from __future__ import annotations

import numpy as np

from mace_mlx_b200.irreps import Irreps
from mace_mlx_b200.spec import ModelSpec
from mace_mlx_b200.structures import Structure, diamond_si
from mace_mlx_b200.weights import random_config, random_weights


def irreps_to_channel_last(x: np.ndarray, irreps: Irreps) -> np.ndarray:
    """Reference layout (u*(2l+1)+m per slot) -> channel-last (m*C+u per slot)."""
    x = np.asarray(x)
    out, o = [], 0
    for m in irreps:
        blk = x[:, o : o + m.dim].reshape(x.shape[0], m.mul, m.ir.dim)
        out.append(blk.transpose(0, 2, 1).reshape(x.shape[0], -1))
        o += m.dim
    return np.concatenate(out, axis=1)


def rel_err(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    scale = max(np.abs(b).max(initial=0.0), 1e-30)
    return float(np.abs(a - b).max(initial=0.0) / scale)


def make_case(arch: str = "small", structure: Structure | None = None, seed: int = 0, *, z_table=None,
              avg_num_neighbors: float | None = None, r_max: float = 6.0, **cfg):
    st = structure if structure is not None else diamond_si(2, 0.05, seed)
    z_table = z_table or list(range(1, 90))
    if avg_num_neighbors is None:
        avg_num_neighbors = 40.0
    config = random_config(arch, z_table=z_table, avg_num_neighbors=avg_num_neighbors, r_max=r_max, **cfg)
    spec = ModelSpec.from_config(config)
    weights = random_weights(spec, seed)
    return config, weights, st


def species_of(numbers, z_table) -> np.ndarray:
    lut = {z: i for i, z in enumerate(z_table)}
    return np.array([lut[int(z)] for z in numbers], dtype=np.int32)


def graph_ptr_of(st: Structure) -> np.ndarray:
    if st.batch is None:
        return np.array([0, len(st)], dtype=np.int32)
    counts = np.bincount(st.batch, minlength=st.num_graphs)
    return np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
