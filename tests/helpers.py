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


def run_gpu(model, st: Structure, r_cut: float | None = None, virial: bool = True):
    """Neighbour list + one evaluation through the C ABI; returns numpy results."""
    import torch

    dev = model.device
    species = model.species_index(st.numbers)
    gp = torch.as_tensor(graph_ptr_of(st), device=dev)
    pos64 = torch.tensor(st.positions, dtype=torch.float64, device=dev)
    periodic = bool(np.any(st.pbc))
    cell64 = torch.tensor(st.cell, dtype=torch.float64, device=dev) if periodic else None
    edges = model.neighbour_list(pos64, cell64, st.pbc, gp, r_cut or model.r_max)
    out = model.evaluate(pos64.float(), cell64.float() if periodic else None, torch.as_tensor(species, device=dev),
                         gp, edges, forces=True, virial=virial and periodic)
    torch.cuda.synchronize(dev)
    res = {
        "energy": out["energy"].cpu().numpy(),
        "node_energy": out["node_energy"].cpu().numpy(),
        "forces": out["forces"].cpu().numpy().astype(np.float64),
    }
    if virial and periodic:
        g = out["virial"].cpu().numpy().reshape(3, 3)
        s = 0.5 * (g + g.T) / abs(np.linalg.det(st.cell))
        res["stress"] = s[[0, 1, 2, 1, 0, 0], [0, 1, 2, 2, 2, 1]]
    return res, edges, species


def assert_parity(gpu: dict, ref: dict, n_atoms: int, stress: bool = False):
    """BASELINE tolerances (absolute) plus relative bounds that keep them meaningful."""
    de = np.abs(gpu["energy"] - ref["energy"]).max()
    escale = max(np.abs(ref["node_energy"]).sum(), 1e-3)
    assert de / n_atoms < 1e-5, f"energy/atom {de / n_atoms:.3e}"
    assert de < 1e-5 * escale + 1e-7, f"energy rel {de / escale:.3e}"
    df = np.abs(gpu["forces"] - ref["forces"]).max()
    fscale = np.abs(ref["forces"]).max()
    assert df < 1e-4, f"forces abs {df:.3e}"
    assert df < 1e-4 * fscale + 1e-9, f"forces rel {df / fscale:.3e}"
    dn = np.abs(gpu["node_energy"] - ref["node_energy"]).max()
    assert dn < 1e-5 * max(np.abs(ref["node_energy"]).max(), 1e-3)
    if stress:
        ds = np.abs(gpu["stress"] - ref["stress"]).max()
        sscale = np.abs(ref["stress"]).max()
        assert ds < 1e-6, f"stress abs {ds:.3e}"
        assert ds < 1e-4 * sscale + 1e-12, f"stress rel {ds / sscale:.3e}"


def graph_ptr_of(st: Structure) -> np.ndarray:
    if st.batch is None:
        return np.array([0, len(st)], dtype=np.int32)
    counts = np.bincount(st.batch, minlength=st.num_graphs)
    return np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
