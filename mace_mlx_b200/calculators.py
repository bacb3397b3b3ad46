"""ASE calculator drop-in: ``MACECalculator`` / ``mace_mp`` / ``mace_off``.

Same constructor arguments, results dictionary, neighbour-list skin cache and
error behaviour as the reference's ``mace_mlx/calculators.py`` (line numbers
below refer to that file); the step itself runs on a B200 through
``libmace_b200``:

* constructor and ``model_paths`` / committee handling     -- :94-125
* model resolution and the converted-model cache layout    -- :28-38, :201-267
* neighbour-list rebuild rule (r_max + skin, skin/2 drift) -- :273-317
* species validation message                               -- :341-371
* sticky stress, results keys, Voigt stress                 -- :384-425, :489-531
* ``mace_mp`` / ``mace_off`` / ``mace_anicc`` / ``mace_omol`` -- :573-640

Differences: ``device`` names a CUDA device ("cuda", "gpu", "cuda:1", or an
index); "cpu" is rejected because this build has no CPU path.  ``use_compile``
(the reference's ``mx.compile`` switch) selects CUDA-graph replay of the fixed
kernel sequence.  Only float32 is computed.
"""

from __future__ import annotations

import os
import warnings
from pathlib import Path

import numpy as np
import torch

from .atoms import Calculator, all_changes
from .model import EdgeSet, MACEModel

_CONVERTER_CACHE_VERSION = 2
_NAMED = ("small", "medium", "large", "medium-mpa-0", "small-0b", "medium-0b", "small-0b2",
          "medium-0b2", "large-0b2", "medium-0b3", "medium-omat-0", "mh-1")


def _conversion_cache_root() -> Path:
    env = os.environ.get("MACE_MLX_CACHE_DIR")
    if env:
        return Path(env).expanduser()
    return Path.home() / ".cache" / "mace_mlx"


def _resolve_device(device) -> torch.device:
    if isinstance(device, torch.device):
        return device
    if isinstance(device, int):
        return torch.device("cuda", device)
    d = str(device or "cuda").lower()
    if d in ("gpu", "cuda", "mps", ""):
        return torch.device("cuda", torch.cuda.current_device() if torch.cuda.is_available() else 0)
    if d.startswith("cuda:") or d.startswith("gpu:"):
        return torch.device("cuda", int(d.split(":", 1)[1]))
    if d == "cpu":
        raise ValueError("device='cpu' is not supported: this MACE build computes on a CUDA GPU only")
    raise ValueError(f"unknown device {device!r}")


class MACEMLXCalculator(Calculator):
    """ASE calculator computing MACE energy, forces and stress on a B200."""

    implemented_properties = ["energy", "energies", "free_energy", "node_energy", "forces", "stress"]
    _converted_cache: dict[str, str] = {}

    def __init__(self, model_path: str | None = None, device="cuda", default_dtype: str = "float32",
                 head: str | None = None, skin: float = 0.5, use_compile: bool = True, **kwargs):
        if model_path is None:
            model_path = kwargs.pop("model_paths", None)
            if isinstance(model_path, (list, tuple)):
                if len(model_path) > 1:
                    raise NotImplementedError(
                        "committee models are not supported; "
                        f"got {len(model_path)} model paths. Pass a single model."
                    )
                model_path = model_path[0] if model_path else None
        if model_path is None:
            model_path = "medium-mpa-0"
        if default_dtype == "float64":
            warnings.warn(
                "float64 is not computed on this build; falling back to float32. "
                "Energies/forces will differ from mace-torch's float64 default at "
                "the float32 precision level."
            )
            default_dtype = "float32"
        if default_dtype != "float32":
            raise NotImplementedError(f"default_dtype={default_dtype!r} is not supported (float32 only)")
        super().__init__(**kwargs)
        self._device = _resolve_device(device)
        model_dir = self._resolve_model(str(model_path))
        # multi-head models: the named head, else the first (an unknown name raises ValueError)
        self.model = MACEModel(model_dir, device=self._device, head=head)
        self._head = self.model.head if len(self.model.heads) > 1 else head
        self.r_max = float(self.model.r_max)
        self.z_table = self.model.z_table
        self._skin = float(skin)
        self._use_compile = use_compile
        # use_compile=True (the reference's default: mx.compile of the step) maps
        # to CUDA-graph replay of the kernel sequence
        self._use_graph = bool(use_compile)
        self._nl_cache: EdgeSet | None = None
        self._cache_positions = None
        self._cache_cell = None
        self._cache_pbc = None
        self._cache_natoms = 0
        self._cached_numbers = None
        self._species_dev = None
        self._graph_ptr_dev = None
        self._stress_always = False
        self._out = None
        self._host = None
        self._blk = self._hblk = None

    # ------------------------------------------------------------------
    @classmethod
    def _resolve_model(cls, model_path: str) -> str:
        is_named = model_path.startswith("off-") or model_path in _NAMED
        if not is_named:
            return model_path
        if model_path in cls._converted_cache and Path(cls._converted_cache[model_path]).exists():
            return cls._converted_cache[model_path]
        target = _conversion_cache_root() / model_path / f"v{_CONVERTER_CACHE_VERSION}"
        if (target / "config.json").exists() and (target / "weights.npz").exists():
            cls._converted_cache[model_path] = str(target)
            return str(target)
        raise FileNotFoundError(
            f"named model {model_path!r} is not in the converted-model cache ({target}). "
            "Convert it once with the reference's converter (needs torch + mace-torch and a "
            "download) or pass the path of a converted config.json + weights.npz directory."
        )

    # ------------------------------------------------------------------
    def _needs_neighbor_update(self, atoms) -> bool:
        if self._nl_cache is None:
            return True
        if len(atoms) != self._cache_natoms:
            return True
        if not np.array_equal(atoms.pbc, self._cache_pbc):
            return True
        # np.allclose(cell, cached, atol=1e-10) written out (it costs tens of us per call)
        cell = np.asarray(atoms.cell, dtype=np.float64)
        if not bool(np.all(np.abs(cell - self._cache_cell) <= 1e-10 + 1e-5 * np.abs(self._cache_cell))):
            return True
        if self._skin <= 0:
            return True
        d = atoms.positions - self._cache_positions
        return float(np.einsum("ij,ij->i", d, d).max(initial=0.0)) > (self._skin / 2) ** 2

    def _species(self, atoms):
        numbers = atoms.get_atomic_numbers()
        if self._species_dev is None or self._cached_numbers is None or not np.array_equal(numbers, self._cached_numbers):
            idx = self.model.species_index(numbers)
            self._species_dev = torch.as_tensor(idx, device=self._device)
            self._cached_numbers = numbers.copy()
            self._graph_ptr_dev = torch.tensor([0, len(numbers)], dtype=torch.int32, device=self._device)
        return self._species_dev

    @staticmethod
    def _views(n: int, blk_in: torch.Tensor, blk_out: torch.Tensor) -> dict:
        """Named views of the input block (cell, positions) and the output block
        (energy, virial, forces, node energies), each starting 64-byte aligned."""
        f_off = 128
        ne_off = (f_off + 12 * n + 63) // 64 * 64
        return {
            "cell": blk_in[0:9].view(3, 3),
            "pos": blk_in[16:16 + 3 * n].view(n, 3),
            "energy": blk_out[0:8].view(torch.float64),
            "virial": blk_out[8:80].view(torch.float64),
            "forces": blk_out[f_off:f_off + 12 * n].view(torch.float32).view(n, 3),
            "node_energy": blk_out[ne_off:ne_off + 4 * n].view(torch.float32),
        }

    def _buffers(self, n: int, stress: bool):
        # inputs and outputs each in one block, so a step moves one host->device
        # and one device->host copy
        if self._out is None or self._out["node_energy"].shape[0] != n:
            dev = self._device
            n_in = 16 + 3 * n
            n_out = (128 + 12 * n + 63) // 64 * 64 + 4 * n
            self._blk = (torch.empty(n_in, dtype=torch.float32, device=dev),
                         torch.empty(n_out, dtype=torch.uint8, device=dev))
            self._hblk = (torch.empty(n_in, dtype=torch.float32, pin_memory=True),
                          torch.empty(n_out, dtype=torch.uint8, pin_memory=True))
            self._out = self._views(n, *self._blk)
            self._host = self._views(n, *self._hblk)
        return self._out, self._host

    # ------------------------------------------------------------------
    def calculate(self, atoms=None, properties=None, system_changes=all_changes):
        super().calculate(atoms, properties, system_changes)
        atoms = self.atoms if atoms is None else atoms
        dev = self._device
        n = len(atoms)
        with torch.cuda.device(dev):
            species = self._species(atoms)
            has_cell = atoms.cell.rank > 0
            out, host = self._buffers(n, False)
            # host -> device: positions (float32) and cell, one copy
            host["pos"].numpy()[:] = atoms.positions
            pos = out["pos"]
            cell = None
            if has_cell:
                host["cell"].numpy()[:] = np.asarray(atoms.cell)
                cell = out["cell"]
            self._blk[0].copy_(self._hblk[0], non_blocking=True)
            if self._needs_neighbor_update(atoms):
                pos64 = torch.as_tensor(atoms.positions, dtype=torch.float64).to(dev)
                cell64 = torch.as_tensor(np.array(atoms.cell), dtype=torch.float64).to(dev) if has_cell else None
                self._nl_cache = self.model.neighbour_list(pos64, cell64, atoms.pbc, self._graph_ptr_dev,
                                                           self.r_max + self._skin, self._nl_cache)
                self._cache_positions = atoms.positions.copy()
                self._cache_cell = np.array(atoms.cell, dtype=np.float64)
                self._cache_pbc = np.array(atoms.pbc).copy()
                self._cache_natoms = n
            if properties is not None and "stress" in properties and atoms.cell.rank == 3:
                self._stress_always = True
            compute_stress = "stress" in (properties or self.implemented_properties)
            compute_stress = (compute_stress or self._stress_always) and atoms.cell.rank == 3
            # replayed as a CUDA graph: every buffer here keeps its address between steps
            self.model.evaluate(pos, cell, species, self._graph_ptr_dev, self._nl_cache, forces=True,
                                virial=compute_stress, out=out, graph=self._use_graph)
            # device -> host: energy, virial, forces and node energies in one copy
            self._hblk[1].copy_(self._blk[1], non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
        energy = float(host["energy"][0])
        self.results["energy"] = energy
        self.results["free_energy"] = energy
        self.results["forces"] = host["forces"].numpy().copy()
        self.results["node_energy"] = host["node_energy"].numpy().copy()
        self.results["energies"] = self.results["node_energy"]
        if compute_stress:
            g = host["virial"].numpy().reshape(3, 3).astype(np.float64)
            s = 0.5 * (g + g.T) / abs(np.linalg.det(np.array(atoms.cell, dtype=np.float64)))
            self.results["stress"] = s[[0, 1, 2, 1, 0, 0], [0, 1, 2, 2, 2, 1]]

    def calculate_batch(self, atoms_list, properties=("energy", "forces")) -> list[dict]:
        """Energies and forces of several structures in one step on the GPU.

        The structures become the graphs of one system (no edges between
        them): one neighbour list and one ``mace_forward_backward`` for the
        whole batch, which keeps the GPU busy where one small structure per
        step would not (NEB images, adsorption scans, active-learning pools).
        They must be non-periodic or share one cell and pbc (``batch_layout``).
        Returns, per structure, the keys ``calculate`` fills except stress
        (the step accumulates one virial for the whole batch): energy,
        free_energy, forces, node_energy, energies.  ``self.results`` and the
        cached neighbour list of ``calculate`` are left untouched.
        """
        if "stress" in properties:
            raise NotImplementedError("calculate_batch gives energies and forces; call calculate() for stress")
        lay = batch_layout(atoms_list)
        dev = self._device
        gp = lay["graph_ptr"]
        with torch.cuda.device(dev):
            species = torch.as_tensor(self.model.species_index(lay["numbers"]).astype(np.int32), device=dev)
            gp_dev = torch.as_tensor(gp, device=dev)
            pos64 = torch.as_tensor(lay["positions"], dtype=torch.float64).to(dev)
            cell64 = None if lay["cell"] is None else torch.as_tensor(lay["cell"], dtype=torch.float64).to(dev)
            edges = self.model.neighbour_list(pos64, cell64, lay["pbc"], gp_dev, self.r_max)
            out = self.model.evaluate(pos64.float(), None if cell64 is None else cell64.float(), species, gp_dev,
                                      edges, forces=True, virial=False)
            energy = out["energy"].cpu().numpy()
            forces = out["forces"].cpu().numpy()
            node_energy = out["node_energy"].cpu().numpy()
        results = []
        for g in range(len(gp) - 1):
            a, b = int(gp[g]), int(gp[g + 1])
            results.append({"energy": float(energy[g]), "free_energy": float(energy[g]),
                            "forces": forces[a:b].copy(), "node_energy": node_energy[a:b].copy(),
                            "energies": node_energy[a:b].copy()})
        return results


def batch_layout(atoms_list) -> dict:
    """Concatenation of several structures into one system of len(atoms_list) graphs.

    The structures must all be non-periodic (a batch of molecules) or share
    one cell and pbc (NEB images, replicas of one cell): the step's neighbour
    list and edge vectors use a single cell.  Returns graph_ptr (int32),
    numbers, positions (float64), cell (3x3 float64 or None) and pbc.
    """
    if len(atoms_list) == 0:
        raise ValueError("calculate_batch needs at least one structure")
    first = atoms_list[0]
    pbc = np.array(first.pbc, dtype=bool).reshape(-1)
    pbc = np.repeat(pbc, 3) if pbc.size == 1 else pbc
    cell = np.asarray(first.cell, dtype=np.float64)
    periodic = bool(pbc.any())
    for k, a in enumerate(atoms_list[1:], start=1):
        pk = np.array(a.pbc, dtype=bool).reshape(-1)
        pk = np.repeat(pk, 3) if pk.size == 1 else pk
        if not np.array_equal(pk, pbc):
            raise ValueError(f"calculate_batch: structure {k} has pbc {pk.tolist()}, structure 0 {pbc.tolist()}; "
                             "a batch shares one cell and pbc")
        if periodic and not np.array_equal(np.asarray(a.cell, dtype=np.float64), cell):
            raise ValueError(f"calculate_batch: structure {k} has another cell than structure 0; "
                             "a periodic batch shares one cell")
    sizes = np.array([len(a) for a in atoms_list], dtype=np.int64)
    return {
        "graph_ptr": np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32),
        "numbers": np.concatenate([np.asarray(a.get_atomic_numbers(), dtype=np.int64) for a in atoms_list]),
        "positions": np.concatenate([np.asarray(a.positions, dtype=np.float64).reshape(-1, 3) for a in atoms_list]),
        "cell": cell if periodic else None,
        "pbc": pbc,
    }


def mace_mp(model: str | None = None, device="cuda", default_dtype: str = "float32", head: str | None = None,
            dispersion: bool = False, return_raw_model: bool = False, **kwargs) -> MACEMLXCalculator:
    """MACE-MP foundation-model calculator (drop-in for ``mace.calculators.mace_mp``)."""
    if return_raw_model:
        raise NotImplementedError("return_raw_model is not supported")
    if dispersion:
        warnings.warn("D3 dispersion corrections are not supported. Ignoring dispersion=True.")
    for key in ("damping", "dispersion_xc", "dispersion_cutoff"):
        kwargs.pop(key, None)
    return MACEMLXCalculator(model_path=model, device=device, default_dtype=default_dtype, head=head, **kwargs)


def mace_off(model: str = "small", device="cuda", default_dtype: str = "float32", **kwargs) -> MACEMLXCalculator:
    """MACE-OFF organic force-field calculator (drop-in for ``mace.calculators.mace_off``)."""
    return MACEMLXCalculator(model_path=f"off-{model}", device=device, default_dtype=default_dtype, **kwargs)


def mace_anicc(**kwargs):
    raise NotImplementedError("mace_anicc is not supported. Use mace-torch for ANI models.")


def mace_omol(**kwargs):
    raise NotImplementedError("mace_omol is not supported. Use mace-torch for OMOL models.")


MACECalculator = MACEMLXCalculator
