"""Seeded synthetic structures with the shapes of the benchmark configurations.

No dataset is involved: every structure is generated from a numpy seed.

* ``diamond_si(reps, sigma, seed)`` -- diamond Si (a = 5.43 A), conventional
  8-atom cell repeated ``reps`` times per axis, Gaussian rattle.
* ``lipso_box(n, seed)`` -- cubic periodic box of Li/P/S/O in 3:1:4:0.5 number
  ratio, density 0.06 atoms/A^3, uniform positions with 1.8 A rejection.
* ``molecule_batch(n_mol, seed)`` -- non-periodic random-walk C/N/O chains
  with hydrogens, 20-60 atoms each, 1.0 A minimum separation.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

SI_A = 5.43
_DIAMOND_FRAC = np.array(
    [
        [0.0, 0.0, 0.0], [0.0, 0.5, 0.5], [0.5, 0.0, 0.5], [0.5, 0.5, 0.0],
        [0.25, 0.25, 0.25], [0.25, 0.75, 0.75], [0.75, 0.25, 0.75], [0.75, 0.75, 0.25],
    ]
)


@dataclass
class Structure:
    positions: np.ndarray  # (N, 3) float64
    numbers: np.ndarray  # (N,) int
    cell: np.ndarray = field(default_factory=lambda: np.zeros((3, 3)))
    pbc: np.ndarray = field(default_factory=lambda: np.zeros(3, dtype=bool))
    batch: np.ndarray | None = None  # (N,) graph index for batches of molecules

    def __len__(self) -> int:
        return len(self.numbers)

    @property
    def num_graphs(self) -> int:
        return 1 if self.batch is None else int(self.batch.max()) + 1


def diamond_si(reps, sigma: float, seed: int) -> Structure:
    """``reps`` conventional cells per axis (an int, or three ints)."""
    nx, ny, nz = (reps, reps, reps) if np.ndim(reps) == 0 else tuple(int(x) for x in reps)
    grid = np.stack(np.meshgrid(np.arange(nx), np.arange(ny), np.arange(nz), indexing="ij"), -1).reshape(-1, 3)
    frac = (grid[:, None, :] + _DIAMOND_FRAC[None]).reshape(-1, 3)
    pos = frac * SI_A
    rng = np.random.default_rng(seed)
    pos = pos + rng.normal(0.0, sigma, size=pos.shape)
    cell = np.diag([nx, ny, nz]).astype(np.float64) * SI_A
    return Structure(pos, np.full(len(pos), 14), cell, np.ones(3, dtype=bool))


def _min_dist_ok(cand, cells, cell_of, pos, rmin, L, ncell):
    c = np.floor(cand / L * ncell).astype(int) % ncell
    for dx in (-1, 0, 1):
        for dy in (-1, 0, 1):
            for dz in (-1, 0, 1):
                key = ((c[0] + dx) % ncell, (c[1] + dy) % ncell, (c[2] + dz) % ncell)
                for j in cells.get(key, ()):
                    d = pos[j] - cand
                    d -= L * np.round(d / L)
                    if d @ d < rmin * rmin:
                        return False, c
    return True, c


def lipso_box(n: int = 8000, seed: int = 2, density: float = 0.06, rmin: float = 1.8) -> Structure:
    ratio = np.array([3.0, 1.0, 4.0, 0.5])
    counts = np.floor(ratio / ratio.sum() * n).astype(int)
    counts[np.argmax(ratio)] += n - counts.sum()
    rng = np.random.default_rng(seed)
    numbers = np.repeat(np.array([3, 15, 16, 8]), counts)
    numbers = numbers[rng.permutation(n)]
    L = (n / density) ** (1.0 / 3.0)
    ncell = max(1, int(L / rmin))
    pos = np.zeros((n, 3))
    cells: dict = {}
    i = 0
    while i < n:
        cand = rng.uniform(0.0, L, size=3)
        ok, c = _min_dist_ok(cand, cells, None, pos[:i], rmin, L, ncell)
        if ok:
            pos[i] = cand
            cells.setdefault(tuple(c), []).append(i)
            i += 1
    return Structure(pos, numbers, np.eye(3) * L, np.ones(3, dtype=bool))


def _molecule(rng, n_atoms: int) -> tuple[np.ndarray, np.ndarray]:
    n_heavy = max(2, int(round(n_atoms * 0.45)))
    n_h = n_atoms - n_heavy
    heavy_z = rng.choice([6, 7, 8], size=n_heavy, p=[0.7, 0.15, 0.15])
    pos = [np.zeros(3)]
    while len(pos) < n_heavy:
        base = pos[-1]
        for _ in range(200):
            v = rng.normal(size=3)
            v /= np.linalg.norm(v)
            cand = base + v * rng.uniform(1.2, 1.5)
            if min(np.linalg.norm(np.array(pos) - cand, axis=1)) >= 1.0 - 1e-12:
                pos.append(cand)
                break
        else:  # restart from a random earlier atom when the walk is boxed in
            pos.append(pos[rng.integers(len(pos))] + rng.normal(size=3) * 3.0)
    zs = list(heavy_z)
    for _ in range(n_h):
        for _ in range(500):
            j = rng.integers(n_heavy)
            v = rng.normal(size=3)
            v /= np.linalg.norm(v)
            cand = pos[j] + v * rng.uniform(1.0, 1.1)
            if min(np.linalg.norm(np.array(pos) - cand, axis=1)) >= 1.0:
                pos.append(cand)
                zs.append(1)
                break
        else:
            raise RuntimeError("could not place hydrogen")
    return np.array(pos), np.array(zs)


def molecule_batch(n_mol: int = 512, seed: int = 3, n_min: int = 20, n_max: int = 60) -> Structure:
    rng = np.random.default_rng(seed)
    P, Z, B = [], [], []
    for g in range(n_mol):
        p, z = _molecule(rng, int(rng.integers(n_min, n_max + 1)))
        P.append(p)
        Z.append(z)
        B.append(np.full(len(z), g))
    return Structure(np.concatenate(P), np.concatenate(Z), np.zeros((3, 3)),
                     np.zeros(3, dtype=bool), np.concatenate(B))


def config_structure(cfg: int) -> Structure:
    """Structure of benchmark configuration ``cfg`` (0..4)."""
    if cfg == 0:
        return diamond_si(3, 0.01, 0)
    if cfg == 1:
        return diamond_si(5, 0.05, 1)
    if cfg == 2:
        return lipso_box(8000, 2)
    if cfg == 3:
        return molecule_batch(512, 3)
    if cfg == 4:
        return diamond_si(50, 0.05, 4)
    raise ValueError(cfg)
