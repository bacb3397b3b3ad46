"""Multi-GPU execution: spatial domain decomposition and structure sharding.

One process per GPU (``torch.distributed``, NCCL over NVLink on the B200
box, gloo on the CPU for the tests).

Spatial decomposition (large periodic systems): the cell is cut into a
``px x py x pz`` grid of domains in fractional coordinates.  Each rank owns
the atoms of its domain and holds, as ghosts, every periodic image of every
atom within ``ghost_width`` of the domain (2 x r_max for two interaction
layers, plus the neighbour-list skin so the ghost set stays valid while atoms
move less than skin / 2).  The rank evaluates the whole model on owned +
ghost atoms as one open (non-periodic) system with the positions unwrapped,
with energy weight 1 on owned and 0 on ghost atoms, so its energy is exactly
the sum of its owned atoms' energies and its gradient is that sum's gradient
with respect to every local atom.  Per step:

  * positions: owned positions are all-gathered (``all_gather``) and each
    rank gathers its local atoms' images (position + integer shift @ cell);
  * forces: local forces are scattered by global atom index and summed over
    ranks (``all_reduce``), which is the reverse halo reduction of the ghost
    contributions onto their owners;
  * energy and virial: ``all_reduce`` of 1 and 9 numbers.

No ghost features are exchanged between layers: the 2 x r_max ghost shell
makes every owned atom's two-layer receptive field local (the alternative the
survey lists, chosen because it needs one position exchange per step instead
of one feature exchange per layer).

Structure sharding (batches of small molecules): ``shard_structures`` assigns
whole structures to ranks, balancing atoms; no data-path collective.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


def grid_for(world: int) -> tuple[int, int, int]:
    """Domain grid (px, py, pz) for `world` ranks, splitting z first, then y, then x."""
    g = [1, 1, 1]
    rest = world
    axis = 2
    for p in _prime_factors(world):
        g[axis] *= p
        rest //= p
        axis = (axis - 1) % 3
    return g[0], g[1], g[2]


def _prime_factors(n: int) -> list[int]:
    out, p = [], 2
    while n > 1:
        while n % p == 0:
            out.append(p)
            n //= p
        p += 1
    return sorted(out, reverse=True)


def shard_structures(sizes, world: int) -> list[list[int]]:
    """Whole structures per rank, greedy by size (largest first onto the lightest rank)."""
    loads = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(sizes)), key=lambda k: -sizes[k]):
        r = min(range(world), key=lambda q: loads[q])
        out[r].append(i)
        loads[r] += sizes[i]
    return [sorted(o) for o in out]


@dataclass
class DomainPlan:
    """Local atoms of one rank: owned first (ascending global index), then ghosts.

    The local system stays periodic along the axes the grid does not split
    (``pbc``) and is open along the split ones, where the ghosts are.
    """

    rank: int
    grid: tuple[int, int, int]
    local_index: np.ndarray  # (n_local,) int64 global atom of each local atom
    local_shift: np.ndarray  # (n_local, 3) int64: local position = pos[g] + shift @ cell
    n_owned: int
    pbc: tuple[bool, bool, bool] = (False, False, False)

    @property
    def n_local(self) -> int:
        return len(self.local_index)

    @property
    def owned_index(self) -> np.ndarray:
        return self.local_index[: self.n_owned]


def plane_spacings(cell: np.ndarray) -> np.ndarray:
    """Distance between adjacent lattice planes along each fractional axis."""
    cell = np.asarray(cell, dtype=np.float64)
    vol = abs(np.linalg.det(cell))
    return np.array([vol / np.linalg.norm(np.cross(cell[(d + 1) % 3], cell[(d + 2) % 3])) for d in range(3)])


def domain_of(positions: np.ndarray, cell: np.ndarray, grid: tuple[int, int, int]) -> np.ndarray:
    """Owning rank of every atom: (ix * py + iy) * pz + iz of its wrapped fractional position."""
    f = np.asarray(positions, dtype=np.float64) @ np.linalg.inv(np.asarray(cell, dtype=np.float64))
    u = f - np.floor(f)
    u = np.where(u >= 1.0, 0.0, u)
    p = np.asarray(grid)
    idx3 = np.minimum((u * p).astype(np.int64), p - 1)
    return (idx3[:, 0] * p[1] + idx3[:, 1]) * p[2] + idx3[:, 2]


def plan_domain(positions: np.ndarray, cell: np.ndarray, grid: tuple[int, int, int], rank: int,
                ghost_width: float) -> DomainPlan:
    """Owned atoms and ghost images of domain `rank` of a fully periodic cell.

    Domain (ix, iy, iz) with rank = (ix * py + iy) * pz + iz covers fractional
    coordinates [i_d / p_d, (i_d + 1) / p_d) of the wrapped positions.  Along
    the split axes (p_d > 1) the ghosts are the images (shift k_d in
    {-1, 0, 1}) of all atoms whose wrapped fractional coordinate falls within
    ghost_width / spacing_d of the domain, owned copies excluded; the unsplit
    axes stay periodic in the local system and need no ghosts.
    """
    pos = np.asarray(positions, dtype=np.float64)
    cell = np.asarray(cell, dtype=np.float64)
    inv = np.linalg.inv(cell)
    f = pos @ inv
    w = np.floor(f)
    u = f - w
    u = np.where(u >= 1.0, 0.0, u)  # guard against rounding to exactly 1
    p = np.asarray(grid)
    idx3 = np.minimum((u * p).astype(np.int64), p - 1)
    ix, iy, iz = rank // (p[1] * p[2]), (rank // p[2]) % p[1], rank % p[2]
    me = np.array([ix, iy, iz])
    owned_mask = np.all(idx3 == me, axis=1)
    lo = me / p
    hi = (me + 1) / p
    split = p > 1
    gw = ghost_width / plane_spacings(cell)
    if np.any(gw[split] >= 1.0):
        # images with |k| > 1 would be needed
        raise ValueError(f"cell thinner than the {ghost_width:.2f} A ghost shell")
    owned = np.nonzero(owned_mask)[0]
    ghosts, shifts = [], []
    ks = [[-1, 0, 1] if split[d] else [0] for d in range(3)]
    for k in np.array(np.meshgrid(*ks, indexing="ij")).reshape(3, -1).T:
        uk = u + k
        inside = np.all(((uk >= lo - gw) & (uk < hi + gw)) | ~split, axis=1)
        if not np.any(k):
            inside &= ~owned_mask
        sel = np.nonzero(inside)[0]
        ghosts.append(sel)
        shifts.append(np.broadcast_to(k, (len(sel), 3)))
    ghosts_a = np.concatenate(ghosts)
    shifts_a = np.concatenate(shifts).astype(np.int64)
    order = np.lexsort((shifts_a[:, 2], shifts_a[:, 1], shifts_a[:, 0], ghosts_a))
    ghosts_a, shifts_a = ghosts_a[order], shifts_a[order]
    local_index = np.concatenate([owned, ghosts_a]).astype(np.int64)
    # local position = pos[g] + (k - w_g) @ cell  (the image of the wrapped atom)
    local_shift = np.concatenate([-w[owned], shifts_a - w[ghosts_a]]).astype(np.int64)
    return DomainPlan(rank, tuple(int(x) for x in p), local_index, local_shift, len(owned),
                      tuple(bool(not x) for x in split))


class SpatialRunner:
    """Energy, forces and virial of one periodic structure on all ranks of `group`.

    Every rank calls ``evaluate`` with the current positions of the atoms it
    owns (plus, on the first call, the full structure to plan the domains).
    The neighbour list and the ghost set are rebuilt when any local atom has
    moved more than skin / 2 since the last build (the reference's rule).
    """

    def __init__(self, model, numbers, cell, world: int, rank: int, *, skin: float = 0.5, group=None,
                 ghost_width: float | None = None, halo: bool = True):
        """halo=True: ghost shell r_max + skin and node features exchanged between
        layers (HaloExchange); halo=False: ghost shell 2 r_max + skin, no exchange
        between layers (each rank recomputes its ghosts' first layer)."""
        import torch

        self.model = model
        self.torch = torch
        self.world, self.rank, self.group = world, rank, group
        self.grid = grid_for(world)
        self.cell = np.asarray(cell, dtype=np.float64)
        self.numbers = np.asarray(numbers)
        self.species_all = model.species_index(self.numbers)
        self.skin = float(skin)
        self.use_halo = bool(halo) and world > 1 and model.spec.num_interactions > 1
        layers = 1 if self.use_halo else model.spec.num_interactions
        self.ghost_width = float(ghost_width if ghost_width is not None else layers * model.r_max + self.skin)
        self.halo = None
        self.r_cut = model.r_max + self.skin
        self.plan: DomainPlan | None = None
        self.edges = None
        self.dev = model.device
        self.cell_dev = torch.tensor(self.cell, dtype=torch.float64, device=self.dev)
        self.volume = abs(np.linalg.det(self.cell))

    # -- planning ------------------------------------------------------
    def _rebuild(self, pos_global64):
        torch = self.torch
        dev = self.dev
        pos_host = pos_global64.cpu().numpy()
        self.plan = plan_domain(pos_host, self.cell, self.grid, self.rank, self.ghost_width)
        pl = self.plan
        if self.use_halo:
            self.halo = HaloExchange(pl, domain_of(pos_host, self.cell, self.grid), self.world, dev, self.group)
        if pl.n_local == pl.n_owned:  # one domain: the periodic structure itself
            self.weight = None
        else:
            self.weight = torch.zeros(pl.n_local, dtype=torch.float32, device=dev)
            self.weight[: pl.n_owned] = 1.0
        pbc = pl.pbc
        cell = self.cell_dev if any(pbc) else None
        self.li = torch.as_tensor(pl.local_index, device=dev)
        self.ls = torch.as_tensor(pl.local_shift, dtype=torch.float64, device=dev)
        self.species = torch.as_tensor(self.species_all[pl.local_index], device=dev)
        self.graph_ptr = torch.tensor([0, pl.n_local], dtype=torch.int32, device=dev)
        loc = self._local(pos_global64)
        self.edges = self.model.neighbour_list(loc, cell, pbc, self.graph_ptr, self.r_cut, edges=self.edges)
        self.cell32 = self.cell_dev.float() if any(pbc) else None
        self.ref_pos = loc.clone()
        self.out = None

    def _local(self, pos_global64):
        return pos_global64[self.li] + self.ls @ self.cell_dev

    def needs_rebuild(self, loc64) -> bool:
        if self.plan is None:
            return True
        torch = self.torch
        disp = (loc64 - self.ref_pos).norm(dim=1).max()
        flag = (disp > 0.5 * self.skin).to(torch.int32).reshape(1)
        if self.world > 1:
            torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MAX, group=self.group)
        return bool(flag.item())

    # -- one step ------------------------------------------------------
    def evaluate(self, pos_global64, *, virial: bool = False) -> dict:
        """pos_global64: (N, 3) float64 device positions of all atoms (after the position exchange)."""
        torch = self.torch
        if self.plan is None:
            self._rebuild(pos_global64)
        else:
            loc = self._local(pos_global64)
            if self.needs_rebuild(loc):
                self._rebuild(pos_global64)
        loc = self._local(pos_global64)
        self.out = self.model.evaluate(loc.float(), self.cell32, self.species, self.graph_ptr, self.edges,
                                       forces=True, virial=virial, out=self.out, energy_weight=self.weight,
                                       halo=self.halo)
        return self.out

    def reduce(self, out: dict, n_atoms: int, *, virial: bool = False) -> dict:
        """Sum energy, forces (scattered by global index) and virial over the ranks."""
        return reduce_local(self.li, out, n_atoms, self.world, virial=virial, group=self.group)


def reduce_local(local_index, out: dict, n_atoms: int, world: int, *, virial: bool = False, group=None) -> dict:
    """Global energy, forces and virial from every rank's local results.

    Forces of local atoms (owned and ghost images) are added into an (n_atoms, 3)
    array by global index and summed over the ranks: the reverse halo
    reduction.  Energies (owned atoms only, by the energy weights) and virials
    are plain sums.
    """
    import torch

    f_loc = out["forces"]
    forces = torch.zeros(n_atoms, 3, dtype=f_loc.dtype, device=f_loc.device)
    forces.index_add_(0, torch.as_tensor(local_index, device=f_loc.device), f_loc)
    scal = out["energy"].clone()
    vir = out["virial"].clone() if virial else None
    if world > 1:
        dist = torch.distributed
        dist.all_reduce(forces, group=group)
        dist.all_reduce(scal, group=group)
        if virial:
            dist.all_reduce(vir, group=group)
    res = {"energy": scal, "forces": forces}
    if virial:
        res["virial"] = vir
    return res


class HaloExchange:
    """Ghost rows of node features (forward) and their gradients (backward) over NCCL.

    Built from a rank's plan: its ghosts, grouped by owning rank, are
    requested from their owners once per neighbour-list rebuild (an
    ``all_to_all`` of global atom ids); then per step
      features:  owners send the rows of the requested atoms, ghosts take them;
      gradients: ghosts send their rows back, owners add them, ghosts are zeroed.
    Both are one ``all_to_all_single`` with uneven splits.  Images of a rank's
    own atoms go through the same path as a copy to itself.
    """

    def __init__(self, plan: DomainPlan, owner_of: np.ndarray, world: int, device, group=None):
        import torch
        import torch.distributed as dist

        self.torch, self.dist, self.group = torch, dist, group
        gid = plan.local_index[plan.n_owned:]
        own = owner_of[gid]
        order = np.argsort(own, kind="stable")
        self.ghost_rows = torch.as_tensor(plan.n_owned + order, device=device)
        self.recv_counts = np.bincount(own, minlength=world).tolist()
        rc = torch.tensor(self.recv_counts, dtype=torch.int64, device=device)
        sc = torch.empty_like(rc)
        dist.all_to_all_single(sc, rc, group=group)
        self.send_counts = sc.cpu().tolist()
        ids_out = torch.as_tensor(np.ascontiguousarray(gid[order]), device=device)
        ids_in = torch.empty(sum(self.send_counts), dtype=torch.int64, device=device)
        dist.all_to_all_single(ids_in, ids_out, output_split_sizes=self.send_counts,
                               input_split_sizes=self.recv_counts, group=group)
        owned = plan.local_index[: plan.n_owned]  # ascending global ids
        want = ids_in.cpu().numpy()
        rows = np.searchsorted(owned, want)
        if np.any(rows >= len(owned)) or np.any(owned[np.minimum(rows, len(owned) - 1)] != want):
            raise RuntimeError("halo request for an atom this rank does not own")
        self.send_rows = torch.as_tensor(rows, device=device)

    def features(self, rows):
        torch = self.torch
        send = rows.index_select(0, self.send_rows)
        recv = torch.empty(len(self.ghost_rows), rows.shape[1], dtype=rows.dtype, device=rows.device)
        self.dist.all_to_all_single(recv, send, output_split_sizes=self.recv_counts,
                                    input_split_sizes=self.send_counts, group=self.group)
        rows.index_copy_(0, self.ghost_rows, recv)

    def gradients(self, rows):
        torch = self.torch
        send = rows.index_select(0, self.ghost_rows)
        recv = torch.empty(len(self.send_rows), rows.shape[1], dtype=rows.dtype, device=rows.device)
        self.dist.all_to_all_single(recv, send, output_split_sizes=self.send_counts,
                                    input_split_sizes=self.recv_counts, group=self.group)
        rows.index_add_(0, self.send_rows, recv)
        rows.index_fill_(0, self.ghost_rows, 0.0)

    def __call__(self, phase: int, layer: int, rows):
        (self.features if phase == 0 else self.gradients)(rows)


class PositionExchange:
    """All-gather of owned positions into the global array (ranks own different counts)."""

    def __init__(self, owned_index_per_rank: list[np.ndarray], device, group=None):
        import torch

        self.torch = torch
        self.group = group
        self.counts = [len(o) for o in owned_index_per_rank]
        self.cap = max(self.counts)
        perm = np.concatenate([np.concatenate([o, -np.ones(self.cap - len(o), np.int64)])
                               for o in owned_index_per_rank])
        keep = perm >= 0
        self.src = torch.as_tensor(np.nonzero(keep)[0], device=device)
        self.dst = torch.as_tensor(perm[keep], device=device)
        self.buf = torch.empty(len(owned_index_per_rank) * self.cap, 3, dtype=torch.float64, device=device)

    def __call__(self, owned_pos64, out64):
        torch = self.torch
        send = torch.zeros(self.cap, 3, dtype=torch.float64, device=owned_pos64.device)
        send[: owned_pos64.shape[0]] = owned_pos64
        torch.distributed.all_gather_into_tensor(self.buf, send, group=self.group)
        out64[self.dst] = self.buf[self.src]
        return out64


__all__ = ["grid_for", "shard_structures", "DomainPlan", "domain_of", "plan_domain", "plane_spacings",
           "SpatialRunner", "HaloExchange", "PositionExchange", "reduce_local"]
