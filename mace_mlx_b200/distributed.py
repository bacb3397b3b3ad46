"""Multi-GPU execution: spatial domain decomposition and structure sharding.

One process per GPU (``torch.distributed``, NCCL over NVLink on the B200
box, gloo on the CPU for the tests).

Spatial decomposition (large periodic systems): the cell is cut into a
``px x py x pz`` grid of domains in fractional coordinates.  Each rank owns
the atoms of its domain and holds, as ghosts, the periodic images of the
atoms within ``ghost_width`` of the domain across the split axes (the local
system stays periodic along unsplit axes).  Local atoms are ordered owned
first, then ghosts.

With ``halo=True`` (the default) the ghost shell is r_max + skin and the
node features are exchanged between the interaction layers: after layer 0
the ghosts' layer-1 input features are overwritten by their owners' rows, and
in the backward the feature gradients gathered on ghost rows are added onto
their owners' rows.  Only owned atoms are receivers (``n_active``): ghost
atoms take part as senders, so no rank repeats another rank's edge work.  On
GPUs with NCCL the exchange runs inside the library (``NativeHaloExchange``:
NCCL send/recv issued on the step's stream, so the whole step, exchange
included, replays as one CUDA graph); otherwise through a host callback with
torch collectives (``HaloExchange``).  With ``halo=False`` the shell is
2 r_max + skin, every local atom is a receiver and nothing is exchanged
between layers.

Per step only halo-sized data moves between ranks: the owners' positions of
the ghost atoms (``GhostExchange.positions``) before the step, the ghost
atoms' forces back to their owners after it (``GhostExchange.forces``), and
the energy and virial (``all_reduce`` of 1 and 9 numbers).  The owned set and
the ghost lists are rebuilt, with one all-gather of the owned positions,
only when some atom has moved more than skin / 2 since the last build (the
reference's rule).

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
    # (n_local, 3) image of each local atom relative to its owner's copy:
    # local position = owner's local position + image @ cell (0 for owned atoms)
    image: np.ndarray | None = None

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
    image = np.concatenate([np.zeros((len(owned), 3), np.int64), shifts_a]).astype(np.int64)
    return DomainPlan(rank, tuple(int(x) for x in p), local_index, local_shift, len(owned),
                      tuple(bool(not x) for x in split), image)


class SpatialRunner:
    """Energy, forces and virial of one periodic structure on all ranks of `group`.

    ``evaluate(pos_global64)`` takes the positions of all atoms (tests, and
    the first call); ``step(own_pos64)`` takes only this rank's owned atoms
    (in ``owned_index`` order) and moves halo-sized data only.  The neighbour
    list, the owned set and the ghost set are rebuilt when any local atom has
    moved more than skin / 2 since the last build (the reference's rule); a
    rebuild during ``step`` all-gathers the owned positions once and may
    change ``owned_index``.
    """

    def __init__(self, model, numbers, cell, world: int, rank: int, *, skin: float = 0.5, group=None,
                 ghost_width: float | None = None, halo: bool = True, native: bool | None = None):
        """halo=True: ghost shell r_max + skin, owned atoms the only receivers, node
        features exchanged between layers (in the library over NCCL when
        ``native``, default: on CUDA with an NCCL process group; else through a
        host callback); halo=False: ghost shell 2 r_max + skin, no exchange
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
        if native is None:
            native = (self.use_halo and torch.device(model.device).type == "cuda"
                      and torch.distributed.is_initialized()
                      and torch.distributed.get_backend(group) == "nccl")
        self.native = bool(native) and self.use_halo
        self.nx = NativeHaloExchange(model, world, rank, group) if self.native else None
        self.halo = None
        self.gx = None
        self.r_cut = model.r_max + self.skin
        self.plan: DomainPlan | None = None
        self.edges = None
        self.dev = model.device
        self.cell_dev = torch.tensor(self.cell, dtype=torch.float64, device=self.dev)
        self.volume = abs(np.linalg.det(self.cell))
        self.graph = False

    # -- planning ------------------------------------------------------
    def _rebuild(self, pos_global64):
        torch = self.torch
        dev = self.dev
        pos_host = pos_global64.detach().cpu().numpy()
        self.plan = plan_domain(pos_host, self.cell, self.grid, self.rank, self.ghost_width)
        pl = self.plan
        self.halo = None
        self.gx = None
        if self.world > 1:
            hp = make_halo_plan(pl, domain_of(pos_host, self.cell, self.grid), self.world, dev, self.group)
            self.gx = GhostExchange(hp, pl, self.cell_dev, self.group)
            if self.use_halo:
                if self.native:
                    self.nx.set_plan(hp, pl.n_owned, pl.n_local, max(self.model.spec.layers[0].hidden.dim,
                                                                     self.model.spec.hidden.dim))
                else:
                    self.halo = HaloExchange(hp, self.group, dev)
        if pl.n_local == pl.n_owned:  # one domain: the periodic structure itself
            self.weight = None
        else:
            self.weight = torch.zeros(pl.n_local, dtype=torch.float32, device=dev)
            self.weight[: pl.n_owned] = 1.0
        pbc = pl.pbc
        cell = self.cell_dev if any(pbc) else None
        self.li = torch.as_tensor(pl.local_index, device=dev)
        self.ls = torch.as_tensor(pl.local_shift, dtype=torch.float64, device=dev)
        self.own_shift = self.ls[: pl.n_owned] @ self.cell_dev
        self.species = torch.as_tensor(self.species_all[pl.local_index], device=dev)
        self.graph_ptr = torch.tensor([0, pl.n_local], dtype=torch.int32, device=dev)
        loc = pos_global64[self.li] + self.ls @ self.cell_dev
        self.loc64 = loc.clone()
        self.edges = self.model.neighbour_list(loc, cell, pbc, self.graph_ptr, self.r_cut, edges=self.edges)
        self.active = None
        if self.use_halo and pl.n_owned < pl.n_local:
            e_active = int(self.edges.row_ptr[pl.n_owned].item())
            self.active = (pl.n_owned, e_active)
        self.cell32 = self.cell_dev.float() if any(pbc) else None
        self.ref_pos = loc.clone()
        self.loc32 = loc.float()
        self.out = None
        # the first step after a (re)plan runs eagerly: NCCL sets up its peer
        # connections on first use, which must not happen inside a graph capture
        self._eager_next = True

    @property
    def owned_index(self) -> np.ndarray:
        return self.plan.owned_index

    def needs_rebuild(self, loc64) -> bool:
        if self.plan is None:
            return True
        torch = self.torch
        n = self.plan.n_owned
        disp = (loc64[:n] - self.ref_pos[:n]).norm(dim=1).max() if n else torch.zeros((), device=loc64.device)
        flag = (disp > 0.5 * self.skin).to(torch.int32).reshape(1)
        if self.world > 1:
            torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MAX, group=self.group)
        return bool(flag.item())

    def _run(self, virial: bool):
        graph = self.graph and self.halo is None and not self._eager_next
        self.out = self.model.evaluate(self.loc32, self.cell32, self.species, self.graph_ptr, self.edges,
                                       forces=True, virial=virial, out=self.out, energy_weight=self.weight,
                                       halo=self.halo, halo_exchange=self.nx if self.native else None,
                                       active=self.active, graph=graph)
        self._eager_next = False
        return self.out

    # -- one step ------------------------------------------------------
    def evaluate(self, pos_global64, *, virial: bool = False) -> dict:
        """pos_global64: (N, 3) float64 device positions of all atoms; local results."""
        if self.plan is None:
            self._rebuild(pos_global64)
        else:
            loc = pos_global64[self.li] + self.ls @ self.cell_dev
            if self.needs_rebuild(loc):
                self._rebuild(pos_global64)
            else:
                self.loc64.copy_(loc)
        self.loc32.copy_(self.loc64)
        return self._run(virial)

    def step(self, own_pos64, *, virial: bool = False, check_skin: bool = True) -> dict:
        """One step from this rank's owned positions (n_owned, 3) float64, in
        ``owned_index`` order: ghost positions from their owners, the model, ghost
        forces back to their owners.  Returns the global energy and virial and the
        owned atoms' forces (float32, ``owned_index`` order)."""
        torch = self.torch
        n = self.plan.n_owned
        own_loc = own_pos64 + self.own_shift
        if check_skin and self.needs_rebuild(torch.cat([own_loc, self.loc64[n:]])):
            # ownership changes: one all-gather of every owned position, then a new plan
            glob = torch.empty(len(self.numbers), 3, dtype=torch.float64, device=self.dev)
            gather_owned(self.plan.owned_index, own_pos64, glob, self.world, self.group)
            self._rebuild(glob)
            return None  # the caller re-reads owned_index and repeats the step
        self.loc64[:n] = own_loc
        if self.gx is not None:
            self.gx.positions(self.loc64)
        self.loc32.copy_(self.loc64)
        out = self._run(virial)
        f_own = self.gx.forces(out["forces"]) if self.gx is not None else out["forces"]
        e = out["energy"].clone()
        vir = out["virial"].clone() if virial else None
        if self.world > 1:
            torch.distributed.all_reduce(e, group=self.group)
            if virial:
                torch.distributed.all_reduce(vir, group=self.group)
        return {"energy": e, "forces": f_own, "virial": vir}

    def reduce(self, out: dict, n_atoms: int, *, virial: bool = False) -> dict:
        """Sum energy, forces (scattered by global index) and virial over the ranks."""
        return reduce_local(self.li, out, n_atoms, self.world, virial=virial, group=self.group)

    def close(self):
        if self.nx is not None:
            self.nx.close()
            self.nx = None


def gather_owned(owned_index, own_pos64, out64, world: int, group=None):
    """All-gather every rank's owned positions into the global (N, 3) array (rebuilds only)."""
    import torch

    if world == 1:
        out64[torch.as_tensor(owned_index, device=out64.device)] = own_pos64
        return out64
    idx = [None] * world
    torch.distributed.all_gather_object(idx, np.asarray(owned_index), group=group)
    cap = max(len(i) for i in idx)
    send = torch.zeros(cap, 3, dtype=torch.float64, device=own_pos64.device)
    send[: own_pos64.shape[0]] = own_pos64
    buf = torch.empty(world * cap, 3, dtype=torch.float64, device=own_pos64.device)
    torch.distributed.all_gather_into_tensor(buf, send, group=group)
    for r, ix in enumerate(idx):
        out64[torch.as_tensor(ix, device=out64.device)] = buf[r * cap: r * cap + len(ix)]
    return out64


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


@dataclass
class HaloPlan:
    """Who sends which rows to whom, per peer rank in rank order.

    send_rows[send_off[p]: ...] are this rank's owned local rows that rank p
    holds as ghosts, in the order p lists them; recv_rows[recv_off[p]: ...] are
    this rank's ghost rows that rank p owns, in the same order as p sends them.
    """

    send_counts: list[int]
    send_rows: np.ndarray
    recv_counts: list[int]
    recv_rows: np.ndarray
    ghost_image: np.ndarray  # (n_recv, 3) image shift of each received ghost row


def make_halo_plan(plan: DomainPlan, owner_of: np.ndarray, world: int, device, group=None) -> HaloPlan:
    """Group this rank's ghosts by owning rank and tell each owner which of its
    atoms are wanted (one ``all_to_all`` of global atom ids), once per rebuild."""
    import torch
    import torch.distributed as dist

    gid = plan.local_index[plan.n_owned:]
    own = owner_of[gid]
    order = np.argsort(own, kind="stable")
    recv_rows = (plan.n_owned + order).astype(np.int32)
    recv_counts = np.bincount(own, minlength=world).tolist()
    rc = torch.tensor(recv_counts, dtype=torch.int64, device=device)
    sc = torch.empty_like(rc)
    dist.all_to_all_single(sc, rc, group=group)
    send_counts = sc.cpu().tolist()
    ids_out = torch.as_tensor(np.ascontiguousarray(gid[order]), device=device)
    ids_in = torch.empty(sum(send_counts), dtype=torch.int64, device=device)
    dist.all_to_all_single(ids_in, ids_out, output_split_sizes=send_counts, input_split_sizes=recv_counts,
                           group=group)
    owned = plan.local_index[: plan.n_owned]  # ascending global ids
    want = ids_in.cpu().numpy()
    rows = np.searchsorted(owned, want)
    if np.any(rows >= len(owned)) or np.any(owned[np.minimum(rows, len(owned) - 1)] != want):
        raise RuntimeError("halo request for an atom this rank does not own")
    image = plan.image[recv_rows] if plan.image is not None else np.zeros((len(recv_rows), 3), np.int64)
    return HaloPlan(send_counts, rows.astype(np.int32), recv_counts, recv_rows, image)


class HaloExchange:
    """Ghost rows of node features (forward) and their gradients (backward)
    with torch collectives, called back by the library between layers.

      features:  owners send the rows of the requested atoms, ghosts take them;
      gradients: ghosts send their rows back, owners add them, ghosts are zeroed.
    Both are one ``all_to_all_single`` with uneven splits.  Works with any
    process group (gloo on the CPU tests); on GPUs ``NativeHaloExchange`` does
    the same inside the step.
    """

    def __init__(self, hp: HaloPlan, group=None, device=None):
        import torch
        import torch.distributed as dist

        self.torch, self.dist, self.group = torch, dist, group
        dev = device
        self.recv_counts, self.send_counts = list(hp.recv_counts), list(hp.send_counts)
        self.ghost_rows = torch.as_tensor(hp.recv_rows.astype(np.int64), device=dev)
        self.send_rows = torch.as_tensor(hp.send_rows.astype(np.int64), device=dev)

    @classmethod
    def from_plan(cls, plan: DomainPlan, owner_of: np.ndarray, world: int, device, group=None) -> "HaloExchange":
        return cls(make_halo_plan(plan, owner_of, world, device, group), group, device)

    def features(self, rows):
        torch = self.torch
        send = rows.index_select(0, self.send_rows.to(rows.device))
        recv = torch.empty(len(self.ghost_rows), rows.shape[1], dtype=rows.dtype, device=rows.device)
        self.dist.all_to_all_single(recv, send, output_split_sizes=self.recv_counts,
                                    input_split_sizes=self.send_counts, group=self.group)
        rows.index_copy_(0, self.ghost_rows.to(rows.device), recv)

    def gradients(self, rows):
        torch = self.torch
        send = rows.index_select(0, self.ghost_rows.to(rows.device))
        recv = torch.empty(len(self.send_rows), rows.shape[1], dtype=rows.dtype, device=rows.device)
        self.dist.all_to_all_single(recv, send, output_split_sizes=self.send_counts,
                                    input_split_sizes=self.recv_counts, group=self.group)
        rows.index_add_(0, self.send_rows.to(rows.device), recv)
        rows.index_fill_(0, self.ghost_rows.to(rows.device), 0.0)

    def __call__(self, phase: int, layer: int, rows):
        (self.features if phase == 0 else self.gradients)(rows)


class NativeHaloExchange:
    """The library's own halo exchange (``mace_halo_*`` in include/mace_b200.h):
    an NCCL communicator of the library's, created once per runner from a unique
    id that rank 0 makes and the process group broadcasts; the plan is uploaded
    at every rebuild.  The step then issues gather kernel -> NCCL send/recv ->
    scatter (features) and the reverse with a fixed-order accumulation
    (gradients) on its own stream, inside its CUDA graph."""

    def __init__(self, model, world: int, rank: int, group=None):
        import ctypes as C

        import torch

        from . import native as nv

        self.C, self.nv, self.lib = C, nv, model.lib
        buf = C.create_string_buffer(128)
        if rank == 0:
            nv.check(self.lib.mace_halo_unique_id(buf, 128), self.lib)
        obj = [buf.raw if rank == 0 else None]
        torch.distributed.broadcast_object_list(obj, src=0, group=group)
        uid = C.create_string_buffer(obj[0], 128)
        self.h = C.c_void_p()
        dev = torch.device(model.device).index or 0
        nv.check(self.lib.mace_halo_create(uid, 128, world, rank, dev, C.byref(self.h)), self.lib)

    def set_plan(self, hp: HaloPlan, n_owned: int, n_local: int, row_cap: int):
        C = self.C
        sc = np.ascontiguousarray(hp.send_counts, dtype=np.int64)
        rc = np.ascontiguousarray(hp.recv_counts, dtype=np.int64)
        sr = np.ascontiguousarray(hp.send_rows, dtype=np.int32)
        rr = np.ascontiguousarray(hp.recv_rows, dtype=np.int32)
        self.nv.check(self.lib.mace_halo_plan(self.h, n_owned, n_local, row_cap, sc.ctypes.data, sr.ctypes.data,
                                              rc.ctypes.data, rr.ctypes.data), self.lib)

    @property
    def handle(self) -> int:
        return self.h.value

    def close(self):
        if self.h:
            self.lib.mace_halo_destroy(self.h)
            self.h = self.C.c_void_p()


class GhostExchange:
    """Per-step halo-sized exchange of positions and forces with the ghost plan.

    positions: owners send the local positions of the requested atoms and each
    ghost row becomes its owner's position + image @ cell;
    forces: ghost rows' forces go back to their owners and are added there.
    """

    def __init__(self, hp: HaloPlan, plan: DomainPlan, cell_dev, group=None):
        import torch

        dev = cell_dev.device
        self.torch, self.group = torch, group
        self.n_owned = plan.n_owned
        self.send_counts, self.recv_counts = list(hp.send_counts), list(hp.recv_counts)
        self.send_rows = torch.as_tensor(hp.send_rows.astype(np.int64), device=dev)
        self.recv_rows = torch.as_tensor(hp.recv_rows.astype(np.int64), device=dev)
        self.offset = torch.as_tensor(hp.ghost_image, dtype=torch.float64, device=dev) @ cell_dev
        self.recv_pos = torch.empty(len(hp.recv_rows), 3, dtype=torch.float64, device=dev)
        self.recv_f = torch.empty(len(hp.send_rows), 3, dtype=torch.float32, device=dev)

    def positions(self, loc64):
        send = loc64.index_select(0, self.send_rows)
        self.torch.distributed.all_to_all_single(self.recv_pos, send, output_split_sizes=self.recv_counts,
                                                 input_split_sizes=self.send_counts, group=self.group)
        loc64.index_copy_(0, self.recv_rows, self.recv_pos + self.offset)

    def forces(self, f_local):
        send = f_local.index_select(0, self.recv_rows)
        self.torch.distributed.all_to_all_single(self.recv_f, send, output_split_sizes=self.send_counts,
                                                 input_split_sizes=self.recv_counts, group=self.group)
        f_own = f_local[: self.n_owned].clone()
        f_own.index_add_(0, self.send_rows, self.recv_f)
        return f_own


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
           "SpatialRunner", "HaloPlan", "make_halo_plan", "HaloExchange", "NativeHaloExchange", "GhostExchange",
           "PositionExchange", "gather_owned", "reduce_local"]
