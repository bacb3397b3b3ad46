"""Host logic of the multi-GPU paths (mace_mlx_b200/distributed.py), on the CPU.

The spatial decomposition is checked geometrically (owned sets partition the
atoms, ghost shells cover every owned atom's receptive field) and end to end:
two gloo ranks evaluate their domains with the float64 oracle, energy weights
1 on owned and 0 on ghost atoms, and the reduced energy, forces and virial
equal the oracle on the whole periodic cell.
"""

import contextlib
import os
import socket
import tempfile

import numpy as np
import pytest
import torch

from helpers import make_case
from mace_mlx_b200.distributed import (grid_for, plan_domain, plane_spacings, reduce_local,
                                       shard_structures)
from mace_mlx_b200.structures import diamond_si
from oracle.model import OracleMACE
from oracle.nl import neighbour_list


def test_grid_and_structure_sharding():
    assert [grid_for(w) for w in (1, 2, 4, 8)] == [(1, 1, 1), (1, 1, 2), (1, 2, 2), (2, 2, 2)]
    assert grid_for(6) == (1, 2, 3)
    sizes = np.random.default_rng(0).integers(20, 61, size=512)
    for world in (1, 2, 4, 8):
        shards = shard_structures(sizes, world)
        assert sorted(i for s in shards for i in s) == list(range(512))
        loads = [sizes[s].sum() for s in shards]
        assert max(loads) - min(loads) <= sizes.max()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_plan_partitions_atoms_and_covers_the_receptive_field(world):
    st = diamond_si(4, 0.05, 31)
    rng = np.random.default_rng(1)
    pos = st.positions + rng.integers(-1, 2, size=(len(st), 3)) @ st.cell  # unwrapped copies
    gw = 4.2
    plans = [plan_domain(pos, st.cell, grid_for(world), r, gw) for r in range(world)]
    owned = np.concatenate([p.owned_index for p in plans])
    assert sorted(owned.tolist()) == list(range(len(st)))
    # every image within gw of an owned atom is local, at the right shift
    i, j, S = neighbour_list(pos, st.cell, st.pbc, gw)
    for p in plans:
        split = ~np.asarray(p.pbc)
        assert split.sum() == sum(g > 1 for g in p.grid)
        full = {(int(g), tuple(s)) for g, s in zip(p.local_index, p.local_shift)}
        assert len(full) == p.n_local  # no image twice
        # periodic (unsplit) axes wrap in the local system: only split-axis shifts must match
        local = {(int(g), tuple(s[split])) for g, s in zip(p.local_index, p.local_shift)}
        own_shift = {int(g): s for g, s in zip(p.owned_index, p.local_shift[: p.n_owned])}
        for a, b, s in zip(i, j, S):
            if int(b) in own_shift:  # receiver b owned: the sender's image pos_a - S @ cell, in b's frame
                need = tuple((own_shift[int(b)] - s)[split].tolist())
                assert (int(a), need) in local
    assert np.all(gw / plane_spacings(st.cell) < 1)


def _weighted_oracle(orc, pos, cell, pbc, species, weight, r_cut):
    i, j, S = neighbour_list(pos, cell, np.asarray(pbc), r_cut)
    p = torch.tensor(pos, dtype=torch.float64, requires_grad=True)
    snd, rcv = torch.as_tensor(i), torch.as_tensor(j)
    v = p[rcv] - p[snd] + torch.as_tensor(S, dtype=torch.float64) @ torch.as_tensor(cell, dtype=torch.float64)
    r = torch.sqrt(torch.clamp((v * v).sum(-1, keepdim=True), min=1e-24))
    _, node_e = orc.energy_from_vectors(v, r, torch.as_tensor(species, dtype=torch.long), snd, rcv, None, 1)
    e = (node_e * torch.as_tensor(weight, dtype=torch.float64)).sum()
    gp, gv = torch.autograd.grad(e, (p, v))
    virial = (v.detach().T @ gv).numpy()
    return e.detach(), -gp, torch.as_tensor(virial)


def _case():
    st = diamond_si(3, 0.05, 32)
    config, weights, _ = make_case("small", st, seed=32, r_max=3.0, avg_num_neighbors=4.0)
    return st, config, weights


def _rank_main(rank, world, port, path, case):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)  # two ranks on a shared CPU
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        st, config, weights = case
        orc = OracleMACE(config, weights)
        gw = 2 * config["r_max"] + 0.5
        plan = plan_domain(st.positions, st.cell, grid_for(world), rank, gw)
        loc = st.positions[plan.local_index] + plan.local_shift @ st.cell
        species = np.zeros(plan.n_local, dtype=np.int64)  # z_table [14]
        weight = np.zeros(plan.n_local)
        weight[: plan.n_owned] = 1.0
        e, f, vir = _weighted_oracle(orc, loc, st.cell, plan.pbc, species, weight, config["r_max"])
        out = {"energy": e.reshape(1), "forces": f, "virial": vir.reshape(9)}
        res = reduce_local(plan.local_index, out, len(st), world, virial=True)
        if rank == 0:
            np.savez(path, energy=res["energy"].numpy(), forces=res["forces"].numpy(),
                     virial=res["virial"].numpy(), n_local=plan.n_local, n_owned=plan.n_owned)
    finally:
        torch.distributed.destroy_process_group()


@contextlib.contextmanager
def _single_threaded_children():
    """Ranks spawned on one shared CPU: one BLAS / OpenMP thread each (else they contend)."""
    keys = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")
    old = {k: os.environ.get(k) for k in keys}
    os.environ.update({k: "1" for k in keys})
    try:
        yield
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_reproduce_the_periodic_oracle():
    st, config, weights = _case()
    orc = OracleMACE(config, weights)
    i, j, S = neighbour_list(st.positions, st.cell, st.pbc, config["r_max"])
    ref = orc.compute(st.positions, np.zeros(len(st), dtype=np.int64), i, j, S, st.cell, stress=True)
    with tempfile.TemporaryDirectory() as tmp, _single_threaded_children():
        path = os.path.join(tmp, "rank0.npz")
        torch.multiprocessing.spawn(_rank_main, args=(2, _free_port(), path, (st, config, weights)), nprocs=2,
                                    join=True)
        got = np.load(path)
    assert got["n_owned"] < got["n_local"]  # real ghosts
    np.testing.assert_allclose(got["energy"][0], ref["energy"][0], rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(got["forces"], ref["forces"], rtol=1e-8, atol=1e-10)
    vol = abs(np.linalg.det(st.cell))
    g = got["virial"].reshape(3, 3)
    s = 0.5 * (g + g.T) / vol
    voigt = s[[0, 1, 2, 1, 0, 0], [0, 1, 2, 2, 2, 1]]
    np.testing.assert_allclose(voigt, ref["stress"], rtol=1e-8, atol=1e-12)


def _halo_rank(rank, world, port, path, pos, cell):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mace_mlx_b200.distributed import HaloExchange, domain_of

        grid = grid_for(world)
        plan = plan_domain(pos, cell, grid, rank, 3.5)
        hx = HaloExchange.from_plan(plan, domain_of(pos, cell, grid), world, "cpu")
        gid = torch.as_tensor(plan.local_index, dtype=torch.float64)
        rows = torch.stack([gid, 2 * gid + 1, -gid], dim=1)
        rows[plan.n_owned:] = -7.0
        hx(0, 0, rows)  # features: ghosts take their owners' rows
        ok_fwd = bool(torch.equal(rows, torch.stack([gid, 2 * gid + 1, -gid], dim=1)))
        g = torch.zeros(plan.n_local, 2, dtype=torch.float64)
        g[plan.n_owned:] = 1.0
        hx(1, 0, g)  # gradients: ghosts' rows go to their owners
        ok_zero = bool(torch.all(g[plan.n_owned:] == 0))
        counts = np.zeros(len(pos))
        np.add.at(counts, plan.local_index[: plan.n_owned], g[: plan.n_owned, 0].numpy())
        ghosts = [None] * world
        torch.distributed.all_gather_object(ghosts, plan.local_index[plan.n_owned:])
        c = torch.as_tensor(counts)
        torch.distributed.all_reduce(c)
        want = np.bincount(np.concatenate(ghosts), minlength=len(pos)).astype(np.float64)
        if rank == 0:
            np.savez(path, ok_fwd=ok_fwd, ok_zero=ok_zero, counts=c.numpy(), want=want,
                     n_ghost=plan.n_local - plan.n_owned)
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_halo_exchange_moves_ghost_rows_and_reduces_gradients(world):
    st = diamond_si(4, 0.05, 33)
    with tempfile.TemporaryDirectory() as tmp, _single_threaded_children():
        path = os.path.join(tmp, "r0.npz")
        torch.multiprocessing.spawn(_halo_rank, args=(world, _free_port(), path, st.positions, st.cell),
                                    nprocs=world, join=True)
        got = np.load(path)
    assert got["n_ghost"] > 0 and got["ok_fwd"] and got["ok_zero"]
    np.testing.assert_array_equal(got["counts"], got["want"])
