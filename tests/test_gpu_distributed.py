"""Spatial domain decomposition on two GPUs (NCCL) against one GPU on the whole cell.

Runs only where two GPUs are visible; the CPU suite covers the same host logic
with gloo ranks and the float64 oracle (test_distributed.py).
"""

import os
import socket
import tempfile

import numpy as np
import pytest
import torch

from helpers import make_case
from mace_mlx_b200.distributed import SpatialRunner
from mace_mlx_b200.model import MACEModel
from mace_mlx_b200.structures import diamond_si

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")]


def _case():
    st = diamond_si(6, 0.05, 41)
    config, weights, _ = make_case("medium", st, seed=41, avg_num_neighbors=44.0)
    return st, config, weights


def _run(model, st, world, rank, halo=True):
    runner = SpatialRunner(model, st.numbers, st.cell, world, rank, skin=0.5, halo=halo)
    pos = torch.tensor(st.positions, dtype=torch.float64, device=model.device)
    out = runner.evaluate(pos, virial=True)
    res = runner.reduce(out, len(st), virial=True)
    torch.cuda.synchronize(model.device)
    return {k: v.cpu().numpy().astype(np.float64) for k, v in res.items()}, runner.plan


def _rank_main(rank, world, port, path, halo):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        st, config, weights = _case()
        model = MACEModel(config=config, weights=weights, device=rank)
        res, plan = _run(model, st, world, rank, halo)
        if rank == 0:
            np.savez(path, n_local=plan.n_local, n_owned=plan.n_owned, **res)
        torch.distributed.barrier()
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("halo", [True, False])
def test_two_gpu_domains_match_one_gpu(halo):
    """halo: r_max ghost shell with layer features exchanged over NCCL; else a 2 r_max shell."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "rank0.npz")
        torch.multiprocessing.spawn(_rank_main, args=(2, port, path, halo), nprocs=2, join=True)
        got = dict(np.load(path))
    st, config, weights = _case()
    ref, _ = _run(MACEModel(config=config, weights=weights, device=0), st, 1, 0)
    assert got["n_owned"] < got["n_local"]
    n = len(st)
    assert abs(got["energy"][0] - ref["energy"][0]) / n < 1e-6
    scale = np.abs(ref["forces"]).max()
    np.testing.assert_allclose(got["forces"], ref["forces"], atol=1e-4 * max(scale, 1e-3))
    np.testing.assert_allclose(got["virial"], ref["virial"], atol=1e-5 * np.abs(ref["virial"]).max())
