"""Spatial domain decomposition on two GPUs against one GPU on the whole cell.

Runs only where two GPUs are visible; the CPU suite covers the same host logic
with gloo ranks and the float64 oracle (test_distributed.py).  Three modes:
the library's own halo exchange (NCCL send/recv inside the step, owned atoms
the only receivers, the step replayed as a CUDA graph, positions and forces
moved halo-sized per step), the host-callback halo with torch collectives,
and the 2 r_max ghost shell without exchange between layers.
"""

import datetime
import faulthandler
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


def _rank_main(rank, world, port, path, mode):
    # a rank that is still running after four minutes prints its stack and exits,
    # so that a stuck exchange fails the test instead of holding both GPUs
    faulthandler.dump_traceback_later(240, exit=True)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                         timeout=datetime.timedelta(seconds=120))
    try:
        st, config, weights = _case()
        model = MACEModel(config=config, weights=weights, device=rank)
        runner = SpatialRunner(model, st.numbers, st.cell, world, rank, skin=0.5, halo=mode != "shell",
                               native=mode == "native")
        runner.graph = mode == "native"
        pos = torch.tensor(st.positions, dtype=torch.float64, device=model.device)
        out = runner.evaluate(pos, virial=True)
        res = runner.reduce(out, len(st), virial=True)
        res = {k: v.cpu().numpy().astype(np.float64) for k, v in res.items()}
        # the halo-sized step path, twice (the second replays the captured graph)
        own = pos[torch.as_tensor(runner.owned_index, device=pos.device)]
        for _ in range(2):
            step = runner.step(own, virial=True)
        f_all = [None] * world
        torch.distributed.all_gather_object(f_all, (runner.owned_index, step["forces"].cpu().numpy()))
        forces = np.zeros((len(st), 3))
        for idx, f in f_all:
            forces[idx] = f
        if rank == 0:
            np.savez(path, n_local=runner.plan.n_local, n_owned=runner.plan.n_owned, step_forces=forces,
                     step_energy=step["energy"].cpu().numpy(), step_virial=step["virial"].cpu().numpy(), **res)
        torch.distributed.barrier()
        runner.close()
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("mode", ["shell", "callback", "native"])
def test_two_gpu_domains_match_one_gpu(mode):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "rank0.npz")
        torch.multiprocessing.spawn(_rank_main, args=(2, port, path, mode), nprocs=2, join=True)
        got = dict(np.load(path))
    st, config, weights = _case()
    model = MACEModel(config=config, weights=weights, device=0)
    runner = SpatialRunner(model, st.numbers, st.cell, 1, 0)
    ref = runner.reduce(runner.evaluate(torch.tensor(st.positions, dtype=torch.float64, device=model.device),
                                        virial=True), len(st), virial=True)
    ref = {k: v.cpu().numpy().astype(np.float64) for k, v in ref.items()}
    assert got["n_owned"] < got["n_local"]
    n = len(st)
    scale = np.abs(ref["forces"]).max()
    for e, f, v in ((got["energy"], got["forces"], got["virial"]),
                    (got["step_energy"], got["step_forces"], got["step_virial"])):
        assert abs(e[0] - ref["energy"][0]) / n < 1e-6
        np.testing.assert_allclose(f, ref["forces"], atol=1e-4 * max(scale, 1e-3))
        np.testing.assert_allclose(v, ref["virial"], atol=1e-5 * np.abs(ref["virial"]).max())
