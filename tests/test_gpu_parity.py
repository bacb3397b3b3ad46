"""CUDA step (through the C ABI) against the float64 CPU oracle.

Tolerances: energy 1e-5 eV/atom, forces 1e-4 eV/A max-abs,
stress 1e-6 eV/A^3 -- plus relative bounds (1e-5 energy, 1e-4 forces/stress of
their own scale) so that the checks stay meaningful at small magnitudes."""

import numpy as np
import pytest
import torch

from helpers import assert_parity, graph_ptr_of, irreps_to_channel_last, make_case, rel_err, run_gpu
from mace_mlx_b200.model import MACEModel, edge_tiles_to_rows
from mace_mlx_b200.spec import ModelSpec
from mace_mlx_b200.structures import diamond_si, lipso_box, molecule_batch
from mace_mlx_b200.weights import random_config, random_weights
from oracle.model import OracleMACE

pytestmark = pytest.mark.gpu
torch.set_num_threads(min(16, torch.get_num_threads()))


def oracle_of(config, weights, st, edges, species, stress):
    s, r, S = edges.numpy()
    orc = OracleMACE(config, weights)
    return orc.compute(st.positions, species, s, r, S, st.cell if np.any(st.pbc) else None,
                       stress=stress, batch=st.batch, num_graphs=st.num_graphs)


def check(config, weights, st, stress=True):
    m = MACEModel(config=config, weights=weights, device=0)
    gpu, edges, species = run_gpu(m, st, virial=stress)
    ref = oracle_of(config, weights, st, edges, species, stress and bool(np.any(st.pbc)))
    assert_parity(gpu, ref, len(st), stress=stress and bool(np.any(st.pbc)))
    return m, gpu, ref, edges


@pytest.mark.parametrize("arch", ["small", "medium", "large"])
def test_archs_on_si64(arch):
    config, weights, st = make_case(arch, diamond_si(2, 0.05, 11), seed=11)
    check(config, weights, st)


def test_config0_small_si216():
    config, weights, st = make_case("small", diamond_si(3, 0.01, 0), seed=0, avg_num_neighbors=46.0)
    check(config, weights, st)


def test_config1_medium_si1000_energy_forces():
    config, weights, st = make_case("medium", diamond_si(5, 0.05, 1), seed=1, avg_num_neighbors=44.0)
    check(config, weights, st, stress=False)


def test_lipso_large_four_species_with_stress():
    st = lipso_box(300, 2)
    config, weights, _ = make_case("large", st, seed=2, z_table=[3, 8, 15, 16], avg_num_neighbors=50.0)
    check(config, weights, st)


def test_off_like_molecule_batch():
    st = molecule_batch(8, 3)
    config, weights, _ = make_case("medium", st, seed=3, z_table=[1, 6, 7, 8], r_max=5.0,
                                   hidden_irreps="96x0e + 96x1o", avg_num_neighbors=12.0)
    m, gpu, ref, _ = check(config, weights, st, stress=False)
    assert gpu["energy"].shape == (8,)


def test_non_residual_first_layer_and_scale_shift():
    cfg = random_config("medium", z_table=[14, 6], avg_num_neighbors=30.0, first_interaction_nonresidual=True,
                        atomic_energies=[-5.4, -8.1], model_type="ScaleShiftMACE")
    cfg["scale"], cfg["shift"] = 1.3, -0.2
    w = random_weights(ModelSpec.from_config(cfg), 4)
    st = diamond_si(2, 0.05, 4)
    st.numbers[::3] = 6
    check(cfg, w, st)


MPA = dict(use_density_normalization=True, distance_transform={}, pair_repulsion={})


@pytest.mark.parametrize("nonres,scale_shift", [(True, True), (False, False)])
def test_mpa_family_density_agnesi_zbl(nonres, scale_shift):
    """Density-normalised blocks, the Agnesi transform and ZBL repulsion (the
    mpa-0 family) on a LiPSO box with pairs inside the ZBL range, with stress."""
    cfg = random_config("medium", z_table=[3, 8, 15, 16], avg_num_neighbors=50.0, first_interaction_nonresidual=nonres,
                        atomic_energies=[-1.9, -4.9, -5.4, -4.1],
                        model_type="ScaleShiftMACE" if scale_shift else "MACE", **MPA)
    if scale_shift:
        cfg["scale"], cfg["shift"] = 1.3, -0.2
    w = random_weights(ModelSpec.from_config(cfg), 6)
    m, gpu, ref, _ = check(cfg, w, lipso_box(300, 2))
    pair = m.debug_buffer("e_layers").cpu().numpy().reshape(-1, len(gpu["forces"]))[-1]
    assert np.abs(pair).max() > 1e-3  # the ZBL term is active in this structure


def test_mpa_family_molecules_open_boundaries():
    st = molecule_batch(6, 5)
    cfg = random_config("medium", z_table=[1, 6, 7, 8], r_max=5.0, first_interaction_nonresidual=True, **MPA)
    w = random_weights(ModelSpec.from_config(cfg), 8)
    check(cfg, w, st, stress=False)


@pytest.mark.parametrize("max_ell,corr", [(2, 3), (3, 2), (1, 1)])
def test_other_lmax_and_correlation(max_ell, corr):
    cfg = random_config("medium", z_table=[14], avg_num_neighbors=40.0, max_ell=max_ell, correlation=corr)
    w = random_weights(ModelSpec.from_config(cfg), 5)
    check(cfg, w, diamond_si(2, 0.05, 5))


def test_per_stage_buffers_medium():
    config, weights, st = make_case("medium", diamond_si(2, 0.05, 1), seed=1)
    m = MACEModel(config=config, weights=weights, device=0)
    gpu, edges, species = run_gpu(m, st, virial=False)
    s, r, S = edges.numpy()
    trace = {}
    OracleMACE(config, weights).compute(st.positions, species, s, r, S, st.cell, trace=trace)
    spec = m.spec
    N, E = len(st), edges.n_edges
    assert rel_err(m.debug_buffer("Y").cpu().numpy().reshape(E, 16), trace["Y"].detach().numpy()) < 1e-5
    assert rel_err(m.debug_buffer("b").cpu().numpy().reshape(E, -1), trace["b"].detach().numpy()) < 1e-5
    for t, lay in enumerate(spec.layers):
        def cmp(stage, key, irreps, grad=False, rows=N):
            ref = trace[key].grad if grad else trace[key].detach()
            ref = ref.numpy()
            if irreps is not None:
                ref = irreps_to_channel_last(ref, irreps)
            got = m.debug_buffer(stage, t)
            if stage == "w":
                got = edge_tiles_to_rows(got, E, ref.shape[1])
            got = got.cpu().numpy().reshape(rows, -1)
            assert rel_err(got, ref) < 2e-5, (t, stage, rel_err(got, ref))

        cmp("up", f"up{t}", lay.irreps_in)
        cmp("w", f"w{t}", None, rows=E)
        cmp("A", f"A{t}", lay.conv.irreps_mid)
        cmp("msg", f"msg{t}", spec.interaction_irreps)
        cmp("B", f"B{t}", lay.hidden)
        cmp("h_out", f"h{t + 1}", lay.hidden)
        cmp("dB", f"B{t}", lay.hidden, grad=True)
        cmp("dmsg", f"msg{t}", spec.interaction_irreps, grad=True)
        cmp("dA", f"A{t}", lay.conv.irreps_mid, grad=True)
        if t > 0:
            cmp("dup", f"up{t}", lay.irreps_in, grad=True)
    assert rel_err(m.debug_buffer("dY").cpu().numpy().reshape(E, 16), trace["Y"].grad.numpy()) < 2e-5
    assert rel_err(m.debug_buffer("dv").cpu().numpy().reshape(E, 3), trace["v"].grad.numpy()) < 2e-5
    assert m.error_flag() == 0


def test_cuda_graph_replay_matches_direct_launches():
    config, weights, st = make_case("medium", diamond_si(2, 0.05, 9), seed=9)
    m = MACEModel(config=config, weights=weights, device=0)
    dev = m.device
    species = torch.as_tensor(m.species_index(st.numbers), device=dev)
    gp = torch.tensor([0, len(st)], dtype=torch.int32, device=dev)
    pos64 = torch.tensor(st.positions, dtype=torch.float64, device=dev)
    cell64 = torch.tensor(st.cell, dtype=torch.float64, device=dev)
    edges = m.neighbour_list(pos64, cell64, st.pbc, gp, m.r_max + 0.5)
    pos, cell = pos64.float(), cell64.float()
    direct = m.evaluate(pos, cell, species, gp, edges, virial=True)
    torch.cuda.synchronize()
    ref = {k: v.clone() for k, v in direct.items()}
    out = {k: torch.empty_like(v) for k, v in direct.items()}
    with torch.cuda.stream(torch.cuda.Stream(dev)):
        for step in range(3):
            if step == 2:  # new positions in the same buffer: replay, not re-capture
                pos.add_(1e-3)
            m.evaluate(pos, cell, species, gp, edges, virial=True, out=out, graph=True)
            torch.cuda.current_stream(dev).synchronize()
            if step < 2:
                for k in ref:
                    torch.testing.assert_close(out[k], ref[k], rtol=0, atol=0)
    again = m.evaluate(pos, cell, species, gp, edges, virial=True)
    torch.cuda.synchronize()
    for k in ref:
        torch.testing.assert_close(out[k], again[k], rtol=0, atol=0)


def test_bitwise_deterministic_and_translation_invariant():
    config, weights, st = make_case("medium", diamond_si(3, 0.05, 8), seed=8)
    m = MACEModel(config=config, weights=weights, device=0)
    a, _, _ = run_gpu(m, st)
    b, _, _ = run_gpu(m, st)
    np.testing.assert_array_equal(a["forces"], b["forces"])
    np.testing.assert_array_equal(a["energy"], b["energy"])
    assert np.abs(a["forces"].sum(0)).max() < 1e-5 * max(1.0, np.abs(a["forces"]).max() * len(st))
    st2 = diamond_si(3, 0.05, 8)
    st2.positions = st2.positions + np.array([0.37, -0.21, 0.05])
    c, _, _ = run_gpu(m, st2)
    np.testing.assert_allclose(c["forces"], a["forces"], atol=1e-4 * np.abs(a["forces"]).max() + 1e-7)


def test_tensor_core_mlp_matches_cuda_core_mlp(monkeypatch):
    """tcgen05 (3-term tf32) radial MLP vs the fp32 CUDA-core kernels."""
    config, weights, st = make_case("medium", diamond_si(3, 0.05, 13), seed=13)
    m_tc = MACEModel(config=config, weights=weights, device=0)
    monkeypatch.setenv("MACE_B200_MLP_CUDA_CORES", "1")
    m_cc = MACEModel(config=config, weights=weights, device=0)
    a, edges, _ = run_gpu(m_tc, st)
    b, _, _ = run_gpu(m_cc, st)
    for t in range(2):
        E, W = edges.n_edges, m_tc.spec.layers[t].mlp_widths[-1]
        wa = edge_tiles_to_rows(m_tc.debug_buffer("w", t), E, W).cpu().numpy()
        wb = edge_tiles_to_rows(m_cc.debug_buffer("w", t), E, W).cpu().numpy()
        assert rel_err(wa, wb) < 1e-5, rel_err(wa, wb)  # both fp32-accurate: ~2^-21 per product
    assert rel_err(a["forces"], b["forces"]) < 2e-5
    assert abs(a["energy"][0] - b["energy"][0]) < 1e-5 * max(1.0, abs(b["energy"][0]))


def test_tensor_core_linears_match_cuda_core_linears(monkeypatch):
    """tcgen05 (3-term tf32) node linears and species-indexed skips vs the fp32 CUDA-core kernel.

    A four-element box puts several species in every 128-row tile (one
    species pass each); at 1200 atoms the launch of layer 1's linear_up with
    its species-indexed skip is large enough for the tensor-core kernel, and
    1200 rows leave a ragged last tile in every job.
    """
    st = lipso_box(1200, seed=5)
    config, weights, _ = make_case("medium", st, seed=14)
    m_tc = MACEModel(config=config, weights=weights, device=0)
    monkeypatch.setenv("MACE_B200_LINEAR_CUDA_CORES", "1")
    m_cc = MACEModel(config=config, weights=weights, device=0)
    a, _, _ = run_gpu(m_tc, st)
    b, _, _ = run_gpu(m_cc, st)
    assert rel_err(a["node_energy"], b["node_energy"]) < 2e-5
    assert rel_err(a["forces"], b["forces"]) < 2e-5
    assert rel_err(a["stress"], b["stress"]) < 2e-5
    assert m_tc.error_flag() == 0


def _eval(m, st, edges, species, weight=None):
    dev = m.device
    gp = torch.as_tensor(graph_ptr_of(st), device=dev)
    cell = torch.tensor(st.cell, dtype=torch.float32, device=dev)
    w = None if weight is None else torch.as_tensor(weight, dtype=torch.float32, device=dev)
    out = m.evaluate(torch.tensor(st.positions, dtype=torch.float32, device=dev), cell,
                     torch.as_tensor(species, device=dev), gp, edges, forces=True, virial=True, energy_weight=w)
    torch.cuda.synchronize(dev)
    return {k: v.cpu().numpy().astype(np.float64) for k, v in out.items()}


def test_receiver_chunks_give_identical_results():
    """Radial work in receiver chunks (MLP recomputed in the backward) equals the one-pass step bitwise."""
    config, weights, st = make_case("medium", diamond_si(3, 0.05, 21), seed=21)
    m = MACEModel(config=config, weights=weights, device=0)
    _, edges, species = run_gpu(m, st)
    a = _eval(m, st, edges, species)
    m.max_chunk_edges = edges.n_edges // 5 + 1
    nodes, ebounds = edges.receiver_chunks(m.max_chunk_edges)
    assert len(nodes) - 1 >= 5 and np.all(np.diff(ebounds) <= m.max_chunk_edges)
    b = _eval(m, st, edges, species)
    for k in ("energy", "node_energy", "forces", "virial"):
        np.testing.assert_array_equal(a[k], b[k])
    assert m.error_flag() == 0


def test_energy_weights_are_linear():
    """E and forces with node weights w plus those with 1 - w equal the unweighted step."""
    config, weights, st = make_case("medium", diamond_si(2, 0.05, 22), seed=22)
    m = MACEModel(config=config, weights=weights, device=0)
    _, edges, species = run_gpu(m, st)
    w = (np.random.default_rng(0).random(len(st)) < 0.4).astype(np.float32)
    full = _eval(m, st, edges, species)
    a = _eval(m, st, edges, species, w)
    b = _eval(m, st, edges, species, 1.0 - w)
    np.testing.assert_allclose(a["node_energy"], full["node_energy"], rtol=0, atol=0)
    np.testing.assert_allclose(a["energy"], (w * full["node_energy"]).sum(), rtol=1e-6)
    np.testing.assert_allclose(a["energy"] + b["energy"], full["energy"], rtol=1e-6)
    scale = np.abs(full["forces"]).max()
    np.testing.assert_allclose(a["forces"] + b["forces"], full["forces"], atol=2e-5 * scale)
    np.testing.assert_allclose(a["virial"] + b["virial"], full["virial"], atol=2e-5 * np.abs(full["virial"]).max())


def test_profiler_eager_and_in_graph():
    """Per-launch event timing works on an eager step and inside the replayed step graph."""
    config, weights, st = make_case("medium", diamond_si(2, 0.05, 17), seed=17)
    m = MACEModel(config=config, weights=weights, device=0)
    _, edges, species = run_gpu(m, st)
    dev = m.device
    gp = torch.as_tensor(graph_ptr_of(st), device=dev)
    pos = torch.tensor(st.positions, dtype=torch.float32, device=dev)
    cell = torch.tensor(st.cell, dtype=torch.float32, device=dev)
    sp = torch.as_tensor(species, device=dev)
    seen = {}
    for graph in (False, True, True):
        m.profile_enable(True)
        m.evaluate(pos, cell, sp, gp, edges, forces=True, graph=graph)
        torch.cuda.synchronize(dev)
        rows = m.profile_read()
        tl = m.profile_timeline()
        m.profile_enable(False)
        assert rows and all(r["ms"] > 0 and r["count"] >= 1 for r in rows)
        assert len(tl) == sum(r["count"] for r in rows)
        assert all(t["end_ms"] >= t["start_ms"] >= 0 for t in tl)
        seen[graph] = {(r["name"], r["layer"]) for r in rows}
    assert seen[False] == seen[True]


def test_two_stream_schedule_matches_single_stream(monkeypatch):
    """The two-stream step (radial MLP on a second stream; layer 0's MLP and
    conv in two parts each when the edge tiles exceed one round of MLP CTAs)
    runs the same per-edge and per-receiver arithmetic in the same
    accumulation order as the single-stream step: identical results.
    Si 6x6x6 (1728 atoms, ~80 000 edges) has more than two tiles per SM."""
    st = diamond_si(6, 0.05, 61)
    config, weights, _ = make_case("medium", st, seed=61, avg_num_neighbors=44.0)
    m2 = MACEModel(config=config, weights=weights, device=0)
    monkeypatch.setenv("MACE_B200_SINGLE_STREAM", "1")
    m1 = MACEModel(config=config, weights=weights, device=0)
    a, edges, _ = run_gpu(m2, st)
    b, _, _ = run_gpu(m1, st)
    n_tiles = (edges.n_edges + 127) // 128
    assert n_tiles > 2 * torch.cuda.get_device_properties(0).multi_processor_count
    for k in ("energy", "node_energy", "forces", "stress"):
        np.testing.assert_array_equal(a[k], b[k], err_msg=k)
    assert m2.error_flag() == 0 and m1.error_flag() == 0
