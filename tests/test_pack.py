"""Host-side packing of the model tables (pack.py), checked on the CPU."""

import numpy as np
import pytest
import torch

from helpers import make_case
from mace_mlx_b200.pack import PackedModel, sc_backward_polynomial, sc_polynomial
from mace_mlx_b200.spec import ModelSpec
from oracle.model import OracleMACE


@pytest.mark.parametrize("arch", ["small", "medium", "large"])
def test_symmetrised_sc_polynomial_equals_dense_contraction(arch):
    """The entry/G tables reproduce the reference's dense einsum contraction."""
    config, weights, _ = make_case(arch, seed=2, z_table=[14, 8])
    spec = ModelSpec.from_config(config)
    orc = OracleMACE(config, weights)
    rng = np.random.default_rng(0)
    lay = spec.layers[0]
    C = spec.C
    n = 6
    species = torch.tensor([0, 1, 0, 1, 1, 0])
    x = torch.tensor(rng.normal(size=(n, spec.interaction_irreps.dim)))
    ref = orc.symmetric_contraction(x, species, 0).numpy()
    # coupling-major features f[node, i, c] with i = l^2 + m
    f = np.concatenate([b.permute(0, 2, 1).numpy() for b in orc._blocks(x, spec.interaction_irreps)], axis=1)
    o_off = 0
    for o, out in enumerate(lay.sc.outputs):
        pre = f"products.0.symmetric_contractions.contractions.{o}"
        Ws = [weights[f"{pre}.weights_max"] if nu == out.correlation else
              weights[f"{pre}.weights.{out.correlation - 1 - nu}"] for nu in range(1, out.correlation + 1)]
        ent, G = sc_polynomial(out.U, Ws, out.ir_out.l)
        d = 2 * out.ir_out.l + 1
        got = np.zeros((n, C, d))
        for e_i, (M, a, b, c, nu) in enumerate(ent):
            term = f[:, a, :].copy()
            if nu >= 2:
                term *= f[:, b, :]
            if nu >= 3:
                term *= f[:, c, :]
            got[:, :, M] += G[species.numpy(), e_i, :] * term
        want = ref[:, o_off:o_off + C * d].reshape(n, C, d)
        np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-12)
        o_off += C * d
        assert len(ent) < sum(int(np.count_nonzero(np.abs(u) > 1e-12)) for u in out.U)


@pytest.mark.parametrize("arch", ["medium", "large"])
def test_sc_backward_polynomial_is_the_gradient(arch):
    """Per-index backward entries reproduce d/df of g . (forward polynomial), by autograd."""
    config, weights, _ = make_case(arch, seed=4, z_table=[14, 8])
    spec = ModelSpec.from_config(config)
    lay = spec.layers[0]
    C = spec.C
    ncoup = spec.interaction_irreps.dim // C
    rng = np.random.default_rng(1)
    n = 3
    species = np.array([0, 1, 1])
    f = torch.tensor(rng.normal(size=(n, ncoup, C)), requires_grad=True)
    outs, total, row0 = [], 0.0, 0
    rows = sum(2 * o.ir_out.l + 1 for o in lay.sc.outputs)
    g = torch.tensor(rng.normal(size=(n, rows, C)))
    for o, out in enumerate(lay.sc.outputs):
        pre = f"products.0.symmetric_contractions.contractions.{o}"
        Ws = [weights[f"{pre}.weights_max"] if nu == out.correlation else
              weights[f"{pre}.weights.{out.correlation - 1 - nu}"] for nu in range(1, out.correlation + 1)]
        ent, G = sc_polynomial(out.U, Ws, out.ir_out.l)
        outs.append((ent, G, row0))
        Gt = torch.tensor(G[species])  # (n, e, C)
        for e_i, (M, a, b, c, nu) in enumerate(ent):
            term = f[:, a, :]
            if nu >= 2:
                term = term * f[:, b, :]
            if nu >= 3:
                term = term * f[:, c, :]
            total = total + (Gt[:, e_i, :] * term * g[:, row0 + M, :]).sum()
        row0 += 2 * out.ir_out.l + 1
    total.backward()
    ent_b, G_b, seg = sc_backward_polynomial(outs, ncoup)
    assert seg[-1] == len(ent_b)
    got = np.zeros((n, ncoup, C))
    fn = f.detach().numpy()
    gn = g.numpy()
    for e_i, (k, b, c, nu1, r) in enumerate(ent_b):
        term = gn[:, r, :].copy()
        if nu1 >= 1:
            term *= fn[:, b, :]
        if nu1 >= 2:
            term *= fn[:, c, :]
        got[:, k, :] += G_b[species, e_i, :] * term
    np.testing.assert_allclose(got, f.grad.numpy(), rtol=1e-9, atol=1e-9)
    for k in range(ncoup):
        assert np.all(ent_b[seg[k]:seg[k + 1], 0] == k)


def test_packed_tables_are_aligned_and_complete():
    config, weights, _ = make_case("medium")
    pm = PackedModel(ModelSpec.from_config(config), weights)
    d = pm.desc
    assert pm.floats.dtype == np.float32 and pm.ints.dtype == np.int32
    assert d.f_emb % 4 == 0 and d.layers[1].f_mlp[3] % 4 == 0
    assert d.layers[1].n_mid == 10 and d.layers[1].wnumel == 1280 and d.layers[1].mid.dim == 5120
    assert [d.layers[1].lin[l].n_src for l in range(4)] == [2, 3, 3, 2]
    assert d.layers[0].sc[1].L == 1 and d.layers[0].sc[1].n_ent == 328
    assert np.all(np.isfinite(pm.floats))


def test_tf32_split_and_swizzled_images_round_trip():
    from mace_mlx_b200.pack import mlp_tc_images, sw128_image, tf32_split

    rng = np.random.default_rng(1)
    a = rng.normal(size=(64, 96)).astype(np.float32)
    hi, lo = tf32_split(a)
    assert np.all((hi.view(np.uint32) & 0x1FFF) == 0)
    np.testing.assert_array_equal(hi + lo, a)
    assert np.abs(lo).max() <= np.abs(a).max() * 2.0 ** -11
    img = sw128_image(a)
    r = np.arange(64)[:, None]
    k = np.arange(96)[None, :]
    off = (k // 32) * 64 * 32 + r * 32 + (((k % 32) // 4) ^ (r % 8)) * 4 + (k % 4)
    np.testing.assert_array_equal(img[off], a)
    assert len(set(off.ravel().tolist())) == a.size
    w = rng.normal(size=(200, 64)).astype(np.float32)  # (out, in) with out not a multiple of 128
    fwd, bwd = mlp_tc_images(w)
    assert fwd.size == 4 * 2 * 64 * 64 and bwd.size == 7 * 2 * 64 * 32
    # forward chunk 3 (outputs 192..255), hi part, row 7 (output 199) holds w[199] up to tf32 rounding
    ch = fwd[3 * 2 * 64 * 64: 3 * 2 * 64 * 64 + 64 * 64]
    rr = 7
    kk = np.arange(64)
    got = ch[(kk // 32) * 64 * 32 + rr * 32 + (((kk % 32) // 4) ^ (rr % 8)) * 4 + (kk % 4)]
    np.testing.assert_allclose(got, w[199], rtol=2.0 ** -11)
    # rows past the last output are zero (hi and lo)
    rr = 40  # output 232
    got = ch[(kk // 32) * 64 * 32 + rr * 32 + (((kk % 32) // 4) ^ (rr % 8)) * 4 + (kk % 4)]
    assert not np.any(got)


def test_edge_tile_layout_round_trip():
    """edge_tiles_to_rows inverts the kernels' 128-edge tile index (common.cuh wt_index)."""
    import torch

    from mace_mlx_b200.model import edge_tiles_to_rows

    E, W = 300, 80
    nch, nt = -(-W // 32), -(-E // 128)
    buf = np.full(nt * nch * 4096, np.nan, np.float32)
    M = np.random.default_rng(0).normal(size=(E, W)).astype(np.float32)
    e = np.arange(E)[:, None]
    c = np.arange(W)[None, :]
    idx = (((e >> 7) * nch + (c >> 5)) << 12) + ((e & 127) << 5) + ((((c >> 2) & 7) ^ (e & 7)) << 2) + (c & 3)
    assert len(np.unique(idx)) == E * W
    buf[idx.ravel()] = M.ravel()
    got = edge_tiles_to_rows(torch.from_numpy(buf), E, W).numpy()
    np.testing.assert_array_equal(got, M)


def test_generated_sc_source_is_current():
    """csrc/sc_gen.cu is what sc_codegen.py writes today."""
    from mace_mlx_b200 import sc_codegen

    assert sc_codegen.OUT.read_text() == sc_codegen.generate()


@pytest.mark.parametrize("name", ["0e", "1o", "2e"])
def test_generated_sc_terms_match_the_polynomial_and_its_gradient(name):
    """The generated forward terms and per-index backward terms equal the table-driven forms."""
    from mace_mlx_b200 import sc_codegen

    ent = sc_codegen.standard_entries(name)
    rng = np.random.default_rng(3)
    G = rng.normal(size=(len(ent), 5))
    f = rng.normal(size=(16, 5))
    dM = 2 * sc_codegen.VARIANTS[name].l + 1
    g = rng.normal(size=(dM, 5))
    ft = torch.tensor(f, requires_grad=True)
    out = torch.zeros(dM, 5, dtype=torch.float64)
    for q, (M, a, b, c, nu) in enumerate(ent.tolist()):
        term = ft[a]
        if nu >= 2:
            term = term * ft[b]
        if nu >= 3:
            term = term * ft[c]
        out[M] = out[M] + torch.tensor(G[q]) * term
    np.testing.assert_allclose(sc_codegen.eval_forward(ent, G, f), out.detach().numpy(), rtol=1e-12, atol=1e-12)
    (out * torch.tensor(g)).sum().backward()
    np.testing.assert_allclose(sc_codegen.eval_backward(ent, G, f, g), ft.grad.numpy(), rtol=1e-10, atol=1e-10)


def test_standard_models_use_the_generated_sc_kernels():
    for arch, sig in [("small", [1, 1]), ("medium", [2, 1]), ("large", [3, 1])]:
        config, weights, _ = make_case(arch, seed=1, z_table=[14])
        pm = PackedModel(ModelSpec.from_config(config), weights)
        assert [pm.desc.layers[t].sc_gen for t in range(2)] == sig, arch
