"""Architecture metadata: instruction lists, slot layouts and the converted
weight-key layout (reference model.py:59-278, utils.py:87-156, linear.py:41-77)."""

import numpy as np
import pytest

from mace_mlx_b200.irreps import Irreps
from mace_mlx_b200.spec import ModelSpec, UnsupportedModel
from mace_mlx_b200.weights import check_weights, load_model_dir, random_config, random_weights, write_random_model


def spec_of(arch, **kw):
    return ModelSpec.from_config(random_config(arch, **kw))


def test_medium_layer1_mid_irreps_and_weight_numel():
    sp = spec_of("medium")
    l0, l1 = sp.layers
    assert [str(m.ir) for m in l0.conv.irreps_mid] == ["0e", "1o", "2e", "3o"]
    assert l0.conv.weight_numel == 512
    # 0e x2, 1o x3, 2e x3, 3o x2 (sorted by (l, p), stable)
    assert [str(m.ir) for m in l1.conv.irreps_mid] == ["0e", "0e", "1o", "1o", "1o", "2e", "2e", "2e", "3o", "3o"]
    assert l1.conv.irreps_mid.dim == 5120
    assert l1.conv.weight_numel == 1280
    # path weights: one path per output slot -> sqrt(2l+1)
    for ins in l1.conv.instrs:
        assert ins.path_weight == pytest.approx(np.sqrt(2 * ins.l3 + 1))
    # hidden irreps: full for all but the last layer
    assert str(l0.hidden) == "128x0e + 128x1o"
    assert str(l1.hidden) == "128x0e"


def test_large_layer1_sizes():
    sp = spec_of("large")
    assert sp.layers[1].conv.weight_numel == 2176
    assert sp.layers[1].conv.irreps_mid.dim == 9088


def test_linear_path_weights_concat_k():
    sp = spec_of("medium")
    lin = sp.layers[1].linear
    # output 1o is fed by three 1o mid slots -> 1/sqrt(3*128)
    for ins in lin.instrs:
        n_src = sum(1 for m in lin.irreps_in if m.ir == lin.irreps_out[ins.i_out].ir)
        assert ins.path_weight == pytest.approx(1 / np.sqrt(128 * n_src))


def test_skip_tp_path_weight():
    sp = spec_of("medium")
    (ins,) = sp.layers[0].skip.instrs
    assert ins.path_weight * ins.cg == pytest.approx(1 / np.sqrt(128 * 89))


def test_weight_keys_follow_reference_layout(tmp_path):
    d = write_random_model(tmp_path / "m", "medium", seed=3)
    config, weights = load_model_dir(d)
    sp = ModelSpec.from_config(config)
    check_weights(sp, weights)
    assert weights["interactions.1.conv_tp_weights.layers.6.weight"].shape == (1280, 64)
    assert weights["interactions.0.conv_tp_weights.layers.0.weight"].shape == (64, 8)
    assert weights["products.0.symmetric_contractions.contractions.1.weights_max"].shape == (89, 51, 128)
    assert weights["products.0.symmetric_contractions.contractions.0.weights.0"].shape == (89, 4, 128)
    assert weights["interactions.0.skip_tp.tp.weights.0"].shape == (128, 89, 128)
    assert weights["readouts.1.linear_1.weights.0"].shape == (128, 16)
    assert weights["readouts.0.linear.weights.0"].shape == (128, 1)
    assert weights["node_embedding.linear.weights.0"].shape == (89, 128)


def test_check_weights_reports_mismatch():
    sp = spec_of("small")
    w = random_weights(sp, 0)
    w["interactions.0.linear.weights.0"] = np.zeros((3, 3), np.float32)
    with pytest.raises(ValueError, match="interactions.0.linear.weights.0"):
        check_weights(sp, w)


def test_unsupported_features_raise():
    """The spec (and so the oracle) reads the mh-1 block and apply_cutoff=False
    with density-normalised blocks; the CUDA path refuses both when the model
    is packed (apply_cutoff=False alone packs, with the envelope flag set), and
    the spec refuses an unknown interaction block and other gates."""
    from mace_mlx_b200.pack import PackedModel

    for kw in (dict(apply_cutoff=False, use_density_normalization=True), dict(nonlinear_interaction=True)):
        cfg = random_config("small", z_table=[14], **kw)
        sp = ModelSpec.from_config(cfg)
        with pytest.raises(UnsupportedModel, match="no CUDA path"):
            PackedModel(sp, random_weights(sp, 0))
    sp = ModelSpec.from_config(random_config("small", z_table=[14], apply_cutoff=False))
    assert PackedModel(sp, random_weights(sp, 0)).desc.envelope_on_weights == 1
    for key, val in [("interaction_cls", "SomeOtherInteractionBlock"), ("gate", "tanh")]:
        with pytest.raises(UnsupportedModel):
            ModelSpec.from_config(dict(random_config("small"), **{key: val}))


def test_nonlinear_block_layout():
    """mh-1 layout (blocks.py:628-743, model.py:192-211, converter.py:677-822):
    scalar-only edge irreps in the first layer, gate input = scalars + one gate
    block per non-scalar block + non-scalars, radial-MLP input num_bessel + 2 C,
    LayerNorm MLP module indices 0/1/3/4/..., alpha and beta scalars."""
    cfg = random_config("medium", z_table=[14, 6], nonlinear_interaction=True, edge_irreps="128x0e + 128x1o + 128x2e")
    sp = ModelSpec.from_config(cfg)
    l0, l1 = sp.layers
    assert str(l0.nonlinear.edge_irreps) == "128x0e" and str(l1.nonlinear.edge_irreps) == "128x0e + 128x1o + 128x2e"
    assert str(l1.linear.irreps_out) == "128x0e + 128x0e + 128x0e + 128x0e + 128x1o + 128x2e + 128x3o"
    assert l0.mlp_widths[0] == sp.num_bessel + 2 * 128 and l0.nonlinear.density_widths == [l0.mlp_widths[0], 64, 1]
    shapes = sp.weight_shapes()
    assert shapes["interactions.0.conv_tp_weights.layers.9.weight"] == (l0.conv.weight_numel, 64)
    assert shapes["interactions.0.conv_tp_weights.layers.7.bias"] == (64,)
    assert shapes["interactions.1.density_fn.layers.3.weight"] == (1, 64)
    assert shapes["interactions.1.source_embedding.weights.0"] == (2, 128)
    assert shapes["interactions.1.alpha"] == () and "interactions.1.skip_tp.tp.weights.0" not in shapes
    check_weights(sp, random_weights(sp, 0))


def test_multi_head_spec_shapes_and_head_selection():
    """Multi-head layout (model.py:89-93, 135-138, converter.py:176-200): readouts of
    H x 0e, a 16 H-wide non-linear readout, (H, elements) atomic energies; per-head
    scale/shift (model.py:527-548); head by name (calculators.py:128-137)."""
    cfg = random_config("medium", z_table=[14, 6], heads=["pt_head", "r2scan", "Default"],
                        atomic_energies=[[-1.0, -2.0], [-3.0, -4.0], [-5.0, -6.0]], model_type="ScaleShiftMACE")
    cfg["scale"], cfg["shift"] = [1.5, 2.5], [0.1, 0.2]
    sp = ModelSpec.from_config(cfg)
    assert sp.num_heads == 3 and sp.head_idx == 0
    shapes = sp.weight_shapes()
    assert shapes["atomic_energies_fn.atomic_energies"] == (3, 2)
    assert shapes["readouts.0.linear.weights.0"] == (sp.C, 3)
    assert shapes["readouts.1.linear_1.weights.0"] == (sp.C, 48)
    assert shapes["readouts.1.linear_2.weights.0"] == (48, 3)
    # linear_2's path weight keeps the full 16 H fan-in
    assert sp.layers[1].readout_2.instrs[0].path_weight == pytest.approx(1 / np.sqrt(48))
    check_weights(sp, random_weights(sp, 0))
    s1 = ModelSpec.from_config(cfg, head="r2scan")
    assert s1.head_idx == 1 and (s1.scale, s1.shift) == (2.5, 0.2)
    np.testing.assert_array_equal(s1.head_atomic_energies(cfg["atomic_energies"]), [-3.0, -4.0])
    s2 = ModelSpec.from_config(cfg, head="Default")  # past the scale list's end: its first entry
    assert s2.head_idx == 2 and (s2.scale, s2.shift) == (1.5, 0.1)
    with pytest.raises(ValueError, match="not found"):
        ModelSpec.from_config(cfg, head="nope")
    # a single-head model ignores the head name, as the reference's calculator does
    assert ModelSpec.from_config(random_config("small"), head="nope").head_idx == 0
    bad = dict(cfg, atomic_energies=[0.0, 0.0])
    with pytest.raises(UnsupportedModel):
        ModelSpec.from_config(bad)


def test_multi_head_pack_slices_the_head():
    """The packed readout of head h is linear_1's columns and linear_2's rows of
    the head's 16-scalar block, column h, with the path weights of the full layer."""
    from mace_mlx_b200.pack import PackedModel

    cfg = random_config("medium", z_table=[14], heads=["a", "b"], atomic_energies=[[-1.0], [-2.0]])
    sp = ModelSpec.from_config(cfg, head="b")
    w = random_weights(sp, 2)
    pm = PackedModel(sp, w)
    f = pm.floats
    d0, d1 = pm.desc.layers[0], pm.desc.layers[1]
    C = sp.C
    np.testing.assert_allclose(f[d0.f_ro1:d0.f_ro1 + C], w["readouts.0.linear.weights.0"][:, 1] / np.sqrt(C),
                               rtol=1e-6)
    assert d1.readout_hidden == 16
    w1 = w["readouts.1.linear_1.weights.0"][:, 16:32] / np.sqrt(C)
    np.testing.assert_allclose(f[d1.f_ro1:d1.f_ro1 + C * 16].reshape(C, 16), w1, rtol=1e-6)
    np.testing.assert_allclose(f[d1.f_ro2:d1.f_ro2 + 16], w["readouts.1.linear_2.weights.0"][16:32, 1] / np.sqrt(32),
                               rtol=1e-6)
    assert f[pm.desc.f_e0] == np.float32(-2.0)


def test_masked_multi_head_readout_equals_the_sliced_single_head_model():
    """The identity the packed readout relies on, in the float64 oracle: head h of
    a two-head model (masked 32-scalar readout, blocks.py:602-609) equals a
    single-head model holding the head's weight slices, linear_2 rescaled from the
    1/sqrt(32) path weight to the single-head 1/sqrt(16)."""
    from mace_mlx_b200.structures import diamond_si
    from oracle.model import OracleMACE
    from oracle.nl import neighbour_list

    cfg = random_config("small", z_table=[14], heads=["a", "b"], atomic_energies=[[-1.0], [-2.0]],
                        model_type="ScaleShiftMACE", avg_num_neighbors=20.0)
    cfg["scale"], cfg["shift"] = [0.7, 1.2], [0.1, -0.3]
    w = random_weights(ModelSpec.from_config(cfg), 4)
    st = diamond_si(1, 0.05, 3)
    i, j, S = neighbour_list(st.positions, st.cell, st.pbc, cfg["r_max"])
    sp = np.zeros(len(st), int)
    h = 1
    one = {k: v for k, v in cfg.items() if k != "heads"}
    one["atomic_energies"], one["scale"], one["shift"] = cfg["atomic_energies"][h], cfg["scale"][h], cfg["shift"][h]
    w1 = dict(w)
    w1["atomic_energies_fn.atomic_energies"] = w["atomic_energies_fn.atomic_energies"][h]
    w1["readouts.0.linear.weights.0"] = w["readouts.0.linear.weights.0"][:, h:h + 1]
    w1["readouts.1.linear_1.weights.0"] = w["readouts.1.linear_1.weights.0"][:, 16 * h:16 * h + 16]
    w1["readouts.1.linear_2.weights.0"] = w["readouts.1.linear_2.weights.0"][16 * h:16 * h + 16, h:h + 1] * np.sqrt(0.5)
    multi = OracleMACE(cfg, w, head="b").compute(st.positions, sp, i, j, S, st.cell, stress=True)
    single = OracleMACE(one, w1).compute(st.positions, sp, i, j, S, st.cell, stress=True)
    for k in ("energy", "node_energy", "forces", "stress"):
        np.testing.assert_allclose(multi[k], single[k], rtol=1e-10, atol=1e-12)


def test_agnostic_product_layout_and_replicated_tables():
    """use_agnostic_product: symmetric-contraction weights of one element
    (model.py:250-258); the packed polynomial tables repeat them per element."""
    from mace_mlx_b200.pack import PackedModel

    cfg = random_config("medium", z_table=[14, 6, 8], use_agnostic_product=True)
    sp = ModelSpec.from_config(cfg)
    shapes = sp.weight_shapes()
    assert shapes["products.0.symmetric_contractions.contractions.0.weights_max"][0] == 1
    assert shapes["products.1.symmetric_contractions.contractions.0.weights.0"][0] == 1
    assert shapes["interactions.0.skip_tp.tp.weights.0"][1] == 3  # the skip stays species-indexed
    pm = PackedModel(sp, random_weights(sp, 1))
    so = pm.desc.layers[0].sc[0]
    G = pm.floats[so.f_G:so.f_G + 3 * so.n_ent * sp.C].reshape(3, so.n_ent, sp.C)
    np.testing.assert_array_equal(G[0], G[1])
    np.testing.assert_array_equal(G[0], G[2])


def test_agnostic_product_equals_replicated_species_weights():
    """In the float64 oracle, the agnostic product (all-ones node attributes,
    blocks.py:527-531) equals the element-indexed product whose weights repeat
    the single set for every element."""
    from mace_mlx_b200.structures import diamond_si
    from oracle.model import OracleMACE
    from oracle.nl import neighbour_list

    cfg = random_config("small", z_table=[14, 6], use_agnostic_product=True, avg_num_neighbors=20.0)
    w = random_weights(ModelSpec.from_config(cfg), 6)
    st = diamond_si(1, 0.05, 4)
    st.numbers[::2] = 6
    i, j, S = neighbour_list(st.positions, st.cell, st.pbc, cfg["r_max"])
    sp = np.where(st.numbers == 14, 0, 1)
    plain = {k: v for k, v in cfg.items() if k != "use_agnostic_product"}
    w2 = {k: (np.repeat(v, 2, axis=0) if ".symmetric_contractions." in k else v) for k, v in w.items()}
    a = OracleMACE(cfg, w).compute(st.positions, sp, i, j, S, st.cell, stress=True)
    b = OracleMACE(plain, w2).compute(st.positions, sp, i, j, S, st.cell, stress=True)
    for k in ("energy", "node_energy", "forces", "stress"):
        np.testing.assert_allclose(a[k], b[k], rtol=1e-10, atol=1e-12)


def test_unknown_head_raises_before_any_device_work():
    from mace_mlx_b200.model import MACEModel

    cfg = random_config("small", z_table=[14], heads=["a", "b"], atomic_energies=[[-1.0], [-2.0]])
    w = random_weights(ModelSpec.from_config(cfg), 0)
    with pytest.raises(ValueError, match="not found in model heads"):
        MACEModel(config=cfg, weights=w, device=0, head="c")


def test_mpa_family_config_and_weight_layout():
    """Density normalisation, Agnesi and ZBL as the reference's converter
    writes them (converter.py:205-300): density_fn weights per layer, the
    Agnesi radii table from the config, ZBL constants, z_table required."""
    cfg = random_config("medium", z_table=[3, 8], first_interaction_nonresidual=True,
                        use_density_normalization=True, distance_transform={}, pair_repulsion={"p": 5})
    assert cfg["interaction_cls"] == "RealAgnosticDensityInteractionBlock"
    sp = ModelSpec.from_config(cfg)
    assert all(lay.density for lay in sp.layers)
    assert sp.agnesi["q"] == pytest.approx(0.9183) and len(sp.agnesi["covalent_radii"]) == 119
    assert sp.zbl["p"] == 5 and sp.zbl["a_exp"] == pytest.approx(0.3)
    assert sp.species_numbers() == [3, 8]
    shapes = sp.weight_shapes()
    assert shapes["interactions.0.density_fn.weight"] == (1, sp.num_bessel)
    assert shapes["interactions.1.density_fn.weight"] == (1, sp.num_bessel)
    c = dict(cfg)
    c.pop("z_table")
    with pytest.raises(UnsupportedModel):
        ModelSpec.from_config(c)


def test_non_residual_first_layer_skip_on_message():
    sp = spec_of("medium", first_interaction_nonresidual=True)
    assert not sp.layers[0].residual
    assert sp.layers[1].residual
    assert [str(m.ir) for m in sp.layers[0].skip.irreps_out] == ["0e", "1o", "2e", "3o"]


def test_irreps_sh():
    assert str(Irreps.spherical_harmonics(3)) == "1x0e + 1x1o + 1x2e + 1x3o"


@pytest.mark.parametrize("n", [1, 7, 1000, 1001])
def test_calculator_transfer_blocks_are_aligned_and_disjoint(n):
    """One host->device and one device->host copy per step: the named views of
    the two blocks start 64-byte aligned, fit their block and do not overlap."""
    import torch

    from mace_mlx_b200.calculators import MACEMLXCalculator

    n_in = 16 + 3 * n
    n_out = (128 + 12 * n + 63) // 64 * 64 + 4 * n
    blk_in = torch.empty(n_in, dtype=torch.float32)
    blk_out = torch.empty(n_out, dtype=torch.uint8)
    v = MACEMLXCalculator._views(n, blk_in, blk_out)
    assert v["pos"].shape == (n, 3) and v["cell"].shape == (3, 3) and v["forces"].shape == (n, 3)
    assert v["energy"].dtype == torch.float64 and v["energy"].numel() == 1 and v["virial"].numel() == 9
    assert v["node_energy"].shape == (n,) and v["node_energy"].dtype == torch.float32
    for blk, names in ((blk_in, ("cell", "pos")), (blk_out, ("energy", "virial", "forces", "node_energy"))):
        base = blk.data_ptr()
        spans = []
        for k in names:
            t = v[k]
            off = t.data_ptr() - base
            assert off % 64 == 0 or k in ("virial",), (k, off)  # virial follows the 8-byte energy
            spans.append((off, off + t.numel() * t.element_size()))
        spans.sort()
        assert spans[-1][1] <= blk.numel() * blk.element_size()
        assert all(a[1] <= b[0] for a, b in zip(spans, spans[1:]))
