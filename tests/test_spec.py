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
    cfg = random_config("small")
    for key, val in [("heads", ["a", "b"]), ("use_agnostic_product", True), ("apply_cutoff", False),
                     ("interaction_cls", "RealAgnosticResidualNonLinearInteractionBlock")]:
        c = dict(cfg, **{key: val})
        with pytest.raises(UnsupportedModel):
            ModelSpec.from_config(c)


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
