"""MACE architecture description derived from a converted-model ``config.json``.

Everything here is construction-time metadata: which irreps each layer carries,
the instruction lists of every equivariant op, their path weights, and the
flat weight-key names of the converted layout.  The construction mirrors the
reference's module tree so that a ``weights.npz`` written for the reference
(``converter.py``) loads unchanged:

* layer irreps and block choice: ``model.py:59-278``
* conv_tp instructions/paths: ``utils.py:87-156`` (uvu, path weight
  ``sqrt(dim_out / sum mul2)``, stable sort of the output slots)
* o3.Linear instructions: ``linear.py:41-77`` (outer loop over input slots,
  inner over output slots, path weight ``1/sqrt(sum mul_in)`` per output)
* skip_tp (FullyConnectedTensorProduct, uvw): ``tensor_product.py:1046-1110``
* symmetric contraction weights: ``symmetric_contraction.py:159-261``; one
  weight set for every element under ``use_agnostic_product`` (``model.py:250-258``,
  ``blocks.py:510, 527-531``)
* readouts: ``blocks.py:540-608``
* density-normalised blocks (``use_density_normalization``): ``blocks.py:282-490``
  (``density_fn`` = bias-free Linear(num_bessel -> 1) per layer)
* Agnesi distance transform (``distance_transform``): ``radial.py:202-262``
* multi-head models (``heads``): readouts of ``H x 0e`` and a ``16 H x 0e``
  non-linear readout MLP (``model.py:89-93, 135-138``, ``blocks.py:553-609``),
  per-head atomic energies and scale/shift (``model.py:302-326, 518-548``),
  head chosen by name (``calculators.py:128-137``)
* ZBL pair repulsion (``pair_repulsion``): ``radial.py:127-199``, wired in
  ``model.py:154-173, 213-231``
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from .cg import U_matrix_real, wigner_3j
from .elements import AGNESI_DEFAULTS, COVALENT_RADII, ZBL_DEFAULTS
from .irreps import Irrep, Irreps

NONLINEAR_INTERACTION = "RealAgnosticResidualNonLinearInteractionBlock"
SUPPORTED_INTERACTIONS = (
    NONLINEAR_INTERACTION,
    "RealAgnosticResidualInteractionBlock",
    "RealAgnosticInteractionBlock",
    "RealAgnosticDensityInteractionBlock",
    "RealAgnosticDensityResidualInteractionBlock",
)


class UnsupportedModel(NotImplementedError):
    pass


@dataclass
class LinearInstr:
    i_in: int
    i_out: int
    mul_in: int
    mul_out: int
    dim: int
    path_weight: float


@dataclass
class LinearSpec:
    """e3nn o3.Linear between two Irreps (weights shared over m)."""

    irreps_in: Irreps
    irreps_out: Irreps
    instrs: list[LinearInstr]

    @staticmethod
    def build(irreps_in: Irreps, irreps_out: Irreps) -> "LinearSpec":
        tot = {
            io: sum(m.mul for m in irreps_in if m.ir == mo.ir)
            for io, mo in enumerate(irreps_out)
        }
        instrs = []
        for ii, mi in enumerate(irreps_in):
            for io, mo in enumerate(irreps_out):
                if mi.ir != mo.ir:
                    continue
                pw = 1.0 / math.sqrt(tot[io]) if tot[io] > 0 else 1.0
                instrs.append(LinearInstr(ii, io, mi.mul, mo.mul, mi.ir.dim, pw))
        return LinearSpec(irreps_in, irreps_out, instrs)

    def weight_shapes(self) -> list[tuple[int, int]]:
        return [(i.mul_in, i.mul_out) for i in self.instrs]


@dataclass
class SkipInstr:
    i_in1: int
    i_out: int
    mul1: int
    mul2: int
    mul_out: int
    dim: int
    path_weight: float
    cg: float  # the diagonal value of wigner_3j(l, 0, l)


@dataclass
class SkipSpec:
    """FullyConnectedTensorProduct(x, one_hot(species)) -> irreps_out (uvw)."""

    irreps_in1: Irreps
    num_elements: int
    irreps_out: Irreps
    instrs: list[SkipInstr]

    @staticmethod
    def build(irreps_in1: Irreps, num_elements: int, irreps_out: Irreps) -> "SkipSpec":
        attrs = Irreps(f"{num_elements}x0e")
        raw = []
        for i1, m1 in enumerate(irreps_in1):
            for i2, m2 in enumerate(attrs):
                for io, mo in enumerate(irreps_out):
                    if m1.ir.p * m2.ir.p != mo.ir.p:
                        continue
                    if not (abs(m1.ir.l - m2.ir.l) <= mo.ir.l <= m1.ir.l + m2.ir.l):
                        continue
                    raw.append((i1, i2, io))
        alpha: dict[int, float] = {}
        for i1, i2, io in raw:
            alpha[io] = alpha.get(io, 0.0) + irreps_in1[i1].mul * attrs[i2].mul
        instrs = []
        for i1, i2, io in raw:
            dim = irreps_out[io].ir.dim
            pw = math.sqrt(dim / alpha[io]) if alpha[io] > 0 else 1.0
            l = irreps_in1[i1].ir.l
            c = float(wigner_3j(l, 0, l)[0, 0, 0])
            instrs.append(
                SkipInstr(i1, io, irreps_in1[i1].mul, num_elements, irreps_out[io].mul,
                          irreps_in1[i1].ir.dim, pw, c)
            )
        return SkipSpec(irreps_in1, num_elements, irreps_out, instrs)

    def weight_shapes(self) -> list[tuple[int, int, int]]:
        return [(i.mul1, i.mul2, i.mul_out) for i in self.instrs]


@dataclass
class ConvInstr:
    """One uvu path of the conv tensor product (mul2 == 1, one per output slot)."""

    i_in1: int
    l1: int
    l2: int
    l3: int
    p3: int
    path_weight: float
    mul: int

    @property
    def cg(self) -> np.ndarray:
        """Path-weighted coupling tensor (2l1+1, 2l2+1, 2l3+1)."""
        return wigner_3j(self.l1, self.l2, self.l3) * self.path_weight


@dataclass
class ConvSpec:
    irreps_in1: Irreps
    irreps_sh: Irreps
    irreps_mid: Irreps
    instrs: list[ConvInstr]  # instrs[k] writes mid slot k, weight slice k

    @staticmethod
    def build(irreps_in1: Irreps, irreps_sh: Irreps, target: Irreps) -> "ConvSpec":
        outs: list = []
        raw = []
        for i, (mul, ir_in) in enumerate(irreps_in1):
            for j, (mul2, ir_edge) in enumerate(irreps_sh):
                for ir_out in ir_in.couple(ir_edge):
                    if target.has(ir_out):
                        k = len(outs)
                        outs.append((mul, ir_out))
                        raw.append((i, j, k, mul2))
        alpha: dict[int, float] = {}
        for i, j, k, mul2 in raw:
            alpha[k] = alpha.get(k, 0.0) + mul2
        mid = Irreps(outs)
        mid_sorted, _, inv = mid.sort()
        instrs = []
        for i, j, k, mul2 in raw:
            ir_out = outs[k][1]
            pw = math.sqrt(ir_out.dim / alpha[k]) if alpha[k] > 0 else 1.0
            instrs.append((inv[k], i, j, ir_out, pw))
        instrs.sort(key=lambda t: t[0])
        if [t[0] for t in instrs] != list(range(len(instrs))):
            raise UnsupportedModel("conv_tp must have exactly one path per output slot")
        out = []
        for k, i, j, ir_out, pw in instrs:
            l1 = irreps_in1[i].ir.l
            l2 = irreps_sh[j].ir.l
            out.append(ConvInstr(i, l1, l2, ir_out.l, ir_out.p, pw, irreps_in1[i].mul))
        return ConvSpec(irreps_in1, irreps_sh, mid_sorted, out)

    @property
    def weight_numel(self) -> int:
        return sum(i.mul for i in self.instrs)


@dataclass
class SCOutput:
    """Symmetric contraction for one output irrep (one ``Contraction``)."""

    ir_out: Irrep
    correlation: int
    U: list[np.ndarray]  # U[nu-1] for nu = 1..correlation, shape ([d_out,] 16^nu, K_nu)
    num_params: list[int]  # K_nu


@dataclass
class SCSpec:
    irreps_in: Irreps
    irreps_out: Irreps
    coupling: Irreps
    num_elements: int
    C: int
    outputs: list[SCOutput]

    @staticmethod
    def build(irreps_in: Irreps, irreps_out: Irreps, correlation: int, num_elements: int) -> "SCSpec":
        coupling = Irreps([(1, m.ir) for m in irreps_in])
        C = irreps_in.count("0e")
        outs = []
        for mul, ir in irreps_out:
            Us = [U_matrix_real(coupling, ir, nu) for nu in range(1, correlation + 1)]
            outs.append(SCOutput(ir, correlation, Us, [u.shape[-1] for u in Us]))
        return SCSpec(irreps_in, irreps_out, coupling, num_elements, C, outs)


@dataclass
class NonLinearSpec:
    """The mh-1 family's RealAgnosticResidualNonLinearInteractionBlock
    (``blocks.py:611-807``): species embeddings concatenated to the radial
    features, radial MLPs with biases and LayerNorm (``radial.py:344-357``), a
    density MLP normalising the message by ``density * beta + alpha``, a
    residual ``linear_res`` of ``linear_up``'s output, an equivariant gate
    (``gate.py``) and ``linear_2``; ``skip_tp`` is a plain linear."""

    edge_irreps: Irreps
    C0: int  # scalar channels of the block's input (width of each species embedding)
    aug_dim: int  # num_bessel + 2 C0: the radial MLPs' input
    embed: LinearSpec  # one-hot (num_elements x 0e) -> C0 x 0e, source and target
    skip_lin: LinearSpec  # irreps_in -> hidden
    linear_res: LinearSpec  # edge_irreps -> gate input
    linear_2: LinearSpec  # irreps_out -> irreps_out
    gate_scalars: Irreps
    gate_gates: Irreps
    gate_gated: Irreps
    density_widths: list[int]  # [aug_dim, 64, 1]


@dataclass
class LayerSpec:
    index: int
    irreps_in: Irreps
    hidden: Irreps  # product output irreps of this layer
    residual: bool
    skip: SkipSpec | None  # None for the non-linear block (its skip is ``nonlinear.skip_lin``)
    linear_up: LinearSpec
    conv: ConvSpec
    mlp_widths: list[int]  # [num_bessel, *radial_MLP, weight_numel]
    linear: LinearSpec
    sc: SCSpec
    prod_linear: LinearSpec
    readout_nonlinear: bool
    density: bool = False  # message / (sum_e tanh((w_d . b_e)^2) + 1) instead of / avg_num_neighbors
    readout_linear: LinearSpec | None = None  # linear readout (not last)
    readout_1: LinearSpec | None = None  # nonlinear readout
    readout_2: LinearSpec | None = None
    nonlinear: NonLinearSpec | None = None  # mh-1 non-linear interaction block


def _add_readouts(lay: LayerSpec, t: int, T: int, layer_hidden: Irreps, H: int) -> None:
    lay.readout_nonlinear = t == T - 1
    if t < T - 1:
        lay.readout_linear = LinearSpec.build(layer_hidden, Irreps(f"{H}x0e"))
    else:
        # 16 hidden scalars per head (model.py:135-138)
        lay.readout_1 = LinearSpec.build(layer_hidden, Irreps(f"{16 * H}x0e"))
        lay.readout_2 = LinearSpec.build(Irreps(f"{16 * H}x0e"), Irreps(f"{H}x0e"))


def _nonlinear_layer(t: int, layer_in: Irreps, layer_hidden: Irreps, edge: Irreps, sh: Irreps,
                     inter_irreps: Irreps, num_bessel: int, radial_MLP: list[int], num_elements: int,
                     correlation: int, sc_elements: int) -> LayerSpec:
    """One non-linear interaction block (blocks.py:628-743): gate irreps split
    from irreps_out (scalars; one gate scalar block per non-scalar block; the
    non-scalars), every linear of the block, the augmented radial-MLP input."""
    C0 = layer_in.count("0e")
    scal = Irreps([m for m in inter_irreps if m.ir.l == 0])
    gated = Irreps([m for m in inter_irreps if m.ir.l > 0])
    gates = Irreps([(m.mul, "0e") for m in gated])
    nonlin = Irreps(list(scal) + list(gates) + list(gated))
    conv = ConvSpec.build(edge, sh, inter_irreps)
    aug = num_bessel + 2 * C0
    nl = NonLinearSpec(
        edge_irreps=edge, C0=C0, aug_dim=aug,
        embed=LinearSpec.build(Irreps(f"{num_elements}x0e"), Irreps(f"{C0}x0e")),
        skip_lin=LinearSpec.build(layer_in, layer_hidden),
        linear_res=LinearSpec.build(edge, nonlin),
        linear_2=LinearSpec.build(inter_irreps, inter_irreps),
        gate_scalars=scal, gate_gates=gates, gate_gated=gated,
        density_widths=[aug, 64, 1],
    )
    return LayerSpec(
        index=t, irreps_in=layer_in, hidden=layer_hidden, residual=True, skip=None,
        linear_up=LinearSpec.build(layer_in, edge), conv=conv,
        mlp_widths=[aug, *radial_MLP, conv.weight_numel],
        linear=LinearSpec.build(conv.irreps_mid, nonlin),  # linear_1
        sc=SCSpec.build(inter_irreps, layer_hidden, correlation, sc_elements),
        prod_linear=LinearSpec.build(layer_hidden, layer_hidden),
        readout_nonlinear=False, nonlinear=nl,
    )


def _radial_mlp_ln_shapes(prefix: str, widths: list[int]) -> dict:
    """Linear(bias) -> LayerNorm -> SiLU stacks (radial.py:344-357): module
    index 3 j for the j-th Linear, 3 j + 1 for its LayerNorm."""
    s = {}
    for j in range(len(widths) - 1):
        s[f"{prefix}.layers.{3 * j}.weight"] = (widths[j + 1], widths[j])
        s[f"{prefix}.layers.{3 * j}.bias"] = (widths[j + 1],)
        if j < len(widths) - 2:
            s[f"{prefix}.layers.{3 * j + 1}.weight"] = (widths[j + 1],)
            s[f"{prefix}.layers.{3 * j + 1}.bias"] = (widths[j + 1],)
    return s


def _nonlinear_weight_shapes(lay: LayerSpec, p: str) -> dict:
    """The non-linear block's arrays besides linear_up (converter.py:677-780)."""
    nl = lay.nonlinear
    s: dict[str, tuple[int, ...]] = {}
    for name, lin in (("source_embedding", nl.embed), ("target_embedding", nl.embed), ("skip_tp", nl.skip_lin),
                      ("linear_res", nl.linear_res), ("linear_1", lay.linear), ("linear_2", nl.linear_2)):
        for k, sh in enumerate(lin.weight_shapes()):
            s[f"{p}.{name}.weights.{k}"] = sh
    s.update(_radial_mlp_ln_shapes(f"{p}.conv_tp_weights", lay.mlp_widths))
    s.update(_radial_mlp_ln_shapes(f"{p}.density_fn", nl.density_widths))
    s[f"{p}.alpha"] = ()
    s[f"{p}.beta"] = ()
    return s


def resolve_head(heads: list[str], head: str | None) -> int:
    """Index of the selected head: the first by default; a name that is not one
    of a multi-head model's heads raises ``ValueError`` (``calculators.py:128-137``;
    a single-head model ignores the name, as there)."""
    if len(heads) == 1 or head is None:
        return 0
    if head not in heads:
        raise ValueError(f"Head '{head}' not found in model heads: {heads}")
    return heads.index(head)


def _per_head(v, head_idx: int) -> float:
    """A scale or shift entry: a scalar, or one value per head where a head past
    the list's end takes the first (``model.py:527-548``)."""
    if isinstance(v, (list, tuple)):
        vals = [float(x) for x in v]
        return vals[head_idx] if head_idx < len(vals) else vals[0]
    return float(v)


@dataclass
class ModelSpec:
    config: dict
    r_max: float
    num_bessel: int
    poly_p: int
    max_ell: int
    num_interactions: int
    num_elements: int
    hidden: Irreps
    C: int
    avg_num_neighbors: float
    radial_MLP: list[int]
    model_type: str
    scale: float
    shift: float
    z_table: list[int] | None
    atomic_energies: np.ndarray  # (num_elements,), or (num_heads, num_elements)
    irreps_sh: Irreps
    interaction_irreps: Irreps
    layers: list[LayerSpec] = field(default_factory=list)
    density: bool = False
    agnesi: dict | None = None  # {"q", "p", "a", "covalent_radii" (indexed by Z)}
    zbl: dict | None = None  # {"p", "a_exp", "a_prefactor", "covalent_radii" (indexed by Z)}
    apply_cutoff: bool = True
    heads: list[str] = field(default_factory=lambda: ["Default"])
    head_idx: int = 0  # the selected head; scale / shift above are already that head's

    @property
    def num_heads(self) -> int:
        return len(self.heads)

    def head_atomic_energies(self, ae) -> np.ndarray:
        """The selected head's per-element energies from a 1-D or (heads, elements)
        table: column ``head`` of ``onehot @ ae.T`` (``blocks.py:53-65``,
        ``model.py:315-326``)."""
        a = np.atleast_2d(np.asarray(ae, dtype=np.float64))
        if self.num_heads == 1:
            return a.reshape(-1)[-self.num_elements:]
        if a.shape != (self.num_heads, self.num_elements):
            raise UnsupportedModel(f"atomic energies of shape {a.shape} for {self.num_heads} heads")
        return a[self.head_idx]

    def species_numbers(self) -> list[int]:
        """Atomic number of every model element index (z_table)."""
        if self.z_table is None:
            raise UnsupportedModel("the distance transform / pair repulsion need the config's z_table")
        return [int(z) for z in self.z_table]

    # ------------------------------------------------------------------
    @staticmethod
    def from_config(config: dict, head: str | None = None) -> "ModelSpec":
        """``head``: the head name of a multi-head model (default: its first head)."""
        cfg = dict(config)
        model_type = cfg.get("model_type", "ScaleShiftMACE")
        density = bool(cfg.get("use_density_normalization", False))
        agnesi = None
        if cfg.get("distance_transform") is not None:
            dt = dict(cfg["distance_transform"])
            agnesi = {k: float(dt.get(k, v)) for k, v in AGNESI_DEFAULTS.items()}
            # the converter writes the radii table into the config (converter.py:274-282)
            agnesi["covalent_radii"] = [float(x) for x in (dt.get("covalent_radii") or COVALENT_RADII)]
        zbl = None
        if cfg.get("pair_repulsion"):
            pr = cfg["pair_repulsion"] if isinstance(cfg["pair_repulsion"], dict) else {}
            zbl = {"p": int(pr.get("p", ZBL_DEFAULTS["p"])), "a_exp": float(pr.get("a_exp", ZBL_DEFAULTS["a_exp"])),
                   "a_prefactor": float(pr.get("a_prefactor", ZBL_DEFAULTS["a_prefactor"]))}
            # the reference reads ase.data.covalent_radii at run time (radial.py:150-152)
            zbl["covalent_radii"] = list(COVALENT_RADII)
        # species-agnostic product: one symmetric-contraction weight set (model.py:250-258)
        agnostic = bool(cfg.get("use_agnostic_product", False))
        # apply_cutoff=False: the envelope multiplies the radial-MLP output and
        # the edge densities instead of the Bessel features (radial.py:313-317)
        apply_cutoff = bool(cfg.get("apply_cutoff", True))
        heads = [str(h) for h in (cfg.get("heads") or ["Default"])]
        head_idx = resolve_head(heads, head)
        inter_cls = cfg.get("interaction_cls", "RealAgnosticResidualInteractionBlock")
        if inter_cls not in SUPPORTED_INTERACTIONS:
            raise UnsupportedModel(f"interaction block {inter_cls} is not supported yet")
        gate = cfg.get("gate", "silu")
        if gate not in ("silu", None):
            raise UnsupportedModel(f"gate {gate!r} is not supported")

        r_max = float(cfg["r_max"])
        num_bessel = int(cfg.get("num_bessel", 10))
        poly_p = int(cfg.get("num_polynomial_cutoff", 5))
        max_ell = int(cfg.get("max_ell", 3))
        T = int(cfg.get("num_interactions", 2))
        hidden = Irreps(cfg.get("hidden_irreps", "128x0e"))
        corr = cfg.get("correlation", 3)
        corr = [int(corr)] * T if isinstance(corr, int) else [int(c) for c in corr]
        num_elements = int(cfg.get("num_elements", 89))
        avg = float(cfg.get("avg_num_neighbors", 1.0))
        radial_MLP = list(cfg.get("radial_MLP") or [64, 64, 64])
        first_nonres = bool(cfg.get("first_interaction_nonresidual", False))
        ae = cfg.get("atomic_energies")
        ae = np.zeros(num_elements) if ae is None else np.asarray(ae, dtype=np.float64)
        if ae.ndim == 2 and ae.shape[0] == 1 and len(heads) == 1:
            ae = ae[0]
        if len(heads) > 1 and (ae.ndim != 2 or ae.shape[0] != len(heads)):
            raise UnsupportedModel(f"a {len(heads)}-head model needs one row of atomic energies per head")

        sh = Irreps.spherical_harmonics(max_ell)
        C = hidden[0].mul
        if any(m.mul != C for m in hidden):
            raise UnsupportedModel("hidden irreps must share one multiplicity")
        inter_irreps = Irreps([(C, ir) for _, ir in sh])
        hidden_scalar = hidden.scalars()

        spec = ModelSpec(
            config=config, r_max=r_max, num_bessel=num_bessel, poly_p=poly_p,
            max_ell=max_ell, num_interactions=T, num_elements=num_elements,
            hidden=hidden, C=C, avg_num_neighbors=avg, radial_MLP=radial_MLP,
            model_type=model_type, scale=_per_head(cfg.get("scale", 1.0), head_idx),
            shift=_per_head(cfg.get("shift", 0.0), head_idx), z_table=cfg.get("z_table"),
            atomic_energies=ae, irreps_sh=sh, interaction_irreps=inter_irreps,
            density=density, agnesi=agnesi, zbl=zbl, heads=heads, head_idx=head_idx, apply_cutoff=apply_cutoff,
        )
        if (agnesi or zbl) and spec.z_table is None:
            raise UnsupportedModel("the distance transform / pair repulsion need the config's z_table")

        H = len(heads)
        layer_in = hidden_scalar
        nonlinear = inter_cls == NONLINEAR_INTERACTION
        edge_cfg = Irreps(cfg["edge_irreps"]) if cfg.get("edge_irreps") else None
        for t in range(T):
            layer_hidden = hidden if t < T - 1 else hidden_scalar
            if nonlinear:
                # the first layer keeps the scalar part of edge_irreps (model.py:192-211)
                edge = (edge_cfg.scalars() if t == 0 else edge_cfg) if edge_cfg is not None else layer_in
                spec.layers.append(_nonlinear_layer(t, layer_in, layer_hidden, edge, sh, inter_irreps, num_bessel,
                                                    radial_MLP, num_elements, corr[t],
                                                    1 if agnostic else num_elements))
                _add_readouts(spec.layers[-1], t, T, layer_hidden, H)
                layer_in = layer_hidden
                continue
            residual = not (t == 0 and first_nonres)
            if residual:
                skip = SkipSpec.build(layer_in, num_elements, layer_hidden)
            else:
                skip = SkipSpec.build(inter_irreps, num_elements, inter_irreps)
            conv = ConvSpec.build(layer_in, sh, inter_irreps)
            lay = LayerSpec(
                index=t,
                irreps_in=layer_in,
                hidden=layer_hidden,
                residual=residual,
                skip=skip,
                linear_up=LinearSpec.build(layer_in, layer_in),
                conv=conv,
                mlp_widths=[num_bessel, *radial_MLP, conv.weight_numel],
                linear=LinearSpec.build(conv.irreps_mid, inter_irreps),
                sc=SCSpec.build(inter_irreps, layer_hidden, corr[t], 1 if agnostic else num_elements),
                prod_linear=LinearSpec.build(layer_hidden, layer_hidden),
                readout_nonlinear=(t == T - 1),
                density=density,
            )
            _add_readouts(lay, t, T, layer_hidden, H)
            spec.layers.append(lay)
            layer_in = layer_hidden
        return spec

    # ------------------------------------------------------------------
    def weight_shapes(self) -> dict[str, tuple[int, ...]]:
        """Every array of the converted ``weights.npz`` with its shape."""
        s: dict[str, tuple[int, ...]] = {
            "atomic_energies_fn.atomic_energies": (self.num_elements,) if self.num_heads == 1
            else (self.num_heads, self.num_elements),
            "node_embedding.linear.weights.0": (self.num_elements, self.C),
            "radial_embedding.bessel_fn.bessel_weights": (self.num_bessel,),
        }
        for lay in self.layers:
            p = f"interactions.{lay.index}"
            for k, sh in enumerate(lay.linear_up.weight_shapes()):
                s[f"{p}.linear_up.weights.{k}"] = sh
            if lay.nonlinear is not None:
                s.update(_nonlinear_weight_shapes(lay, p))
                self._product_readout_shapes(lay, s)
                continue
            w = lay.mlp_widths
            for j in range(len(w) - 1):
                s[f"{p}.conv_tp_weights.layers.{2 * j}.weight"] = (w[j + 1], w[j])
            if lay.density:
                s[f"{p}.density_fn.weight"] = (1, self.num_bessel)
            for k, sh in enumerate(lay.linear.weight_shapes()):
                s[f"{p}.linear.weights.{k}"] = sh
            for k, sh in enumerate(lay.skip.weight_shapes()):
                s[f"{p}.skip_tp.tp.weights.{k}"] = sh
            self._product_readout_shapes(lay, s)
        return s

    @staticmethod
    def _product_readout_shapes(lay: LayerSpec, s: dict) -> None:
        q = f"products.{lay.index}"
        for c, out in enumerate(lay.sc.outputs):
            cp = f"{q}.symmetric_contractions.contractions.{c}"
            s[f"{cp}.weights_max"] = (lay.sc.num_elements, out.num_params[-1], lay.sc.C)
            for j, nu in enumerate(range(out.correlation - 1, 0, -1)):
                s[f"{cp}.weights.{j}"] = (lay.sc.num_elements, out.num_params[nu - 1], lay.sc.C)
        for k, sh in enumerate(lay.prod_linear.weight_shapes()):
            s[f"{q}.linear.weights.{k}"] = sh
        r = f"readouts.{lay.index}"
        if lay.readout_linear is not None:
            for k, sh in enumerate(lay.readout_linear.weight_shapes()):
                s[f"{r}.linear.weights.{k}"] = sh
        else:
            for k, sh in enumerate(lay.readout_1.weight_shapes()):
                s[f"{r}.linear_1.weights.{k}"] = sh
            for k, sh in enumerate(lay.readout_2.weight_shapes()):
                s[f"{r}.linear_2.weights.{k}"] = sh
