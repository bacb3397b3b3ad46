"""Pack a converted model (spec + weights.npz arrays) into the flat tables of
``mace_model_desc`` (``include/mace_b200.h``).

Conversions done here, once per model:
* path weights (and the constant CG diagonal of the skip product) are folded
  into the weight matrices;
* every node-feature table uses a channel-last layout per irrep slot
  (``off[s] + m*C + u``) instead of the reference's irreps-major ``u*(2l+1)+m``;
* both a matrix and its transpose are stored where the backward needs one;
* the symmetric-contraction tensors ``U`` become per-output lists of non-zeros,
  segmented by the output component ``M``.
"""

from __future__ import annotations

import math

import numpy as np

from . import native as nv
from .cg import sh_coupling
from .spec import LayerSpec, ModelSpec, UnsupportedModel

U_EPS = 1e-12  # |U| below this is rounding noise of the coupling recursion


class _Tables:
    def __init__(self):
        self.f: list[np.ndarray] = []
        self.nf = 0
        self.i: list[np.ndarray] = []
        self.ni = 0

    def addf(self, a, align: int = 4) -> int:
        a = np.ascontiguousarray(np.asarray(a, dtype=np.float32).ravel())
        lead = (-self.nf) % align
        if lead:
            self.f.append(np.zeros(lead, np.float32))
            self.nf += lead
        off = self.nf
        # keep every table 16-byte aligned for vector loads
        pad = (-a.size) % 4
        self.f.append(a)
        if pad:
            self.f.append(np.zeros(pad, np.float32))
        self.nf += a.size + pad
        return off

    def addi(self, a) -> int:
        a = np.ascontiguousarray(np.asarray(a, dtype=np.int32).ravel())
        off = self.ni
        self.i.append(a)
        self.ni += a.size
        return off

    def arrays(self):
        f = np.concatenate(self.f) if self.f else np.zeros(1, np.float32)
        i = np.concatenate(self.i) if self.i else np.zeros(1, np.int32)
        return f, i


def _slots(irreps, C: int) -> nv.Slots:
    s = nv.Slots()
    if len(irreps) > nv.MAX_IN:
        raise UnsupportedModel("too many irrep slots in a node-feature table")
    s.n = len(irreps)
    o = 0
    for q, m in enumerate(irreps):
        if m.mul != C:
            raise UnsupportedModel("all irrep slots must have the model's channel count")
        s.l[q] = m.ir.l
        s.off[q] = o
        o += C * m.ir.dim
    s.dim = o
    return s


def tf32_split(a: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """fp32 -> (hi, lo): hi rounded to tf32 (nearest, ties away), lo = a - hi."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    hi = (((u + 0x1000) & 0xFFFFE000) & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    return hi, (a - hi).astype(np.float32)


def sw128_image(m: np.ndarray) -> np.ndarray:
    """(rows, K) fp32 matrix in the 128B-swizzled K-major tensor-core layout.

    K is split into 32-wide column panels (rows x 128 bytes each, rows
    contiguous); the 16-byte chunk j of row r sits at chunk j ^ (r % 8).
    Returns a flat float32 array of rows*K values.
    """
    rows, K = m.shape
    assert K % 32 == 0 and rows % 8 == 0
    r = np.arange(rows)[:, None]
    k = np.arange(K)[None, :]
    off = (k // 32) * rows * 32 + r * 32 + (((k % 32) // 4) ^ (r % 8)) * 4 + (k % 4)
    out = np.zeros(rows * K, np.float32)
    out[off.ravel()] = m.ravel()
    return out


def _hilo_image(m: np.ndarray) -> np.ndarray:
    hi, lo = tf32_split(m)
    return np.concatenate([sw128_image(hi), sw128_image(lo)])


def mlp_tc_trunk_images(hidden_out_in: list[np.ndarray]) -> tuple[np.ndarray, np.ndarray]:
    """Images of the 64 x 64 hidden layers 1.. for the tcgen05 kernels.

    Forward operand B[o][i] is the (out, in) matrix; backward operand B[i][o]
    is its transpose.  Each as tf32 hi then lo, 128B-swizzled K-major.
    """
    if not hidden_out_in:
        return np.zeros(4, np.float32), np.zeros(4, np.float32)
    fwd = np.concatenate([_hilo_image(np.asarray(w, np.float32)) for w in hidden_out_in])
    bwd = np.concatenate([_hilo_image(np.ascontiguousarray(np.asarray(w, np.float32).T)) for w in hidden_out_in])
    return fwd, bwd


def mlp_tc_images(w_last_out_in: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Operand images of the last radial-MLP layer for the tcgen05 kernels.

    ``w_last_out_in`` is the converted (out, in) weight with in = 64.  Forward:
    per 64-output chunk the (64 x 64) slice (zero rows past the last output),
    tf32 hi then lo.  Backward: per 32-output chunk the (64 x 32) slice of the
    transpose, hi then lo.
    """
    W = np.asarray(w_last_out_in, dtype=np.float32)
    n_out, n_in = W.shape
    pad_f = -(-n_out // 64) * 64
    Wf = np.zeros((pad_f, n_in), np.float32)
    Wf[:n_out] = W
    fwd = np.concatenate([_hilo_image(Wf[c:c + 64]) for c in range(0, pad_f, 64)])
    pad_b = -(-n_out // 32) * 32
    Wb = np.zeros((n_in, pad_b), np.float32)
    Wb[:, :n_out] = W.T
    hi, lo = tf32_split(Wb)
    bwd = np.concatenate([np.concatenate([sw128_image(hi[:, c:c + 32]), sw128_image(lo[:, c:c + 32])])
                          for c in range(0, pad_b, 32)])
    return fwd, bwd


def sc_polynomial(Us: list[np.ndarray], Ws: list[np.ndarray], L: int):
    """Rewrite one output of the symmetric contraction as a polynomial in f.

    The reference evaluates  out[M] = sum_nu sum U_nu[M, a_1..a_nu, k] W_nu[z, k, c] prod_q f[a_q]
    (symmetric_contraction.py:95-121, 505-595).  The product of the f's is
    symmetric in the a's, so U_nu is summed over index permutations onto
    sorted tuples a_1 <= ... <= a_nu, and contracted with the (constant) species
    weights once: G[z, e, c] = sum_k U_sym[e, k] W_nu[z, k, c].  Returns
    (entries (n, 5): M, a, b, c, nu), G (num_elements, n, C) float64).
    Us[nu-1] has shape ([2L+1,] d^nu, K_nu); Ws[nu-1] has shape (num_el, K_nu, C).
    """
    ents, Gs = [], []
    for nu, (U, W) in enumerate(zip(Us, Ws), start=1):
        if L == 0:
            U = U[None]
        if U.shape[1] > 16:
            raise UnsupportedModel("symmetric-contraction coupling dimension above 16")
        nz = np.argwhere(np.abs(U) > U_EPS)
        vals = U[tuple(nz.T)]
        keys = np.concatenate([nz[:, :1], np.sort(nz[:, 1:1 + nu], axis=1)], axis=1)
        uniq, inv = np.unique(keys, axis=0, return_inverse=True)
        inv = inv.reshape(-1)
        Usym = np.zeros((len(uniq), U.shape[-1]))
        np.add.at(Usym, (inv, nz[:, -1]), vals)
        G = np.einsum("ek,zkc->zec", Usym, W.astype(np.float64))
        e = np.zeros((len(uniq), 5), dtype=np.int64)
        e[:, 0] = uniq[:, 0]
        e[:, 1:1 + nu] = uniq[:, 1:]
        e[:, 4] = nu
        ents.append(e)
        Gs.append(G)
    ent = np.concatenate(ents)
    G = np.concatenate(Gs, axis=1)
    order = np.lexsort((ent[:, 3], ent[:, 2], ent[:, 1], ent[:, 4], ent[:, 0]))
    return ent[order], G[:, order]


def _sc_tables(Us, Ws, L: int, tb: _Tables) -> tuple[int, int, int]:
    ent, G = sc_polynomial(Us, Ws, L)
    dM = 2 * L + 1
    seg = np.zeros(dM + 1, dtype=np.int64)
    for M in range(dM):
        seg[M + 1] = seg[M] + np.count_nonzero(ent[:, 0] == M)
    packed = ent[:, 0] | (ent[:, 1] << 4) | (ent[:, 2] << 8) | (ent[:, 3] << 12) | (ent[:, 4] << 16)
    i_off = tb.addi(np.concatenate([seg, packed]).astype(np.int32))
    f_off = tb.addf(G)
    return i_off, f_off, len(ent)


def sc_backward_polynomial(outs: list[tuple[np.ndarray, np.ndarray, int]], ncoup: int):
    """Gradient of the symmetric-contraction polynomials w.r.t. the coupling features.

    ``outs`` holds, per product output slot, (entries, G, row0) from
    ``sc_polynomial`` and the slot's first row (offset / C) in the product
    output.  For out[r][c] = sum_e G[z,e,c] prod_q f[a_q], the derivative is
      df[k][c] = sum_r g[r][c] sum_{e of r, k in e} mult_k(e) G[z,e,c] prod_{q != one k} f[a_q],
    returned as entries (k, b, c, nu', r) sorted by k (nu' = degree - 1, b <= c
    the remaining indices) and G' = mult_k x G, shape (num_elements, n, C).
    """
    rows, Gs = [], []
    for ent, G, row0 in outs:
        for e in range(len(ent)):
            M, nu = int(ent[e, 0]), int(ent[e, 4])
            idx = [int(v) for v in ent[e, 1:1 + nu]]
            for k in sorted(set(idx)):
                rem = list(idx)
                rem.remove(k)
                rem += [0] * (2 - len(rem))
                rows.append((k, rem[0], rem[1], nu - 1, row0 + M))
                Gs.append(idx.count(k) * G[:, e, :])
    ent_b = np.array(rows, dtype=np.int64).reshape(-1, 5)
    G_b = np.stack(Gs, axis=1) if Gs else np.zeros((0, 0, 0))
    order = np.lexsort((ent_b[:, 2], ent_b[:, 1], ent_b[:, 3], ent_b[:, 4], ent_b[:, 0]))
    ent_b, G_b = ent_b[order], G_b[:, order]
    seg = np.zeros(ncoup + 1, dtype=np.int64)
    for k in range(ncoup):
        seg[k + 1] = seg[k] + np.count_nonzero(ent_b[:, 0] == k)
    return ent_b, G_b, seg


def _sc_generated_signature(lay: LayerSpec, spec: ModelSpec, ents: list[np.ndarray]) -> int:
    """Id of the generated SC kernels (sc_gen.cu) serving this layer, or 0."""
    from . import sc_codegen as gen

    if lay.sc.coupling != gen.COUPLING or spec.interaction_irreps.dim != 16 * spec.C:
        return 0
    names = tuple(str(out.ir_out) for out in lay.sc.outputs)
    if names not in gen.SIGNATURES or any(out.correlation != gen.CORRELATION for out in lay.sc.outputs):
        return 0
    for name, ent in zip(names, ents):
        ref = gen.standard_entries(name)
        if ref.shape != ent.shape or not np.array_equal(ref, ent):
            return 0
    return gen.SIGNATURES.index(names) + 1


def _layer(spec: ModelSpec, lay: LayerSpec, w: dict, tb: _Tables) -> nv.LayerDesc:
    C = spec.C
    t = lay.index
    d = nv.LayerDesc()
    d.C = C
    d.residual = int(lay.residual)
    d.in_ = _slots(lay.irreps_in, C)
    d.hid = _slots(lay.hidden, C)
    d.inter = _slots(spec.interaction_irreps, C)
    if lay.hidden[0].ir.l != 0:
        raise UnsupportedModel("hidden irreps must start with the scalar block")
    # skip_tp
    sk = lay.skip
    d.n_skip = len(sk.instrs)
    for q, ins in enumerate(sk.instrs):
        W = w[f"interactions.{t}.skip_tp.tp.weights.{q}"].astype(np.float64) * (ins.path_weight * ins.cg)
        d.skip_in[q] = ins.i_in1
        d.skip_out[q] = ins.i_out
        d.f_skip[q] = tb.addf(W.transpose(1, 0, 2))  # (z, u, w)
        d.f_skip_t[q] = tb.addf(W.transpose(1, 2, 0))  # (z, w, u)
    # linear_up (1-to-1)
    for q, ins in enumerate(lay.linear_up.instrs):
        if ins.i_in != q or ins.i_out != q:
            raise UnsupportedModel("linear_up must map each slot to itself")
        W = w[f"interactions.{t}.linear_up.weights.{q}"].astype(np.float64) * ins.path_weight
        d.f_up[q] = tb.addf(W)
        d.f_up_t[q] = tb.addf(W.T)
    # radial MLP
    widths = lay.mlp_widths
    d.n_mlp = len(widths) - 1
    if d.n_mlp > 7:
        raise UnsupportedModel("radial MLP too deep")
    for j, wd in enumerate(widths):
        d.mlp_w[j] = wd
    for j in range(d.n_mlp):
        Wm = w[f"interactions.{t}.conv_tp_weights.layers.{2 * j}.weight"].astype(np.float64)  # (out, in)
        d.f_mlp[j] = tb.addf(Wm.T)
        d.f_mlp_t[j] = tb.addf(Wm)
    d.f_mlp_tc = d.f_mlp_tc_bwd = d.f_mlp_tc_trunk = d.f_mlp_tc_trunk_bwd = -1
    if all(wd == 64 for wd in widths[1:-1]) and widths[0] <= 16:
        last = w[f"interactions.{t}.conv_tp_weights.layers.{2 * (d.n_mlp - 1)}.weight"]
        fwd_img, bwd_img = mlp_tc_images(last)
        d.f_mlp_tc = tb.addf(fwd_img, align=32)
        d.f_mlp_tc_bwd = tb.addf(bwd_img, align=32)
        hidden = [w[f"interactions.{t}.conv_tp_weights.layers.{2 * j}.weight"] for j in range(1, d.n_mlp - 1)]
        tf, tbw = mlp_tc_trunk_images(hidden)
        d.f_mlp_tc_trunk = tb.addf(tf, align=32)
        d.f_mlp_tc_trunk_bwd = tb.addf(tbw, align=32)
    # conv_tp slots
    cv = lay.conv
    if len(cv.instrs) > nv.MAX_MID:
        raise UnsupportedModel("too many conv_tp output slots")
    d.n_mid = len(cv.instrs)
    off = m_off = 0
    for k, ins in enumerate(cv.instrs):
        cs = d.conv[k]
        cs.l1, cs.l2, cs.l3, cs.src = ins.l1, ins.l2, ins.l3, ins.i_in1
        cs.off = off
        cs.m_off = m_off
        cs.f_cg = tb.addf(ins.cg)
        off += C * (2 * ins.l3 + 1)
        m_off += (2 * ins.l1 + 1) * (2 * ins.l3 + 1)
    d.m_tot = m_off
    d.wnumel = cv.weight_numel
    d.mid.n = 0
    d.mid.dim = off
    # interaction linear: one concat-K group per output slot
    groups: dict[int, list] = {}
    for q, ins in enumerate(lay.linear.instrs):
        groups.setdefault(ins.i_out, []).append((ins.i_in, w[f"interactions.{t}.linear.weights.{q}"], ins.path_weight))
    for io in range(len(spec.interaction_irreps)):
        g = groups.get(io, [])
        if len(g) > nv.MAX_SRC or not g:
            raise UnsupportedModel("interaction linear group size out of range")
        lg = d.lin[io]
        lg.n_src = len(g)
        mats = []
        for q, (src, W, pw) in enumerate(g):
            lg.src[q] = src
            mats.append(W.astype(np.float64) * pw)
        Wc = np.concatenate(mats, axis=0)
        lg.f_w = tb.addf(Wc)
        lg.f_wt = tb.addf(Wc.T)
    # symmetric contraction
    sc_outs = []
    for o, out in enumerate(lay.sc.outputs):
        so = d.sc[o]
        so.L = out.ir_out.l
        so.corr = out.correlation
        if out.correlation > nv.MAX_CORR:
            raise UnsupportedModel("correlation order above 3 is not supported")
        pre = f"products.{t}.symmetric_contractions.contractions.{o}"
        Ws = []
        for nu in range(1, out.correlation + 1):
            if nu == out.correlation:
                Ws.append(w[f"{pre}.weights_max"])
            else:
                Ws.append(w[f"{pre}.weights.{out.correlation - 1 - nu}"])
        if lay.sc.num_elements == 1 and spec.num_elements > 1:
            # species-agnostic product (one weight set, blocks.py:527-531): every
            # element's row holds it, so the species-indexed kernels apply it to all nodes
            Ws = [np.repeat(np.asarray(W), spec.num_elements, axis=0) for W in Ws]
        so.i_ent, so.f_G, so.n_ent = _sc_tables(out.U, Ws, so.L, tb)
        ent, G = sc_polynomial(out.U, Ws, so.L)
        sc_outs.append((ent, G, d.hid.off[o] // C))
    ncoup = spec.interaction_irreps.dim // C
    ent_b, G_b, seg_b = sc_backward_polynomial(sc_outs, ncoup)
    packed = ent_b[:, 1] | (ent_b[:, 2] << 4) | (ent_b[:, 3] << 8) | (ent_b[:, 4] << 10)
    d.sc_n_bwd = len(ent_b)
    d.i_sc_bwd = tb.addi(np.concatenate([seg_b, packed]).astype(np.int32))
    d.f_sc_bwd = tb.addf(G_b)
    d.sc_gen = _sc_generated_signature(lay, spec, [e for e, _, _ in sc_outs])
    # product linear (1-to-1)
    for q, ins in enumerate(lay.prod_linear.instrs):
        if ins.i_in != q or ins.i_out != q:
            raise UnsupportedModel("product linear must map each slot to itself")
        W = w[f"products.{t}.linear.weights.{q}"].astype(np.float64) * ins.path_weight
        d.f_prod[q] = tb.addf(W)
        d.f_prod_t[q] = tb.addf(W.T)
    # readout: the selected head's column.  A multi-head non-linear readout masks
    # its 16 H hidden scalars to the head's block of 16 before linear_2
    # (blocks.py:602-609), so it equals a 16-wide readout on that block's
    # linear_1 columns and linear_2 rows, keeping linear_2's 1/sqrt(16 H) path weight.
    h = spec.head_idx
    if lay.readout_linear is not None:
        (ins,) = lay.readout_linear.instrs
        if ins.i_in != 0:
            raise UnsupportedModel("linear readout must read the scalar slot")
        d.readout_nonlinear = 0
        d.f_ro1 = tb.addf(w[f"readouts.{t}.linear.weights.0"][:, h].astype(np.float64) * ins.path_weight)
    else:
        (i1,) = lay.readout_1.instrs
        (i2,) = lay.readout_2.instrs
        fph = i1.mul_out // spec.num_heads
        rows = slice(h * fph, (h + 1) * fph)
        d.readout_nonlinear = 1
        d.readout_hidden = fph
        w1 = w[f"readouts.{t}.linear_1.weights.0"][:, rows].astype(np.float64) * i1.path_weight
        d.f_ro1 = tb.addf(np.ascontiguousarray(w1))
        d.f_ro2 = tb.addf(w[f"readouts.{t}.linear_2.weights.0"][rows, h].astype(np.float64) * i2.path_weight)
    # density normalisation: density_fn = bias-free Linear(num_bessel -> 1), weight (1, num_bessel)
    d.density = int(lay.density)
    d.f_density = tb.addf(w[f"interactions.{t}.density_fn.weight"].reshape(-1)) if lay.density else -1
    return d


class PackedModel:
    """Owns the numpy tables that ``desc`` points into."""

    def __init__(self, spec: ModelSpec, weights: dict):
        if spec.max_ell > 3:
            raise UnsupportedModel("max_ell above 3 is not supported")
        if spec.num_interactions > nv.MAX_LAYERS:
            raise UnsupportedModel("too many interaction layers")
        if any(lay.nonlinear is not None for lay in spec.layers):
            raise UnsupportedModel("the mh-1 non-linear interaction block has no CUDA path")
        if not spec.apply_cutoff and any(lay.density for lay in spec.layers):
            raise UnsupportedModel("apply_cutoff=False with density-normalised blocks has no CUDA path")
        tb = _Tables()
        d = nv.ModelDesc()
        d.abi_version = nv.ABI_VERSION
        d.num_layers = spec.num_interactions
        d.num_elements = spec.num_elements
        d.num_bessel = spec.num_bessel
        d.max_ell = spec.max_ell
        d.poly_p = spec.poly_p
        d.scale_shift = int(spec.model_type == "ScaleShiftMACE")
        d.envelope_on_weights = int(not spec.apply_cutoff)
        d.C = spec.C
        d.r_max = spec.r_max
        d.inv_avg_num_neighbors = 1.0 / spec.avg_num_neighbors
        d.scale = spec.scale
        d.shift = spec.shift
        ae = weights.get("atomic_energies_fn.atomic_energies", spec.atomic_energies)
        d.f_e0 = tb.addf(spec.head_atomic_energies(ae))
        d.f_emb = tb.addf(weights["node_embedding.linear.weights.0"].astype(np.float64) / math.sqrt(spec.num_elements))
        d.f_bessel = tb.addf(weights["radial_embedding.bessel_fn.bessel_weights"])
        d.f_sh = tb.addf(np.concatenate([sh_coupling(2).ravel(), sh_coupling(3).ravel()]))
        for t, lay in enumerate(spec.layers):
            d.layers[t] = _layer(spec, lay, weights, tb)
        d.f_radius_agnesi = d.f_radius_zbl = d.f_znum = -1
        if spec.agnesi is not None or spec.zbl is not None:
            znum = spec.species_numbers()
            d.f_znum = tb.addf(np.asarray(znum, dtype=np.float64))
        if spec.agnesi is not None:
            ag = spec.agnesi
            d.agnesi = 1
            d.agnesi_q, d.agnesi_p, d.agnesi_a = ag["q"], ag["p"], ag["a"]
            d.f_radius_agnesi = tb.addf(np.asarray([ag["covalent_radii"][z] for z in znum], dtype=np.float64))
        if spec.zbl is not None:
            zb = spec.zbl
            d.zbl = 1
            d.zbl_p = zb["p"]
            d.zbl_a_exp, d.zbl_a_prefactor = zb["a_exp"], zb["a_prefactor"]
            d.f_radius_zbl = tb.addf(np.asarray([zb["covalent_radii"][z] for z in znum], dtype=np.float64))
        self.floats, self.ints = tb.arrays()
        d.floats = self.floats.ctypes.data_as(nv.C.POINTER(nv.f32))
        d.n_floats = self.floats.size
        d.ints = self.ints.ctypes.data_as(nv.C.POINTER(nv.i32))
        d.n_ints = self.ints.size
        self.desc = d
        self.spec = spec
