"""Coupling constants (host-side, fp64): real Wigner 3j, real Clebsch-Gordan, and
the symmetric-contraction coupling tensors ``U``.

These follow the conventions the reference fixes in ``mace_mlx/clebsch_gordan.py``
(which in turn follows e3nn / mace-torch), because the converted weights live in
that basis and any sign or ordering change would silently change the model:

* real spherical-harmonic basis: the complex->real unitary with the
  Condon-Shortley phase (``clebsch_gordan.py:26-45``);
* rotation generators of that basis: the y-generator ``i J_y`` taken from the
  complex ladder operators (``clebsch_gordan.py:48-64``) and the z-generator that
  differentiates the reference's z-rotation block (``clebsch_gordan.py:67-76``);
* sign convention of the 3j symbol for sorted ``l1 <= l2 <= l3``: centre element
  positive, else first non-zero element positive (``clebsch_gordan.py:229-235``);
  unsorted triples come from the sorted one by the e3nn transposition rules
  (``clebsch_gordan.py:238-272``);
* ``U_matrix_real``: the recursive n-fold coupling of ``_wigner_nj`` with a stable
  ``(l, p)`` sort per level and the paths stacked on the last axis
  (``clebsch_gordan.py:296-445``).

The invariant vector is computed differently from the reference: instead of the
null space of ``D(R) - 1`` summed over five fixed random rotations, this module
takes the null space of the Lie-algebra action ``X1 + X2 + X3`` for the two
generators above.  Both give the same (unique up to sign) unit vector, so after
the shared sign rule the tables agree to rounding (checked against the
reference's own tables in ``tests/test_cg.py``).
"""

from __future__ import annotations

import functools
import math

import numpy as np

from .irreps import Irrep, Irreps

__all__ = ["wigner_3j", "so3_clebsch_gordan", "U_matrix_real", "sh_coupling"]


@functools.lru_cache(maxsize=None)
def _complex_to_real(l: int) -> np.ndarray:
    """Unitary ``Q`` with ``Y_real = Q Y_complex`` (Condon-Shortley phase)."""
    d = 2 * l + 1
    q = np.zeros((d, d), dtype=np.complex128)
    s = 1.0 / math.sqrt(2.0)
    q[l, l] = 1.0
    for m in range(1, l + 1):
        q[l + m, l + m] = (-1) ** m * s
        q[l + m, l - m] = s
        q[l - m, l + m] = -1j * (-1) ** m * s
        q[l - m, l - m] = 1j * s
    return q


@functools.lru_cache(maxsize=None)
def _generators(l: int) -> tuple[np.ndarray, np.ndarray]:
    """Real-basis rotation generators (Xz, Xy) of degree ``l``."""
    d = 2 * l + 1
    # i*J_y in the complex |l,m> basis: (J+ - J-)/2.
    jc = np.zeros((d, d), dtype=np.float64)
    for m in range(-l, l + 1):
        if m + 1 <= l:
            jc[m + l + 1, m + l] = 0.5 * math.sqrt(l * (l + 1) - m * (m + 1))
        if m - 1 >= -l:
            jc[m + l - 1, m + l] = -0.5 * math.sqrt(l * (l + 1) - m * (m - 1))
    q = _complex_to_real(l)
    xy = (q @ jc @ q.conj().T).real
    # z-rotation by theta acts on the (i, 2l-i) pair with frequency l-i.
    xz = np.zeros((d, d), dtype=np.float64)
    for i in range(d):
        if i != l:
            xz[i, d - 1 - i] = float(l - i)
    return xz, xy


@functools.lru_cache(maxsize=None)
def _w3j_sorted(l1: int, l2: int, l3: int) -> np.ndarray:
    assert l1 <= l2 <= l3
    d1, d2, d3 = 2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1
    if l3 > l1 + l2:
        return np.zeros((d1, d2, d3))
    g1, g2, g3 = _generators(l1), _generators(l2), _generators(l3)
    i1, i2, i3 = np.eye(d1), np.eye(d2), np.eye(d3)
    blocks = []
    for a in range(2):
        blocks.append(
            np.kron(g1[a], np.kron(i2, i3))
            + np.kron(i1, np.kron(g2[a], i3))
            + np.kron(i1, np.kron(i2, g3[a]))
        )
    mat = np.concatenate(blocks, axis=0)
    _, sv, vt = np.linalg.svd(mat)
    if sv.size > 1 and sv[-2] < 1e-6:
        raise RuntimeError(f"3j null space of ({l1},{l2},{l3}) is not one-dimensional")
    q = vt[-1].reshape(d1, d2, d3).copy()
    q /= np.linalg.norm(q)
    q[np.abs(q) < 1e-14] = 0.0
    centre = q[l1, l2, l3]
    if centre != 0.0:
        if centre < 0:
            q = -q
    else:
        first = q.flat[np.flatnonzero(q)[0]]
        if first < 0:
            q = -q
    return q


@functools.lru_cache(maxsize=None)
def wigner_3j(l1: int, l2: int, l3: int) -> np.ndarray:
    """Unit-norm real 3j tensor of shape (2l1+1, 2l2+1, 2l3+1), e3nn convention."""
    if l3 < abs(l1 - l2) or l3 > l1 + l2:
        return np.zeros((2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1))
    sign = (-1) ** (l1 + l2 + l3)
    if l1 <= l2 <= l3:
        out = _w3j_sorted(l1, l2, l3)
    elif l1 <= l3 <= l2:
        out = _w3j_sorted(l1, l3, l2).transpose(0, 2, 1) * sign
    elif l2 <= l1 <= l3:
        out = _w3j_sorted(l2, l1, l3).transpose(1, 0, 2) * sign
    elif l3 <= l2 <= l1:
        out = _w3j_sorted(l3, l2, l1).transpose(2, 1, 0) * sign
    elif l2 <= l3 <= l1:
        out = _w3j_sorted(l2, l3, l1).transpose(2, 0, 1)
    else:  # l3 <= l1 <= l2
        out = _w3j_sorted(l3, l1, l2).transpose(1, 2, 0)
    out = np.ascontiguousarray(out)
    out.setflags(write=False)
    return out


def so3_clebsch_gordan(l1: int, l2: int, l3: int) -> np.ndarray:
    """Component-normalised real CG: ``wigner_3j * sqrt(2 l3 + 1)``."""
    return wigner_3j(l1, l2, l3) * math.sqrt(2 * l3 + 1)


@functools.lru_cache(maxsize=None)
def sh_coupling(l: int) -> np.ndarray:
    """Recursion tensor ``Y_l = einsum(Y_{l-1}, Y_1, T_l)`` of the component SH.

    ``T_l = CG(l-1, 1, l) * sqrt((2l+1)/(3l))`` (reference
    ``spherical_harmonics.py:31-40``); shape (2l-1, 3, 2l+1).
    """
    return so3_clebsch_gordan(l - 1, 1, l) * math.sqrt((2 * l + 1) / (3 * l))


# ---------------------------------------------------------------------------
# U tensors of the symmetric contraction
# ---------------------------------------------------------------------------


def _couple_paths(irrepss: list[Irreps], filter_mid, keep_last=None):
    """n-fold coupling paths ``(ir_out, tensor)`` sorted stably by (l, p).

    ``tensor`` has shape ``(ir_out.dim, *[irreps.dim for irreps in irrepss])``.
    ``keep_last`` (a set of irreps) drops, at the outermost level only, paths
    whose output is not wanted; the stable sort makes this equivalent to
    filtering afterwards.
    """
    if len(irrepss) == 1:
        (irr,) = irrepss
        eye = np.eye(irr.dim)
        out, i = [], 0
        for mul, ir in irr:
            for _ in range(mul):
                out.append((ir, eye[i : i + ir.dim]))
                i += ir.dim
        return out
    *left_list, right = irrepss
    left_dims = [x.dim for x in left_list]
    out = []
    for ir_left, c_left in _couple_paths(left_list, filter_mid):
        i = 0
        c_left2 = c_left.reshape(ir_left.dim, -1)
        for mul, ir in right:
            for ir_out in ir_left.couple(ir):
                if filter_mid is not None and ir_out not in filter_mid:
                    continue
                if keep_last is not None and ir_out not in keep_last:
                    continue
                w = wigner_3j(ir_out.l, ir_left.l, ir.l) * math.sqrt(ir_out.dim)
                c = np.einsum("jk,ijl->ikl", c_left2, w)
                c = c.reshape(ir_out.dim, *left_dims, ir.dim)
                for u in range(mul):
                    e = np.zeros((ir_out.dim, *left_dims, right.dim))
                    e[..., i + u * ir.dim : i + (u + 1) * ir.dim] = c
                    out.append((ir_out, e))
            i += mul * ir.dim
    out.sort(key=lambda t: (t[0].l, t[0].p))
    return out


@functools.lru_cache(maxsize=None)
def _U_cached(irreps_in: str, ir_out: Irrep, correlation: int) -> np.ndarray:
    irr = Irreps(irreps_in)
    filt = None
    if correlation == 4:
        filt = {Irrep(l, 1 if l % 2 == 0 else -1) for l in range(12)}
    paths = _couple_paths([irr] * correlation, filt, keep_last={ir_out})
    pieces = [np.squeeze(t)[..., None] for ir, t in paths if ir == ir_out]
    if not pieces:
        shape = (*([irr.dim] * correlation), 1)
        if ir_out.dim != 1:
            shape = (ir_out.dim, *shape)
        u = np.zeros(shape)
    else:
        u = np.concatenate(pieces, axis=-1)
    u.setflags(write=False)
    return u


def U_matrix_real(irreps_in, ir_out, correlation: int) -> np.ndarray:
    """Coupling tensor of one output irrep, shape ``([ir.dim,] d, ..., d, K)``.

    ``d = irreps_in.dim`` repeated ``correlation`` times; ``K`` = number of
    coupling paths.  The leading ``ir.dim`` axis is absent for scalar outputs
    (the reference squeezes it away, ``clebsch_gordan.py:421``).
    """
    return _U_cached(str(Irreps(irreps_in)), Irrep.parse(ir_out), int(correlation))
