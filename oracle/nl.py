"""ORACLE (test infrastructure only; never imported by the product path).

numpy fp64 restatement of the reference's neighbour list contract: the
``"ijS"`` list of matscipy / ASE that ``mace_mlx/calculators.py:40-62`` calls
with cutoff ``r_max + skin`` (``calculators.py:295-297``).  The set is every
``(i, j, S)`` with ``|x_j - x_i + S @ cell| < r_cut`` except ``i == j, S == 0``;
``S`` is zero along non-periodic axes.  Both directions are present.  The
reference then uses ``sender = i``, ``receiver = j`` and
``v = pos[j] - pos[i] + S @ cell`` (``utils.py:47-84``).

matscipy 0.8 / ASE 3.22 (the reference's pinned dependencies) are not installed
here; this restates their published definition of the list.
"""

from __future__ import annotations

import itertools

import numpy as np


def _shift_ranges(pos, cell, pbc, r_cut):
    ranges = []
    if not np.any(pbc):
        return [range(0, 1)] * 3
    inv = np.linalg.inv(cell)
    frac = pos @ inv
    vol = abs(np.linalg.det(cell))
    for d in range(3):
        if not pbc[d]:
            ranges.append(range(0, 1))
            continue
        a, b = cell[(d + 1) % 3], cell[(d + 2) % 3]
        h = vol / np.linalg.norm(np.cross(a, b))
        n = int(np.ceil(r_cut / h))
        span = int(np.ceil(frac[:, d].max() - frac[:, d].min()))
        ranges.append(range(-n - span, n + span + 1))
    return ranges


def neighbour_list(pos, cell, pbc, r_cut, batch=None):
    """Return (sender, receiver, shifts) as int64 arrays, sorted by (i, j, S)."""
    pos = np.asarray(pos, dtype=np.float64)
    cell = np.asarray(cell, dtype=np.float64)
    pbc = np.asarray(pbc, dtype=bool)
    out_i, out_j, out_s = [], [], []
    if batch is not None:
        batch = np.asarray(batch)
        for g in np.unique(batch):
            idx = np.nonzero(batch == g)[0]
            gi, gj, gs = neighbour_list(pos[idx], cell, pbc, r_cut)
            out_i.append(idx[gi])
            out_j.append(idx[gj])
            out_s.append(gs)
        i, j, s = (np.concatenate(x) for x in (out_i, out_j, out_s))
        order = np.lexsort((s[:, 2], s[:, 1], s[:, 0], j, i))
        return i[order], j[order], s[order]
    n = len(pos)
    rc2 = r_cut * r_cut
    for S in itertools.product(*_shift_ranges(pos, cell, pbc, r_cut)):
        S = np.array(S, dtype=np.int64)
        off = S.astype(np.float64) @ cell if np.any(pbc) else np.zeros(3)
        for i0 in range(0, n, 512):
            pi = pos[i0 : i0 + 512]
            d = (pos[None, :, :] - pi[:, None, :]) + off
            d2 = np.einsum("ijc,ijc->ij", d, d)
            ii, jj = np.nonzero(d2 < rc2)
            ii = ii + i0
            keep = ~((ii == jj) & (not np.any(S)))
            out_i.append(ii[keep])
            out_j.append(jj[keep])
            out_s.append(np.repeat(S[None], keep.sum(), axis=0))
    i = np.concatenate(out_i) if out_i else np.zeros(0, np.int64)
    j = np.concatenate(out_j) if out_j else np.zeros(0, np.int64)
    s = np.concatenate(out_s) if out_s else np.zeros((0, 3), np.int64)
    order = np.lexsort((s[:, 2], s[:, 1], s[:, 0], j, i))
    return i[order], j[order], s[order]


def min_gap_to_cutoff(pos, cell, sender, receiver, shifts, r_cut) -> float:
    """Smallest | |v| - r_cut | over the listed edges (tie diagnostics)."""
    if len(sender) == 0:
        return np.inf
    v = pos[receiver] - pos[sender] + shifts.astype(np.float64) @ np.asarray(cell, dtype=np.float64)
    return float(np.min(np.abs(np.linalg.norm(v, axis=1) - r_cut)))
