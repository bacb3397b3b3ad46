"""Per-element constants used by the distance transform and pair repulsion.

``COVALENT_RADII[Z]`` (Angstrom) is the covalent-radius table of B. Cordero et
al., "Covalent radii revisited", Dalton Trans. (2008) 2832-2838: single-bond
radii, sp3 carbon, low-spin Mn/Fe/Co.  Index 0 and the elements the paper does
not cover (Z >= 97) hold the placeholder 0.2.  This is the table that ASE
ships as ``ase.data.covalent_radii``, which the reference reads at run time for
its ZBL repulsion (``radial.py:127-199``) and its converter writes into
``config.json`` as ``distance_transform.covalent_radii`` for the Agnesi
transform (``converter.py:274-282``).  A converted model's own list is always
preferred; this table is the fallback when a config does not carry one.
"""

from __future__ import annotations

_MISSING = 0.2

COVALENT_RADII: tuple[float, ...] = (
    _MISSING,
    0.31, 0.28,                                                  # H He
    1.28, 0.96, 0.84, 0.76, 0.71, 0.66, 0.57, 0.58,              # Li-Ne
    1.66, 1.41, 1.21, 1.11, 1.07, 1.05, 1.02, 1.06,              # Na-Ar
    2.03, 1.76, 1.70, 1.60, 1.53, 1.39, 1.39, 1.32, 1.26,        # K-Co
    1.24, 1.32, 1.22, 1.22, 1.20, 1.19, 1.20, 1.20, 1.16,        # Ni-Kr
    2.20, 1.95, 1.90, 1.75, 1.64, 1.54, 1.47, 1.46, 1.42,        # Rb-Rh
    1.39, 1.45, 1.44, 1.42, 1.39, 1.39, 1.38, 1.39, 1.40,        # Pd-Xe
    2.44, 2.15, 2.07, 2.04, 2.03, 2.01, 1.99, 1.98, 1.98,        # Cs-Eu
    1.96, 1.94, 1.92, 1.92, 1.89, 1.90, 1.87, 1.87,              # Gd-Lu
    1.75, 1.70, 1.62, 1.51, 1.44, 1.41, 1.36, 1.36, 1.32,        # Hf-Hg
    1.45, 1.46, 1.48, 1.40, 1.50, 1.50,                          # Tl-Rn
    2.60, 2.21, 2.15, 2.06, 2.00, 1.96, 1.90, 1.87, 1.80, 1.69,  # Fr-Cm
) + (_MISSING,) * 22                                             # Bk-Og

assert len(COVALENT_RADII) == 119

# Agnesi transform defaults (reference radial.py:212-218)
AGNESI_DEFAULTS = {"q": 0.9183, "p": 4.5791, "a": 1.0805}
# ZBL defaults (reference radial.py:137-142)
ZBL_DEFAULTS = {"p": 6, "a_exp": 0.300, "a_prefactor": 0.4543}
