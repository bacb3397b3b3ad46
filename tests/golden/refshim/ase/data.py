"""Stand-in of ``ase.data``: the covalent-radii table (test infrastructure only).

The reference's ZBL repulsion reads ``ase.data.covalent_radii`` at run time.
The values are the published table of Cordero et al., Dalton Trans. (2008)
2832-2838 (the source ASE cites), defined once in the package this repository
ships (``mace_mlx_b200.elements``) and shared here, so both sides of the
parity comparison use one table."""

import numpy as np

from mace_mlx_b200.elements import COVALENT_RADII

covalent_radii = np.asarray(COVALENT_RADII, dtype=np.float64)
