"""B200-native MACE energy + forces + stress step.

Drop-in for the compute path of mace-mlx: the ASE calculator API
(``MACECalculator``, ``mace_mp``, ``mace_off``) over converted-model
directories (``config.json`` + ``weights.npz``), computed by hand-written
sm_100a CUDA kernels in ``libmace_b200.so`` through a C ABI
(``include/mace_b200.h``).
"""

from .atoms import Atoms
from .irreps import Irrep, Irreps
from .spec import ModelSpec, UnsupportedModel
from .weights import load_model_dir, write_random_model

__all__ = [
    "Atoms", "Irrep", "Irreps", "ModelSpec", "UnsupportedModel", "load_model_dir", "write_random_model",
    "MACECalculator", "MACEMLXCalculator", "mace_mp", "mace_off", "MACEModel",
]


def __getattr__(name):  # torch-dependent pieces load lazily
    if name in ("MACECalculator", "MACEMLXCalculator", "mace_mp", "mace_off", "mace_anicc", "mace_omol"):
        from . import calculators

        return getattr(calculators, name)
    if name == "MACEModel":
        from .model import MACEModel

        return MACEModel
    raise AttributeError(name)
