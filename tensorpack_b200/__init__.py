"""tensorpack_b200: B200-native (sm_100a) packed-quadtree MTC GEMM.

Drop-in for the quantized-inference hot path of Sharexi/TensorPack ("MTC"):
``tensorpack_b200.kernels.gemm`` mirrors ``mtc.kernels.gemm`` (MTCMatrix,
mtc_gemm) and ``tensorpack_b200.nn.layers`` mirrors the quantized linear
layer of ``mtc.nn.layers``.  ``install_mtc_alias()`` registers these modules
under the reference's import paths for code that imports ``mtc``.
"""

import sys

from .core.arena import MemoryArena
from .core.types import PrecisionMode
from .kernels.gemm import MTCMatrix, mtc_gemm

__version__ = "0.1.0"
__all__ = ["MTCMatrix", "mtc_gemm", "MemoryArena", "PrecisionMode", "install_mtc_alias"]


def install_mtc_alias():
    """Make ``import mtc.kernels.gemm`` / ``mtc.nn.layers`` / ``mtc.core.types``
    / ``mtc.core.arena`` resolve to this package (for unmodified callers)."""
    import types

    from . import core, kernels, nn
    from .core import arena, types as ctypes_mod
    from .kernels import gemm
    from .nn import layers

    pkg = types.ModuleType("mtc")
    pkg.__path__ = []
    pkg.PrecisionMode = PrecisionMode
    pkg.MemoryArena = MemoryArena
    mods = {"mtc": pkg, "mtc.core": core, "mtc.core.types": ctypes_mod, "mtc.core.arena": arena,
            "mtc.kernels": kernels, "mtc.kernels.gemm": gemm, "mtc.nn": nn, "mtc.nn.layers": layers}
    for name, mod in mods.items():
        sys.modules[name] = mod
    pkg.core, pkg.kernels, pkg.nn = core, kernels, nn
    return pkg
