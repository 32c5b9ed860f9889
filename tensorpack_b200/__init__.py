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
    """Make the reference's import paths resolve to this package, for
    unmodified callers: ``mtc.kernels.gemm`` (MTCMatrix, mtc_gemm),
    ``mtc.nn.layers`` (LinearMTCAdaptive, LinearFP32), ``mtc.core.types``,
    ``mtc.core.arena``, and ``mtc.core.quadtree`` / ``mtc.core.permutation``
    (QuadtreeRD, PermutedQuadtreeRD, qt_dequant, permuted_qt_dequant,
    unpermute, index_bits: the GPU allocators and exact reconstructions).
    Returns the ``mtc`` package object."""
    import types

    from . import quant
    from .core import arena, types as types_mod
    from .kernels import gemm
    from .nn import layers

    def package(name, **children):
        mod = types.ModuleType(name)
        mod.__path__ = []
        for k, v in children.items():
            setattr(mod, k, v)
        return mod

    core = package("mtc.core", types=types_mod, arena=arena, quadtree=quant, permutation=quant)
    kernels = package("mtc.kernels", gemm=gemm)
    nn = package("mtc.nn", layers=layers)
    pkg = package("mtc", core=core, kernels=kernels, nn=nn, PrecisionMode=PrecisionMode, MemoryArena=MemoryArena)
    mods = {"mtc": pkg, "mtc.core": core, "mtc.core.types": types_mod, "mtc.core.arena": arena,
            "mtc.core.quadtree": quant, "mtc.core.permutation": quant,
            "mtc.kernels": kernels, "mtc.kernels.gemm": gemm, "mtc.nn": nn, "mtc.nn.layers": layers}
    for name, mod in mods.items():
        sys.modules[name] = mod
    return pkg
