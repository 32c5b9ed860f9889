"""install_mtc_alias() makes the reference's import paths resolve to this
package (no GPU needed to import; the GPU test bodies are in
tests/test_gpu_reference_callers.py)."""

import sys


def test_reference_import_paths_resolve_here():
    import tensorpack_b200

    saved = {k: v for k, v in sys.modules.items() if k == "mtc" or k.startswith("mtc.")}
    try:
        tensorpack_b200.install_mtc_alias()
        import mtc.core.permutation as P
        import mtc.kernels.gemm as G
        import mtc.nn.layers as L
        from mtc.core.quadtree import QuadtreeRD, qt_allocate, qt_dequant  # noqa: F401
        from mtc.core.permutation import PermutedQuadtreeRD, index_bits, permuted_qt_dequant, unpermute  # noqa
        from mtc.kernels.gemm import MTCMatrix, mtc_gemm  # noqa: F401
        from mtc.nn.layers import LinearFP32, LinearMTCAdaptive  # noqa: F401

        assert G.__name__ == "tensorpack_b200.kernels.gemm"
        assert L.__name__ == "tensorpack_b200.nn.layers"
        assert P.__name__ == "tensorpack_b200.quant"
        assert index_bits(256, 512, True, True) == 256 * 8 + 512 * 9
    finally:
        for k in [k for k in sys.modules if k == "mtc" or k.startswith("mtc.")]:
            del sys.modules[k]
        sys.modules.update(saved)
