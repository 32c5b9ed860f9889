"""CPU oracle for the packed-quadtree MTC GEMM path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``tensorpack_b200`` imports this package;
only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` (including ``bench.py --impl reference``) may call it, and they
call it as the checker / the timed CPU reference, never as the product path.

``mtc_oracle`` is a restatement, in numpy and numba, of the reference's
algorithms for this path (MTC-RD candidate search and selection, the MTC-QT
quadtree pruning, the MTC-QT-P channel permutation, the exact dequantisation,
the per-mode arena packing and the packed block GEMM).  Each function cites the
reference file:line it follows.  It is pinned against golden vectors produced
by the reference itself (``tests/golden/make_golden.py``).
"""
