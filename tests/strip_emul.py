"""Exact emulation of the strip kernel's arithmetic (test helper).

The strip-stream decode forms, per weight, q * fp16(fp16(x) * fp16(s 2^e))
when the pre-scaled leaf scale is exact in fp16 and the mode is not P16, and
q * fp32(fp16(x) * fp32(s 2^e)) otherwise; the products are summed here in
fp64, so kernel results differ from this only by summation order.
"""

import numpy as np


def emulated_product(mat, deq_orig, X, exp2):
    """The exact products the kernel forms, summed in fp64 (original order)."""
    K, N = mat.shape
    ls = mat.leaf_set
    S = np.zeros((K, N), np.float32)
    Md = np.zeros((K, N), np.int32)
    for r, c, s, md, sc in zip(ls.row, ls.col, ls.size, ls.mode, ls.scale):
        S[r:r + s, c:c + s] = sc
        Md[r:r + s, c:c + s] = md
    pr = np.arange(K) if mat.row_perm is None else np.asarray(mat.row_perm)
    pc = np.arange(N) if mat.col_perm is None else np.asarray(mat.col_perm)
    Wst = np.asarray(deq_orig, np.float32)[pr][:, pc]  # stored-order dequant (q * s in fp32)
    Q = np.where(S != 0, np.rint(Wst / np.where(S != 0, S, 1)), 0).astype(np.float64)
    Q[Md == 0] = 0
    s32 = np.ldexp(S, exp2).astype(np.float32)
    s16 = s32.astype(np.float16)
    fast = (Md != 16) & (s16.astype(np.float32) == s32) & np.isfinite(s16)
    x16 = X[:, pr].astype(np.float16).astype(np.float32)
    Y = np.zeros((X.shape[0], N))
    for m in range(X.shape[0]):
        pf = (x16[m][:, None] * s16.astype(np.float32)).astype(np.float16).astype(np.float64)
        pg = (x16[m][:, None] * s32).astype(np.float32).astype(np.float64)
        Y[m] = np.ldexp((Q * np.where(fast, pf, pg)).sum(axis=0), -exp2)
    out = np.empty_like(Y)
    out[:, pc] = Y
    return out, fast
