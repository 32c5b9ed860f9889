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


def emulated_product_torch(mat, stored, X, exp2):
    """The same emulation with torch on X's device, for full-size layers.

    ``stored`` is the oracle dequant in stored (permuted) order, ``X`` an
    (M, K) float32 tensor; leaves are aligned to their edge, so each edge's
    scales fill a block view of the matrix.  Returns the (M, N) float64
    product in original column order."""
    import torch

    dev = X.device
    K, N = mat.shape
    ls = mat.leaf_set
    S = torch.zeros(K, N, dtype=torch.float32, device=dev)
    Md = torch.zeros(K, N, dtype=torch.int16, device=dev)
    for s in np.unique(ls.size):
        s = int(s)
        sel = ls.size == s
        bi = torch.from_numpy((ls.row[sel] // s).astype(np.int64)).to(dev)
        bj = torch.from_numpy((ls.col[sel] // s).astype(np.int64)).to(dev)
        Sv = S.view(K // s, s, N // s, s).permute(0, 2, 1, 3)
        Mv = Md.view(K // s, s, N // s, s).permute(0, 2, 1, 3)
        Sv[bi, bj] = torch.from_numpy(ls.scale[sel].astype(np.float32)).to(dev)[:, None, None]
        Mv[bi, bj] = torch.from_numpy(ls.mode[sel].astype(np.int16)).to(dev)[:, None, None]
    Wst = torch.from_numpy(np.ascontiguousarray(stored, dtype=np.float32)).to(dev)
    Q = torch.where(S != 0, torch.round(Wst / torch.where(S != 0, S, torch.ones_like(S))), torch.zeros_like(S))
    Q[Md == 0] = 0
    del Wst
    Q = Q.double()
    s32 = torch.ldexp(S, torch.tensor(float(exp2), device=dev)).float()
    s16 = s32.half()
    fast = (Md != 16) & (s16.float() == s32) & torch.isfinite(s16)
    del S, Md
    pr = None if mat.row_perm is None else torch.from_numpy(np.asarray(mat.row_perm, np.int64)).to(dev)
    x16 = (X if pr is None else X[:, pr]).half().float()
    Y = torch.empty(X.shape[0], N, dtype=torch.float64, device=dev)
    for m in range(X.shape[0]):
        pf = (x16[m][:, None] * s16.float()).half().double()
        pg = (x16[m][:, None] * s32).double()
        Y[m] = torch.ldexp((Q * torch.where(fast, pf, pg)).sum(dim=0), torch.tensor(float(-exp2), device=dev))
        del pf, pg
    if mat.col_perm is None:
        return Y
    out = torch.empty_like(Y)
    out[:, torch.from_numpy(np.asarray(mat.col_perm, np.int64)).to(dev)] = Y
    return out
