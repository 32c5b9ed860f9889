"""CPU model of the device micro-block format (tensorpack_b200/csrc/mtc_common.cuh).

The encoder mirrors the repack's plane layout (mtc_repack.cu, fill_tiles) and
the decoder mirrors the fp16 magic-number decoders (decode_half_codes): a LOP3
of a field into fp16 1024.0, then fused fp16 FMAs with the same constants.
fp16 FMA is emulated exactly (product and sum in float64, one rounding to
fp16).  Every code of every mode must come back exactly, which proves the bit
positions and constants of the format before any GPU runs it.
"""

import itertools

import numpy as np
import pytest

QR = {2: (-2, 1), 3: (-4, 3), 4: (-8, 7), 5: (-16, 15), 6: (-32, 31), 8: (-128, 127)}
PW = {2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 8: 8}
MAGIC = 0x6400


def f16(x):
    return np.float16(x)


def h_from_bits(b):
    return np.array([b], dtype=np.uint16).view(np.float16)[0]


def fma16(a, b, c):
    return f16(np.float64(a) * np.float64(b) + np.float64(c))


def lop_or(x, mask):
    """(x & mask) | 0x64006400 -> (lo fp16, hi fp16)."""
    v = (x & mask) | 0x64006400
    return h_from_bits(v & 0xFFFF), h_from_bits(v >> 16)


def fma2(pair, c1, c0):
    return fma16(pair[0], c1, c0), fma16(pair[1], c1, c0)


def encode_mb(q, m):
    """q: 4x4 ints (row r, col c).  Returns (prim words dict, sec value)."""
    wp = PW[m]
    bias = 1 << (m - 1)
    pw = [0, 0, 0, 0]
    sv = 0
    for h, j, hi in itertools.product(range(2), range(4), range(2)):
        c, r = 2 * h + (j >> 1), 2 * (j & 1) + hi
        u = int(q[r][c]) + bias
        lo, up = u & ((1 << wp) - 1), u >> wp
        if wp == 2:
            pw[0] |= lo << (8 * h + 2 * j + 16 * hi)
        elif wp == 4:
            pw[h] |= lo << (4 * (j & 1) + 8 * (j >> 1) + 16 * hi)
        else:
            pw[2 * h + (j >> 1)] |= lo << (8 * ((j & 1) + 2 * hi))
        if m in (3, 5):
            sv |= up << (4 * h + j + 8 * hi)
        if m == 6:
            sv |= up << (8 * h + 2 * j + 16 * hi)
    return pw, sv


def byte_perm_4140(s):
    return (s & 0xFF) | ((s >> 8) & 0xFF) << 16


def decode_half(m, pw, sv, h):
    """Python twin of decode_half_codes; returns codes [(lo, hi)] for j = 0..3."""
    out = []
    for j in range(4):
        if m == 2:
            v = pw[0] >> (8 * h)
            c = 1.0 / (1 << (2 * j))
            out.append(fma2(lop_or(v, 0x00030003 << (2 * j)), c, -1024.0 * c - 2.0))
        elif m == 4:
            w = pw[h]
            x = (w >> 8) if (j >> 1) else w
            c = 1.0 / 16 if (j & 1) else 1.0
            out.append(fma2(lop_or(x, 0x00F000F0 if (j & 1) else 0x000F000F), c, -1024.0 * c - 8.0))
        elif m == 8:
            w = pw[2 * h + (j >> 1)]
            x = (w >> 8) if (j & 1) else w
            out.append(fma2(lop_or(x, 0x00FF00FF), 1.0, -1152.0))
        elif m == 3:
            v = pw[0] >> (8 * h)
            v1 = byte_perm_4140(sv & 0xFFFF) >> (4 * h)
            c2, c1 = 1.0 / (1 << (2 * j)), 4.0 / (1 << j)
            inner = fma2(lop_or(v1, 0x00010001 << j), c1, -1024.0 * c1 - 4.0 - 1024.0 * c2)
            t = lop_or(v, 0x00030003 << (2 * j))
            out.append((fma16(t[0], c2, inner[0]), fma16(t[1], c2, inner[1])))
        else:  # 5, 6
            w = pw[h]
            if m == 5:
                vs = byte_perm_4140(sv & 0xFFFF) >> (4 * h)
                mask, cs = 0x00010001 << j, 16.0 / (1 << j)
            else:
                vs = sv >> (8 * h)
                mask, cs = 0x00030003 << (2 * j), 16.0 / (1 << (2 * j))
            c4 = 1.0 / 16 if (j & 1) else 1.0
            bias = 16.0 if m == 5 else 32.0
            inner = fma2(lop_or(vs, mask), cs, -1024.0 * cs - bias - 1024.0 * c4)
            x = (w >> 8) if (j >> 1) else w
            t = lop_or(x, 0x00F000F0 if (j & 1) else 0x000F000F)
            out.append((fma16(t[0], c4, inner[0]), fma16(t[1], c4, inner[1])))
    return out


def _constant_exact(v):
    return float(f16(v)) == v


@pytest.mark.parametrize("m", [2, 3, 4, 5, 6, 8])
def test_decoder_constants_are_exact_fp16(m):
    """Every constant the CUDA decoder builds with f16_bits() must be exact."""
    for j in range(4):
        consts = []
        if m == 2:
            c = 1.0 / (1 << (2 * j)); consts += [c, -1024 * c - 2]
        if m == 4:
            c = 1.0 / 16 if j & 1 else 1.0; consts += [c, -1024 * c - 8]
        if m == 3:
            c2, c1 = 1.0 / (1 << (2 * j)), 4.0 / (1 << j); consts += [c2, c1, -1024 * c1 - 4 - 1024 * c2]
        if m in (5, 6):
            c4 = 1.0 / 16 if j & 1 else 1.0
            cs = 16.0 / (1 << j) if m == 5 else 16.0 / (1 << (2 * j))
            consts += [c4, cs, -1024 * cs - (16 if m == 5 else 32) - 1024 * c4]
        for v in consts:
            assert _constant_exact(v), (m, j, v)


@pytest.mark.parametrize("m", [2, 3, 4, 5, 6, 8])
def test_every_code_decodes_exactly(m):
    lo, hi = QR[m]
    rng = np.random.default_rng(m)
    cases = [np.full((4, 4), v) for v in range(lo, hi + 1)]          # every code, everywhere
    cases += [rng.integers(lo, hi + 1, size=(4, 4)) for _ in range(200)]
    for q in cases:
        pw, sv = encode_mb(q, m)
        for h in range(2):
            for j, (a, b) in enumerate(decode_half(m, pw, sv, h)):
                c, r = 2 * h + (j >> 1), 2 * (j & 1)
                assert float(a) == q[r][c] and float(b) == q[r + 1][c], (m, h, j)


def test_fp16_weight_rounding_is_single():
    """q * s16 in fp16 (HMUL2) equals RN_fp16(q * s) when s is exact in fp16."""
    rng = np.random.default_rng(0)
    for _ in range(2000):
        s = np.float32(rng.standard_normal() * 2.0 ** rng.integers(-10, 4))
        s = np.array([s], np.float32).view(np.uint32) & 0xFFFF0000
        s = s.view(np.float32)[0]
        q = int(rng.integers(-128, 128))
        if float(f16(s)) != float(s):
            continue
        assert f16(np.float64(q) * np.float64(f16(s))) == f16(np.float32(q) * s)


def dec_row(mode):
    """Python twin of make_dec_row (table of the mode-uniform decoder)."""
    wp = 2 if mode in (2, 3) else (8 if mode == 8 else 4)
    ws = 1 if mode in (3, 5) else (2 if mode == 6 else 0)
    bias = float(1 << (mode - 1))
    rows = []
    for j in range(4):
        if wp == 2:
            pm, pos = 0x00030003 << (2 * j), 2 * j
        elif wp == 4:
            pm, pos = (0x00F000F0 if j & 1 else 0x000F000F), (4 if j & 1 else 0)
        else:
            pm, pos = 0x00FF00FF, 0
        sm, cs = 0, 0.0
        if ws == 1:
            sm, cs = 0x00010001 << j, float(1 << wp) / (1 << j)
        if ws == 2:
            sm, cs = 0x00030003 << (2 * j), float(1 << wp) / (1 << (2 * j))
        c = 1.0 / (1 << pos)
        rows.append((pm, sm, c, cs, -1024.0 * cs - bias - 1024.0 * c))
    return wp, ws, rows


def decode_half_uniform(m, pw, sv, h):
    """Python twin of decode_half_uniform (without the final scale multiply)."""
    wp, ws, rows = dec_row(m)
    words = {2: [pw[0]], 4: pw[:2], 8: pw}[wp]
    if wp == 2:
        A = B = words[0] >> (8 * h)
    elif wp == 4:
        A = B = words[h]
    else:
        A, B = words[2 * h], words[2 * h + 1]
    x = [A, A >> (8 if wp == 8 else 0), B >> (8 if wp == 4 else 0), B >> (0 if wp == 2 else 8)]
    S = 0
    if ws == 1:
        S = byte_perm_4140(sv & 0xFFFF) >> (4 * h)
    if ws == 2:
        S = sv >> (8 * h)
    out = []
    for j, (pm, sm, c, cs, K) in enumerate(rows):
        for v in (c, cs, K):
            assert _constant_exact(v), (m, j, v)
        fp = lop_or(x[j], pm)
        fs = lop_or(S, sm)
        inner = (fma16(fs[0], cs, K), fma16(fs[1], cs, K))
        out.append((fma16(fp[0], c, inner[0]), fma16(fp[1], c, inner[1])))
    return out


@pytest.mark.parametrize("m", [2, 3, 4, 5, 6, 8])
def test_uniform_decoder_is_exact(m):
    lo, hi = QR[m]
    rng = np.random.default_rng(100 + m)
    cases = [np.full((4, 4), v) for v in range(lo, hi + 1)]
    cases += [rng.integers(lo, hi + 1, size=(4, 4)) for _ in range(200)]
    for q in cases:
        pw, sv = encode_mb(q, m)
        for h in range(2):
            for j, (a, b) in enumerate(decode_half_uniform(m, pw, sv, h)):
                c, r = 2 * h + (j >> 1), 2 * (j & 1)
                assert float(a) == q[r][c] and float(b) == q[r + 1][c], (m, h, j)
