"""CPU check of the packed weight-stream format and of the integer recipes the
fused matmul kernels use to decode it (quipsharp_b200/csrc/qs_pack.cu,
qs_gemv.cu, qs_gemm_tc.cu): pack 8 codes into a 16-byte quad, then rebuild
each code's eight fp16 weights with the same shifts / XORs / byte permutes /
f16x2 adds, and compare with the oracle decode (bit-exact)."""
import numpy as np
import pytest

from oracle import quipsharp_oracle as O
from quipsharp_b200.codebooks.tables import e8p_abs_table_x2, e8_1bit_table_x2

M32 = 0xFFFFFFFF


def prmt(a, b, sel):
    src = [(a >> (8 * i)) & 0xFF for i in range(4)] + [(b >> (8 * i)) & 0xFF for i in range(4)]
    out = 0
    for i in range(4):
        nib = (sel >> (4 * i)) & 0xF
        byte = src[nib & 7]
        if nib & 8:
            byte = 0xFF if byte & 0x80 else 0
        out |= byte << (8 * i)
    return out


def hi_bytes(rows_x2):
    out = []
    for r in rows_x2:
        hb = [int(np.array(v / 2.0, dtype=np.float16).view(np.uint16)) for v in r]
        assert all(h & 0xFF == 0 for h in hb)
        hb = [h >> 8 for h in hb]
        out.append((hb[0] | hb[1] << 8 | hb[2] << 16 | hb[3] << 24,
                    hb[4] | hb[5] << 8 | hb[6] << 16 | hb[7] << 24))
    return out


E8P_HB = hi_bytes(e8p_abs_table_x2())
ONEBIT_HB = hi_bytes(e8_1bit_table_x2())


# Byte order of the coordinates in the two sign bit-slices of a quad: after the
# prefix-parity XOR and a shift by the code's slot, byte sign bits 1 and 3 hold the
# flips of one natural coordinate pair and bytes 0 and 2 those of the next one.
ORDER_A = (2, 0, 3, 1)
ORDER_B = (6, 4, 7, 5)


def pack_e8p_quad(codes):
    """Mirror of pack_e8p_kernel for one row's 8 codes."""
    w0 = w1 = w2 = w3 = 0
    for c, code in enumerate(int(x) & 0xFFFF for x in codes):
        idx = code >> 8
        if c < 4:
            w0 |= idx << (8 * c)
        else:
            w1 |= idx << (8 * (c - 4))
        f = [(code >> (7 - i)) & 1 for i in range(7)]
        f.append(f[0] ^ f[1] ^ f[2] ^ f[3] ^ f[4] ^ f[5] ^ f[6])  # even number of flips
        par = 0
        for j, coord in enumerate(ORDER_A):
            par ^= f[coord]
            w2 |= par << (8 * j + 7 - c)
        for j, coord in enumerate(ORDER_B[:3]):
            par ^= f[coord]
            w3 |= par << (8 * j + 7 - c)
        assert par ^ f[ORDER_B[3]] == 0
        w3 |= ((code & 1) ^ 1) << (31 - c)
    return w0, w1, w2, w3


def f16x2(word):
    return np.array([word & 0xFFFF, word >> 16], dtype=np.uint16).view(np.float16)


def flips(q):
    """FA / FB of the kernels: byte sign bits of coordinates (2, 0, 3, 1) / (6, 4, 7, 5)
    of every code of the quad (code c at bit 7 - c of each byte)."""
    _, _, w2, w3 = q
    fa = (w2 ^ (w2 << 8)) & M32
    fb = ((w3 & 0x00FFFFFF) ^ (((w3 << 8) | (w2 >> 24)) & M32)) & M32
    return fa, fb


def pair_words(hb):
    """f16x2 words of the natural coordinate pairs (0,1), (2,3), (4,5), (6,7)."""
    lo, hi = hb
    b = [(lo >> (8 * i)) & 0xFF for i in range(4)] + [(hi >> (8 * i)) & 0xFF for i in range(4)]
    return [(b[2 * p] << 8) | (b[2 * p + 1] << 24) for p in range(4)]


def shift_words_tmem(w3):
    """Mirror of the decode matmul's shift words: sw[p] holds the +-1/4 of codes
    (2p, 2p+1) in its (low, high) halves."""
    u = prmt(w3, (w3 << 1) & M32, 0x7030)
    return [0x34003400 ^ (((u << (2 * p)) & M32) & 0x80008000) for p in range(4)]


def decode_quad_like_gemv(q):
    """Mirror of the decode matmul (qs_gemv.cu e8p_words / shift_words): sign*|t|
    words of the natural pairs (one AND-XOR each) plus the +-1/4 shift words the
    tensor core adds against per-code activation sums."""
    w0, w1, _, w3 = q
    fa, fb = flips(q)
    shift = np.zeros(8, np.float32)
    for p, w in enumerate(shift_words_tmem(w3)):
        shift[2 * p], shift[2 * p + 1] = f16x2(w)
    out = []
    for c in range(8):
        idxsrc = w0 if c < 4 else w1
        idx = prmt(idxsrc, 0, 0x4440 | (c & 3))
        assert idx == (idxsrc >> (8 * (c & 3))) & 0xFF
        t01, t23, t45, t67 = pair_words(E8P_HB[idx])
        words = [t01 ^ (((fa << c) & M32) & 0x80008000), t23 ^ (((fa << (c + 8)) & M32) & 0x80008000),
                 t45 ^ (((fb << c) & M32) & 0x80008000), t67 ^ (((fb << (c + 8)) & M32) & 0x80008000)]
        vals = np.concatenate([f16x2(w) for w in words]).astype(np.float32)
        out.append(vals + shift[c])
    return np.stack(out)


def decode_quad_like_gemm(q):
    """Mirror of the prefill GEMM's decode (qs_gemm_tc.cu decode_e8p_row): table
    high bytes permuted to the bit-slice order, one AND-XOR per four coordinates,
    byte permutes to natural f16x2 pairs, shift added with an f16x2 add."""
    w0, w1, _, w3 = q
    fa, fb = flips(q)
    out = []
    for c in range(8):
        idxsrc = w0 if c < 4 else w1
        idx = (idxsrc >> (8 * (c & 3))) & 0xFF
        lo, hi = E8P_HB[idx]
        tl = prmt(lo, 0, 0x1302) ^ (((fa << c) & M32) & 0x80808080)
        th = prmt(hi, 0, 0x1302) ^ (((fb << c) & M32) & 0x80808080)
        sw = 0x34003400 ^ (prmt((w3 << c) & M32, 0, 0xB4B4) & 0x80008000)
        words = [prmt(tl, 0, 0x3414), prmt(tl, 0, 0x2404), prmt(th, 0, 0x3414), prmt(th, 0, 0x2404)]
        s_lo, s_hi = f16x2(sw)
        assert s_lo == s_hi
        # f16x2 add: exact, every decoded value is k/4 with |k| <= 11
        vals = np.concatenate([f16x2(w) + f16x2(sw) for w in words]).astype(np.float32)
        out.append(vals)
    return np.stack(out)


@pytest.mark.parametrize("decode", [decode_quad_like_gemv, decode_quad_like_gemm])
def test_e8p_packed_decode_matches_oracle(decode):
    rng = np.random.default_rng(0)
    edge = np.array([0, 1, 0xFF, 0x100, 0x7FFF, 0x8000, 0xFFFE, 0xFFFF])
    for trial in range(300):
        codes = edge if trial == 0 else rng.integers(0, 65536, 8)
        got = decode(pack_e8p_quad(codes))
        assert np.array_equal(got, O.e8p_decode(codes)), codes


@pytest.mark.parametrize("decode", [decode_quad_like_gemv, decode_quad_like_gemm])
def test_e8p_packed_decode_all_sign_patterns(decode):
    # every (sign7, shift) combination for a spread of table rows
    for idx in (0, 1, 100, 226, 227, 255):
        low = np.arange(256)
        codes = (idx << 8) | low
        for q in range(32):
            blk = codes[8 * q: 8 * q + 8]
            assert np.array_equal(decode(pack_e8p_quad(blk)), O.e8p_decode(blk))


def test_onebit_packed_decode_matches_oracle():
    for idx in range(256):
        words = pair_words(ONEBIT_HB[idx])
        got = np.concatenate([f16x2(w) for w in words]).astype(np.float32)
        assert np.array_equal(got, O.e8_1bit_decode(np.array([idx]))[0])
        lo, hi = ONEBIT_HB[idx]
        words = [prmt(lo, 0, 0x1404), prmt(lo, 0, 0x3424), prmt(hi, 0, 0x1404), prmt(hi, 0, 0x3424)]
        got = np.concatenate([f16x2(w) for w in words]).astype(np.float32)
        assert np.array_equal(got, O.e8_1bit_decode(np.array([idx]))[0])
