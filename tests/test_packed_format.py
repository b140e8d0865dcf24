"""CPU check of the packed weight-stream format and of the integer recipe the
fused matmul kernel uses to decode it (quipsharp_b200/csrc/qs_pack.cu,
qs_gemv.cu): pack 8 codes into a 16-byte quad, then rebuild each code's eight
fp16 weights with the same shifts / XORs / byte permutes / f16x2 add, and
compare with the oracle decode (bit-exact)."""
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


def pack_e8p_quad(codes):
    """Mirror of pack_e8p_kernel for one row's 8 codes."""
    w0 = w1 = w2 = w3 = 0
    for c, code in enumerate(int(x) & 0xFFFF for x in codes):
        idx = code >> 8
        if c < 4:
            w0 |= idx << (8 * c)
        else:
            w1 |= idx << (8 * (c - 4))
        g = 0
        for i in range(7):
            g ^= (code >> (7 - i)) & 1
            if i < 4:
                w2 |= g << (8 * i + 7 - c)
            else:
                w3 |= g << (8 * (i - 4) + 7 - c)
        w3 |= ((code & 1) ^ 1) << (31 - c)
    return w0, w1, w2, w3


def f16x2(word):
    return np.array([word & 0xFFFF, word >> 16], dtype=np.uint16).view(np.float16)


def decode_quad_like_kernel(q):
    """Mirror of stage_item<E8P> (e8p_words + shift_words) for one row quad ->
    (8, 8) floats: sign*|t| words from the table plus the +-1/4 shift words the
    tensor core adds against per-code activation sums."""
    w0, w1, w2, w3 = q
    flo = (w2 ^ (w2 << 8)) & M32
    fhi = ((w3 & 0x00FFFFFF) ^ (((w3 << 8) | (w2 >> 24)) & M32)) & M32
    # shift words: sw[p] = (code 2p+1 in the low half, code 2p in the high half)
    y = prmt(w3, (w3 << 1) & M32, 0x3070)
    sw = [0x34003400 ^ (((y << (2 * p)) & M32) & 0x80008000) for p in range(4)]
    shift = np.zeros(8, np.float32)
    for p in range(4):
        lo, hi = f16x2(sw[p])
        shift[2 * p + 1], shift[2 * p] = lo, hi
    out = []
    for c in range(8):
        idxsrc = w0 if c < 4 else w1
        idx = prmt(idxsrc, 0, 0x4440 | (c & 3))
        assert idx == (idxsrc >> (8 * (c & 3))) & 0xFF
        T = E8P_HB[idx]
        tl = T[0] ^ (((flo << c) & M32) & 0x80808080)
        th = T[1] ^ (((fhi << c) & M32) & 0x80808080)
        words = [prmt(tl, 0, 0x1404), prmt(tl, 0, 0x3424), prmt(th, 0, 0x1404), prmt(th, 0, 0x3424)]
        vals = np.concatenate([f16x2(w) for w in words]).astype(np.float32)
        out.append(vals + shift[c])
    return np.stack(out)


def test_e8p_packed_decode_matches_oracle():
    rng = np.random.default_rng(0)
    edge = np.array([0, 1, 0xFF, 0x100, 0x7FFF, 0x8000, 0xFFFE, 0xFFFF])
    for trial in range(300):
        codes = edge if trial == 0 else rng.integers(0, 65536, 8)
        got = decode_quad_like_kernel(pack_e8p_quad(codes))
        assert np.array_equal(got, O.e8p_decode(codes)), codes


def test_e8p_packed_decode_all_sign_patterns():
    # every (sign7, shift) combination for a spread of table rows
    for idx in (0, 1, 100, 226, 227, 255):
        low = np.arange(256)
        codes = (idx << 8) | low
        for q in range(32):
            blk = codes[8 * q: 8 * q + 8]
            assert np.array_equal(decode_quad_like_kernel(pack_e8p_quad(blk)), O.e8p_decode(blk))


def test_onebit_packed_decode_matches_oracle():
    for idx in range(256):
        lo, hi = ONEBIT_HB[idx]
        words = [prmt(lo, 0, 0x1404), prmt(lo, 0, 0x3424), prmt(hi, 0, 0x1404), prmt(hi, 0, 0x3424)]
        got = np.concatenate([f16x2(w) for w in words]).astype(np.float32)
        assert np.array_equal(got, O.e8_1bit_decode(np.array([idx]))[0])
