"""CPU oracle for the quantized-linear forward path -- TEST INFRASTRUCTURE ONLY.

This module is a plain-numpy restatement of the reference (numbersletter/quipsharp)
algorithm for the hot path `QuantizedLinear.forward`.  It exists to check the
CUDA kernels; it is never imported by the product package.  Only `tests/`,
`__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of
`bench.py` may use it.

Parity pin: every function here is checked against golden vectors produced by
running the reference itself (tests/golden/make_golden.py imports the reference
and writes tests/golden/*.npz); tests/test_oracle_golden.py asserts equality
(bit-exact for tables and decode, tight tolerance for the floating-point
transforms whose summation order differs from torch's pocketfft / MKL).

Each function cites the reference file:line it restates (paths relative to the
reference project root).
"""
from __future__ import annotations

import itertools

import numpy as np

CODE_DIM = 8

# quipsharp/codebooks/e8p.py:31-61 -- the 29 norm^2=12 padding rows (x2).
_PAD29_X2 = np.array([
    [3, 1, 1, 1, 3, 3, 3, 3], [1, 3, 1, 1, 3, 3, 3, 3], [1, 1, 3, 1, 3, 3, 3, 3],
    [1, 1, 1, 3, 3, 3, 3, 3], [3, 3, 3, 1, 3, 3, 1, 1], [3, 3, 3, 1, 3, 1, 3, 1],
    [3, 3, 3, 1, 1, 3, 3, 1], [3, 3, 3, 1, 3, 1, 1, 3], [3, 3, 3, 1, 1, 3, 1, 3],
    [3, 3, 3, 1, 1, 1, 3, 3], [3, 3, 1, 3, 3, 3, 1, 1], [3, 3, 1, 3, 3, 1, 3, 1],
    [3, 3, 1, 3, 1, 3, 3, 1], [3, 3, 1, 3, 3, 1, 1, 3], [3, 3, 1, 3, 1, 3, 1, 3],
    [3, 3, 1, 3, 1, 1, 3, 3], [3, 1, 3, 3, 3, 3, 1, 1], [3, 1, 3, 3, 3, 1, 3, 1],
    [3, 1, 3, 3, 1, 3, 3, 1], [3, 1, 3, 3, 3, 1, 1, 3], [3, 1, 3, 3, 1, 3, 1, 3],
    [1, 3, 3, 3, 1, 1, 3, 3], [1, 3, 3, 3, 3, 3, 1, 1], [1, 3, 3, 3, 3, 1, 3, 1],
    [1, 3, 3, 3, 1, 3, 3, 1], [1, 3, 3, 3, 3, 1, 1, 3], [1, 3, 3, 3, 1, 3, 1, 3],
    [1, 1, 3, 3, 1, 3, 3, 3], [3, 3, 1, 1, 3, 3, 3, 1],
], dtype=np.int64)


def e8p_abs_table() -> np.ndarray:
    """(256, 8) float32 E8P base table.

    Restates quipsharp/codebooks/e8p.py:64-89: the distinct |x| patterns of
    D8-hat = {x in Z^8 + 1/2 : sum(x) even} with ||x||^2 <= 10, sorted
    lexicographically (torch.unique(dim=0) order), followed by the 29 padding
    rows, then every row with an odd coordinate sum has its last coordinate
    negated (e8p.py:75-81).  Any abs pattern of half-integers admits an
    even-sum sign choice (one flip changes the sum by an odd integer), so the
    abs patterns are exactly the half-integer patterns inside the ball.
    """
    vals2 = (1, 3, 5, 7)  # 2*|x| for |x| in {0.5, 1.5, 2.5, 3.5}
    rows = [r for r in itertools.product(vals2, repeat=CODE_DIM)
            if sum(v * v for v in r) <= 40]          # ||x||^2 <= 10  <=>  sum (2x)^2 <= 40
    rows.sort()                                       # lexicographic == torch.unique order
    base2 = np.concatenate([np.array(rows, dtype=np.int64), _PAD29_X2], axis=0)
    assert base2.shape == (256, CODE_DIM), base2.shape
    odd = (base2.sum(-1) // 2) % 2 != 0               # sum(x) = sum(2x)/2 is an integer
    base2[odd, -1] *= -1
    return (base2.astype(np.float32) / np.float32(2.0)).astype(np.float32)


def _integer_shell(norm_sq: int) -> np.ndarray:
    """quipsharp/codebooks/e8_1bit.py:32-39, in itertools.product (== cartesian_prod) order."""
    bound = int(norm_sq ** 0.5)
    vals = range(-bound, bound + 1)
    out = [r for r in itertools.product(vals, repeat=CODE_DIM)
           if sum(v * v for v in r) == norm_sq and sum(r) % 2 == 0]
    return np.array(out, dtype=np.float64)


def _half_integer_shell(norm_sq: int) -> np.ndarray:
    """quipsharp/codebooks/e8_1bit.py:42-49 (coordinates x2 to stay integral)."""
    bound = int(norm_sq ** 0.5) + 1
    vals2 = [2 * v + 1 for v in range(-bound, bound)]  # 2*(v + 0.5)
    out = [r for r in itertools.product(vals2, repeat=CODE_DIM)
           if sum(v * v for v in r) == 4 * norm_sq and (sum(r) // 2) % 2 == 0]
    return np.array(out, dtype=np.float64) / 2.0


def e8_1bit_table() -> np.ndarray:
    """(256, 8) float32 table: zero row, the 240 norm^2=2 shell (integer part
    then half-integer part), then the first 15 integer norm^2=4 vectors.
    Restates quipsharp/codebooks/e8_1bit.py:52-71."""
    shell = np.concatenate([_integer_shell(2), _half_integer_shell(2)], axis=0)
    assert shell.shape == (240, CODE_DIM)
    pad = _integer_shell(4)[:15]
    table = np.concatenate([np.zeros((1, CODE_DIM)), shell, pad], axis=0)
    assert table.shape == (256, CODE_DIM)
    return table.astype(np.float32)


_ABS = None
_ONEBIT = None


def _tables():
    global _ABS, _ONEBIT
    if _ABS is None:
        _ABS, _ONEBIT = e8p_abs_table(), e8_1bit_table()
    return _ABS, _ONEBIT


def e8p_unpack(code: np.ndarray):
    """quipsharp/codebooks/e8p.py:174-180: [abs:8][sign7:7][shift:1]; sign bit i
    (coordinate i < 7) is bit (7 - i) of the code."""
    code = np.asarray(code, dtype=np.int64)
    abs_idx = (code >> 8) & 0xFF
    shift_bit = code & 1
    sign_int = (code >> 1) & 0x7F
    bits = np.stack([(sign_int >> (6 - i)) & 1 for i in range(7)], axis=-1)
    return abs_idx, bits, shift_bit


_E8P_LUT = None


def e8p_decode(code: np.ndarray) -> np.ndarray:
    """E8PCodebook.dequantize via a 65536 x 8 lookup table built once from
    `e8p_decode_bits` (same values, bit for bit; only the 16 low bits of a code
    matter, e8p.py:174-180).  This keeps the CPU baseline fast."""
    global _E8P_LUT
    if _E8P_LUT is None:
        _E8P_LUT = e8p_decode_bits(np.arange(65536))
    return np.take(_E8P_LUT, np.asarray(code, dtype=np.int64) & 0xFFFF, axis=0)


def e8p_decode_bits(code: np.ndarray) -> np.ndarray:
    """E8PCodebook.dequantize: quipsharp/codebooks/e8p.py:92-101, 197-199.
    The 8th flip is the parity of the 7 stored flips; shift bit 1 -> +1/4."""
    abs_tab, _ = _tables()
    abs_idx, bits, shift_bit = e8p_unpack(code)
    base = abs_tab[abs_idx]
    inferred = bits.sum(-1) % 2
    flips = np.concatenate([bits, inferred[..., None]], axis=-1).astype(np.float32)
    signed = base * (np.float32(1.0) - np.float32(2.0) * flips)
    shift = (np.float32(2.0) * shift_bit.astype(np.float32) - np.float32(1.0)) * np.float32(0.25)
    return (signed + shift[..., None]).astype(np.float32)


def e8_1bit_decode(idx: np.ndarray) -> np.ndarray:
    """E8OneBitCodebook.dequantize: quipsharp/codebooks/e8_1bit.py:86-87 (plain
    table gather; indices must lie in [-256, 256) like torch indexing)."""
    _, tab = _tables()
    idx = np.asarray(idx, dtype=np.int64)
    if idx.size and (idx.min() < -256 or idx.max() >= 256):
        raise IndexError("1-bit codebook index out of range")
    return np.take(tab, idx % 256, axis=0)


E8P = "e8p"
E8_1BIT = "e8_1bit"


def stage_decode(kind: str, code: np.ndarray) -> np.ndarray:
    return e8p_decode(code) if kind == E8P else e8_1bit_decode(code)


def rvq_decode(codes, kinds, scales) -> np.ndarray:
    """rvq_dequantize (quipsharp/rvq.py:83-88) through RVQCodebookAdapter
    (quipsharp/quantize.py:43-45): sum_i fl32(decode_i(code_i) * fl32(s_i)),
    accumulated left to right in float32."""
    total = None
    for kind, code, s in zip(kinds, codes, scales):
        vals = stage_decode(kind, code)
        vals *= np.float32(s)                      # float32 * float32, rounded once
        if total is None:
            total = vals
        else:
            total += vals
    return total


def dequantize_linear(codes: np.ndarray, kinds, stage_scales, layer_scale: float,
                      m: int, n: int, g: int = 8) -> np.ndarray:
    """quipsharp/quantize.py:107-113 with the int16 -> & 0xFFFF unpacking of
    quipsharp/checkpoint.py:136.  codes: (m, n/8) for one stage or
    (stages, m, n/8).  Returns the (m, n) float32 transformed weight."""
    c = np.asarray(codes).astype(np.int64) & 0xFFFF
    if c.ndim == 2:
        c = c[None]
    T = n // g
    assert c.shape[1:] == (m, T), (c.shape, m, T)
    if len(kinds) == 1 and stage_scales is None:
        blocks = stage_decode(kinds[0], c[0])                 # (m, T, 8)
    else:
        blocks = rvq_decode([c[i] for i in range(c.shape[0])], kinds, stage_scales)
    w = blocks.reshape(m, n)
    return (w * np.float32(layer_scale)).astype(np.float32)


def is_pow2(n: int) -> bool:
    """quipsharp/hadamard.py:9-10."""
    return n > 0 and (n & (n - 1)) == 0


def fwht(x: np.ndarray) -> np.ndarray:
    """Orthonormal Sylvester FWHT over the last axis, float32, same butterfly
    order as quipsharp/hadamard.py:17-40 (h = 1, 2, 4, ...; then * n^-1/2)."""
    x = np.asarray(x, dtype=np.float32)
    n = x.shape[-1]
    if not is_pow2(n):
        raise ValueError(f"fwht requires a power-of-two size along dim, got {n}")
    shape = x.shape
    y = x.reshape(-1, n).copy()
    h = 1
    while h < n:
        y = y.reshape(-1, n // (2 * h), 2, h)
        a = y[:, :, 0, :]
        b = y[:, :, 1, :]
        y = np.stack((a + b, a - b), axis=2).reshape(-1, n)
        h *= 2
    return (y * np.float32(n ** -0.5)).astype(np.float32).reshape(shape)


def rht_transform_input(x: np.ndarray, sv: np.ndarray) -> np.ndarray:
    """quipsharp/incoherence.py:86-88: fwht(x * sv)."""
    return fwht((np.asarray(x, np.float32) * np.asarray(sv, np.float32)).astype(np.float32))


def rht_transform_output(y: np.ndarray, su: np.ndarray) -> np.ndarray:
    """quipsharp/incoherence.py:91-93: fwht(y) * su."""
    return (fwht(y) * np.asarray(su, np.float32)).astype(np.float32)


def rfft_to_transformed(x: np.ndarray, phase: np.ndarray) -> np.ndarray:
    """quipsharp/rfft.py:37-47: view adjacent reals as complex, multiply by
    phase, orthonormal FFT, view back as reals.  Computed in complex128 and
    rounded to float32 (pocketfft's own rounding is not reproduced)."""
    x = np.asarray(x, dtype=np.float32)
    n = x.shape[-1]
    assert n == 2 * phase.shape[-1], f"expected last dim {2 * phase.shape[-1]}, got {n}"
    xc = x[..., 0::2].astype(np.float64) + 1j * x[..., 1::2].astype(np.float64)
    pc = np.asarray(phase).astype(np.complex64).astype(np.complex128)
    X = np.fft.fft(xc * pc, axis=-1, norm="ortho")
    out = np.empty(x.shape, dtype=np.float32)
    out[..., 0::2] = X.real
    out[..., 1::2] = X.imag
    return out


def rfft_from_transformed(y: np.ndarray, phase: np.ndarray) -> np.ndarray:
    """quipsharp/rfft.py:50-60: orthonormal IFFT, then multiply by conj(phase)."""
    y = np.asarray(y, dtype=np.float32)
    n = y.shape[-1]
    assert n == 2 * phase.shape[-1], f"expected last dim {2 * phase.shape[-1]}, got {n}"
    yc = y[..., 0::2].astype(np.float64) + 1j * y[..., 1::2].astype(np.float64)
    pc = np.asarray(phase).astype(np.complex64).astype(np.complex128)
    X = np.fft.ifft(yc, axis=-1, norm="ortho") * np.conj(pc)
    out = np.empty(y.shape, dtype=np.float32)
    out[..., 0::2] = X.real
    out[..., 1::2] = X.imag
    return out


def transform_kind_for(m: int, n: int) -> str:
    """quipsharp/incoherence.py:115-131: RHT iff both dims are powers of two."""
    return "rht" if (is_pow2(m) and is_pow2(n)) else "rfft"


def linear_forward(x: np.ndarray, codes, kinds, stage_scales, layer_scale: float,
                   transform_kind: str, su=None, sv=None, phase_u=None, phase_v=None,
                   bias=None, out_dtype=None) -> np.ndarray:
    """QuantizedLinear.forward (quipsharp/checkpoint.py:141-146) ->
    linear_forward (quipsharp/quantize.py:116-124): upcast to float32,
    transform_in, x2 @ What^T, transform_out, + bias, cast back."""
    xf = np.asarray(x, dtype=np.float32)
    n = xf.shape[-1]
    c = np.asarray(codes)
    m = c.shape[-2]
    w = dequantize_linear(c, kinds, stage_scales, layer_scale, m, n)
    if transform_kind == "rht":
        x2 = rht_transform_input(xf, sv)
    else:
        x2 = rfft_to_transformed(xf, phase_v)
    y1 = (x2.astype(np.float32) @ w.T).astype(np.float32)
    y = rht_transform_output(y1, su) if transform_kind == "rht" else rfft_from_transformed(y1, phase_u)
    if bias is not None:
        y = (y + np.asarray(bias, np.float32)).astype(np.float32)
    return y if out_dtype is None else y.astype(out_dtype)


# ---- codebook construction: nearest-point search and the scale sweep --------------

def e8p_nearest(y: np.ndarray) -> np.ndarray:
    """E8PCodebook.quantize values (quipsharp/codebooks/e8p.py:104-160), float32.

    For z = y + 1/4 and z = y - 1/4, each of the 256 base rows takes the signs
    agreeing with z (flip where z_i a_i < 0), repaired to even parity by toggling
    the coordinate with the smallest |z_i a_i| (first on ties); the row nearest to
    z wins (first on ties), the + side wins ties between sides, and the value is
    v - 1/4 (+ side) or v + 1/4 (- side).  y: (S, 8) float32."""
    abs_tab, _ = _tables()
    y = np.asarray(y, dtype=np.float32)

    def side(z):
        prod = z[:, None, :] * abs_tab[None]                       # (S, 256, 8)
        flip = prod < 0
        wrong = flip.sum(-1) % 2 == 1
        mc = np.abs(prod).argmin(-1)                               # first smallest
        s_idx, k_idx = np.nonzero(wrong)
        flip[s_idx, k_idx, mc[s_idx, k_idx]] ^= True
        vals = np.where(flip, -abs_tab[None], abs_tab[None]).astype(np.float32)
        d2 = ((z[:, None, :] - vals) ** 2).sum(-1, dtype=np.float32)
        k = d2.argmin(-1)                                          # first nearest row
        r = np.arange(z.shape[0])
        return vals[r, k], d2[r, k]

    pv, pd = side((y + np.float32(0.25)).astype(np.float32))
    mv, md = side((y - np.float32(0.25)).astype(np.float32))
    plus = (pd <= md)[:, None]
    return np.where(plus, pv - np.float32(0.25), mv + np.float32(0.25)).astype(np.float32)


def e8_1bit_nearest(y: np.ndarray) -> np.ndarray:
    """E8OneBitCodebook.quantize values (quipsharp/codebooks/e8_1bit.py:81-84):
    the table row nearest to y (first on ties), float32."""
    _, tab = _tables()
    y = np.asarray(y, dtype=np.float32)
    d2 = ((y[:, None, :] - tab[None]) ** 2).sum(-1, dtype=np.float32)
    return tab[d2.argmin(-1)]


def stage_nearest(kind: str, y: np.ndarray) -> np.ndarray:
    return e8p_nearest(y) if kind == E8P else e8_1bit_nearest(y)


def rvq_quantize_vals(x: np.ndarray, stages) -> np.ndarray:
    """rvq_quantize values (quipsharp/rvq.py:69-80): per stage (kind, scale),
    q = Q(r / s), total += q s, r -= q s, in float32."""
    r = np.asarray(x, dtype=np.float32)
    total = np.zeros_like(r)
    for kind, s in stages:
        s = np.float32(s)
        q = stage_nearest(kind, (r / s).astype(np.float32))
        qs = (q * s).astype(np.float32)
        total = (total + qs).astype(np.float32)
        r = (r - qs).astype(np.float32)
    return total


def sweep_scale_mse(x: np.ndarray, stages, candidates, rvq: bool, prev=()) -> np.ndarray:
    """Per candidate s: mean (x' - s Q(x' / s))^2 over all elements, float64, where
    x' = x - rvq_quantize(x, prev) (rvq.py:28-37, 53-66).  Q is the plain codebook
    stages[0][0] (rvq False) or the RVQ of `stages` (rvq True)."""
    x = np.asarray(x, dtype=np.float32)
    if prev:
        x = (x - rvq_quantize_vals(x, prev)).astype(np.float32)
    out = []
    for s in candidates:
        s = np.float32(s)
        y = (x / s).astype(np.float32)
        q = rvq_quantize_vals(y, stages) if rvq else stage_nearest(stages[0][0], y)
        e = (x - (q * s).astype(np.float32)).astype(np.float32)
        out.append(float(np.mean((e * e).astype(np.float32), dtype=np.float64)))
    return np.array(out)
