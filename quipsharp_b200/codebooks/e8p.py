"""E8P 2-bit codebook on B200 (mirrors quipsharp/codebooks/e8p.py).

A 16-bit code [abs:8][sign7:7][shift:1] selects one of 256 base rows, flips the
signs of coordinates 0..6 by its sign bits and of coordinate 7 by their parity,
and adds +-1/4 (e8p.py:92-101, 174-180).  `E8PCodebook.dequantize` runs the
bit-exact decode kernel (`qs_decode`).  The nearest-point encoder
(`quantize`, e8p.py:104-162) belongs to offline quantization and is not provided.
"""
from __future__ import annotations

import torch
from torch import Tensor

from .. import _native as N
from .tables import e8p_abs_table_x2, d8hat_abs_patterns_x2, PAD29_X2

CODE_DIM = 8
ABS_TABLE_SIZE = 256


def _enumerate_d8hat_abs_le_norm10() -> Tensor:
    """The 227 |x| patterns of D8-hat with ||x||^2 <= 10 (e8p.py:64-72)."""
    return torch.tensor(d8hat_abs_patterns_x2(), dtype=torch.float32) / 2


_PAD29_RAW = torch.tensor(PAD29_X2, dtype=torch.float32) / 2


def build_abs_table() -> Tensor:
    """(256, 8) float32 E8P base table (e8p.py:84-89)."""
    return torch.tensor(e8p_abs_table_x2(), dtype=torch.float32) / 2


def unpack_code(code: Tensor):
    """e8p.py:174-180: (abs_idx, sign_bits7 (..., 7), shift_bit)."""
    abs_idx = (code >> 8) & 0xFF
    shift_bit = code & 1
    sign_int = (code >> 1) & 0x7F
    sign_bits7 = torch.stack([(sign_int >> (6 - i)) & 1 for i in range(7)], dim=-1)
    return abs_idx, sign_bits7, shift_bit


def pack_code(abs_idx: Tensor, sign_bits7: Tensor, shift_bit: Tensor) -> Tensor:
    """e8p.py:165-171: [abs_idx:8][sign_bits7:7][shift_bit:1]."""
    sign_int = torch.zeros_like(abs_idx, dtype=torch.int64)
    for i in range(7):
        sign_int = sign_int | (sign_bits7[..., i].to(torch.int64) << (6 - i))
    return (abs_idx.to(torch.int64) << 8) | (sign_int << 1) | shift_bit.to(torch.int64)


def decode_from_table(abs_idx: Tensor, sign_bits7: Tensor, shift_bit: Tensor,
                      abs_table: Tensor) -> Tensor:
    """Decode unpacked fields against an arbitrary table (e8p.py:92-101).  The
    packed-code path `E8PCodebook.dequantize` is the kernel-backed one."""
    base = abs_table[abs_idx]
    inferred = sign_bits7.sum(-1) % 2
    all_flip = torch.cat([sign_bits7, inferred.unsqueeze(-1)], dim=-1)
    signed = base * (1 - 2 * all_flip.to(base.dtype))
    shift = (2 * shift_bit.to(base.dtype) - 1) * 0.25
    return signed + shift.unsqueeze(-1)


def decode_codes(kind: int, code: Tensor) -> Tensor:
    """Kernel decode of any integer code tensor (...,) -> (..., 8) float32."""
    N.require_cuda(code)
    c = code if code.dtype in N.CODE_DTYPES else code.to(torch.int64)
    c = c.contiguous()
    out = torch.empty(*c.shape, CODE_DIM, device=c.device, dtype=torch.float32)
    N.check(N.lib().qs_decode(kind, N.ptr(c), N.CODE_DTYPES[c.dtype], c.numel(), N.ptr(out),
                              N.stream_of(c)))
    return out


class E8PCodebook:
    """2-bit (16 bits / 8 dims) E8P codebook (e8p.py:183-199)."""

    kind = N.QS_CB_E8P

    def __init__(self, device=None):
        self.abs_table = build_abs_table().to(device=device)

    def quantize(self, x: Tensor):
        raise NotImplementedError("E8P encoding is offline quantization; this package provides "
                                  "the inference path only")

    def dequantize(self, code: Tensor) -> Tensor:
        return decode_codes(N.QS_CB_E8P, code)
