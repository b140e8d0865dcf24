"""1-bit E8 codebook on B200 (mirrors quipsharp/codebooks/e8_1bit.py): 256
vectors (zero, the 240-vector norm^2=2 shell, 15 norm^2=4 vectors); decode is
a table gather (e8_1bit.py:86-87) done by `qs_decode`.  Out-of-range indices
raise IndexError like torch indexing."""
from __future__ import annotations

import torch
from torch import Tensor

from .. import _native as N
from .e8p import decode_codes
from .tables import e8_1bit_table_x2, _int_shell_x2, _half_shell_x2

CODE_DIM = 8
TABLE_SIZE = 256


def _norm2_shell() -> Tensor:
    """The 240 minimal vectors of E8 (e8_1bit.py:52-56)."""
    return torch.tensor(_int_shell_x2(2) + _half_shell_x2(2), dtype=torch.float32) / 2


def build_table() -> Tensor:
    """(256, 8) float32 table (e8_1bit.py:67-71)."""
    return torch.tensor(e8_1bit_table_x2(), dtype=torch.float32) / 2


class E8OneBitCodebook:
    """1-bit (8 bits / 8 dims) codebook (e8_1bit.py:73-87)."""

    kind = N.QS_CB_E8_1BIT

    def __init__(self, device=None):
        self.table = build_table().to(device=device)

    def quantize(self, x: Tensor):
        raise NotImplementedError("1-bit E8 encoding is offline quantization; this package "
                                  "provides the inference path only")

    def dequantize(self, idx: Tensor) -> Tensor:
        return decode_codes(N.QS_CB_E8_1BIT, idx)
