"""Fast Walsh-Hadamard transform on B200 (mirrors quipsharp/hadamard.py).

`fwht` keeps the reference signature and semantics (orthonormal natural-order
Sylvester transform along `dim`, ValueError for a non-power-of-two size,
quipsharp/hadamard.py:17-40) and runs the shared-memory butterfly kernel of
libquipsharp_b200 (`qs_fwht`).  CUDA tensors only.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import _native as N


def is_pow2(n: int) -> bool:
    """quipsharp/hadamard.py:9-10."""
    return n > 0 and (n & (n - 1)) == 0


def next_pow2(n: int) -> int:
    """quipsharp/hadamard.py:13-14."""
    return 1 << (n - 1).bit_length()


def _fwht_rows(x2d: Tensor, pre: Tensor | None = None, post: Tensor | None = None) -> Tensor:
    """y = post * H(pre * x) / sqrt(n) over the rows of a contiguous 2-D tensor."""
    rows, n = x2d.shape
    y = torch.empty_like(x2d)
    N.check(N.lib().qs_fwht(N.ptr(x2d), n, N.ptr(y), n, N.IO_DTYPES[x2d.dtype], rows, n,
                            N.ptr(pre), N.ptr(post), N.stream_of(x2d)))
    return y


def fwht(x: Tensor, dim: int = -1) -> Tensor:
    """Orthonormal fast Walsh-Hadamard transform along `dim` (H_n @ x / sqrt(n))."""
    x = x.movedim(dim, -1)
    n = x.shape[-1]
    if not is_pow2(n):
        raise ValueError(f"fwht requires a power-of-two size along dim, got {n}")
    N.require_cuda(x)
    if x.dtype not in N.IO_DTYPES:
        raise TypeError(f"fwht: unsupported dtype {x.dtype}")
    shape = x.shape
    y = _fwht_rows(x.reshape(-1, n).contiguous())
    return y.view(shape).movedim(-1, dim)


def rademacher(n: int, device=None, dtype=torch.float32, generator=None) -> Tensor:
    """Uniform random +-1 vector (quipsharp/hadamard.py:43-46)."""
    bits = torch.randint(0, 2, (n,), device=device, generator=generator)
    return bits.to(dtype) * 2 - 1
