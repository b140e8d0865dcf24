"""Randomized Hadamard incoherence transforms on B200 (mirrors quipsharp/incoherence.py).

Inference-time activation transforms of Algorithm 2 (quipsharp/incoherence.py:86-93):
    x2 = fwht(x * sv)       (transform_input)
    y  = fwht(y1) * su      (transform_output)
Each is one fused kernel (sign multiply folded into the load / store of the
shared-memory FWHT).  Offline incoherence processing of weights and Hessians
(quipsharp/incoherence.py:48-83) belongs to quantization and is not provided.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from . import _native as N
from .hadamard import _fwht_rows, fwht, is_pow2


def _as_f32(v: Tensor, device) -> Tensor:
    return v.to(device=device, dtype=torch.float32).contiguous()


def transform_input(x: Tensor, sv: Tensor) -> Tensor:
    """Algorithm 2 step 1: fwht(x * sv) over the last dim (incoherence.py:86-88)."""
    n = x.shape[-1]
    if not is_pow2(n):
        raise ValueError(f"fwht requires a power-of-two size along dim, got {n}")
    N.require_cuda(x, sv)
    out_dtype = torch.promote_types(x.dtype, sv.dtype)
    xin = x.to(out_dtype).reshape(-1, n).contiguous()
    return _fwht_rows(xin, pre=_as_f32(sv, x.device)).view(*x.shape[:-1], n)


def transform_output(y: Tensor, su: Tensor) -> Tensor:
    """Algorithm 2 step 3: fwht(y) * su over the last dim (incoherence.py:91-93)."""
    m = y.shape[-1]
    if not is_pow2(m):
        raise ValueError(f"fwht requires a power-of-two size along dim, got {m}")
    N.require_cuda(y, su)
    out_dtype = torch.promote_types(y.dtype, su.dtype)
    yin = y.to(out_dtype).reshape(-1, m).contiguous()
    return _fwht_rows(yin, post=_as_f32(su, y.device)).view(*y.shape[:-1], m)


@dataclass
class IncoherenceSigns:
    """Row / column sign vectors of a randomized-Hadamard layer (incoherence.py:29-45)."""
    su: Tensor  # (m,)
    sv: Tensor  # (n,)

    def transform_input(self, x: Tensor) -> Tensor:
        return transform_input(x, self.sv)

    def transform_output(self, y: Tensor) -> Tensor:
        return transform_output(y, self.su)

    def reconstruct_weight(self, what: Tensor) -> Tensor:
        return reconstruct_weight(what, self)


def reconstruct_weight(what: Tensor, signs: IncoherenceSigns) -> Tensor:
    """Invert the weight transform (incoherence.py:74-77): H_m What H_n * su * sv."""
    Z = fwht(fwht(what, dim=0), dim=1)
    return Z * signs.su.unsqueeze(1) * signs.sv.unsqueeze(0)


def linear_via_transformed(x: Tensor, what: Tensor, signs: IncoherenceSigns) -> Tensor:
    """Dense Algorithm 2 with an unquantized transformed weight (incoherence.py:96-104)."""
    return transform_output(transform_input(x, signs.sv) @ what.T, signs.su)


def incoherence_mu(W: Tensor) -> float:
    """Definition 2.1's incoherence parameter (incoherence.py:107-112)."""
    m, n = W.shape
    return (W.abs().max() * (m * n) ** 0.5 / W.norm()).item()
