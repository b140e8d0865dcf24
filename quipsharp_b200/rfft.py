"""Randomized-FFT incoherence transforms on B200 (mirrors quipsharp/rfft.py).

`to_transformed_space` / `from_transformed_space` keep the reference semantics
(quipsharp/rfft.py:37-60): adjacent reals form complex numbers, which are
multiplied by a unit phase and FFT'd with orthonormal scaling (or IFFT'd and
multiplied by the conjugate phase).  They run the mixed-radix shared-memory
FFT kernel of libquipsharp_b200 (`qs_rfft`); results are float32 like the
reference's complex64 arithmetic.  Row lengths up to 32768 reals whose half has
prime factors up to 43 are supported.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import Tensor

from . import _native as N


def random_phase(n_half: int, device=None, generator=None) -> Tensor:
    """Uniform random unit-modulus complex vector (quipsharp/rfft.py:31-34)."""
    theta = torch.rand(n_half, device=device, generator=generator) * (2 * math.pi)
    return torch.polar(torch.ones_like(theta), theta)


def _rfft_rows(x2d: Tensor, phase: Tensor, inverse: bool) -> Tensor:
    rows, n = x2d.shape
    y = torch.empty_like(x2d)
    ph = torch.view_as_real(phase.to(device=x2d.device, dtype=torch.complex64).contiguous())
    N.check(N.lib().qs_rfft(int(inverse), N.ptr(x2d), n, N.ptr(y), n, N.IO_DTYPES[x2d.dtype],
                            rows, n, N.ptr(ph), N.stream_of(x2d)))
    return y


def to_transformed_space(x: Tensor, phase: Tensor, dim: int = -1) -> Tensor:
    """Enter the RFFT space: complex view, * phase, orthonormal FFT (rfft.py:37-47)."""
    x = x.movedim(dim, -1)
    n = x.shape[-1]
    assert n == 2 * phase.shape[-1], f"expected last dim {2 * phase.shape[-1]}, got {n}"
    N.require_cuda(x, phase)
    shape = x.shape
    y = _rfft_rows(x.reshape(-1, n).to(torch.float32).contiguous(), phase, inverse=False)
    return y.view(shape).movedim(-1, dim)


def from_transformed_space(y: Tensor, phase: Tensor, dim: int = -1) -> Tensor:
    """Exit the RFFT space: orthonormal IFFT, * conj(phase) (rfft.py:50-60)."""
    y = y.movedim(dim, -1)
    n = y.shape[-1]
    assert n == 2 * phase.shape[-1], f"expected last dim {2 * phase.shape[-1]}, got {n}"
    N.require_cuda(y, phase)
    shape = y.shape
    x = _rfft_rows(y.reshape(-1, n).to(torch.float32).contiguous(), phase, inverse=True)
    return x.view(shape).movedim(-1, dim)


@dataclass
class RFFTPhases:
    """Row / column phases of an RFFT layer (rfft.py:63-77)."""
    phase_u: Tensor  # (m//2,) complex
    phase_v: Tensor  # (n//2,) complex

    def transform_input(self, x: Tensor) -> Tensor:
        return to_transformed_space(x, self.phase_v, dim=-1)

    def transform_output(self, y: Tensor) -> Tensor:
        return from_transformed_space(y, self.phase_u, dim=-1)

    def reconstruct_weight(self, what: Tensor) -> Tensor:
        return reconstruct_weight(what, self)


def reconstruct_weight(what: Tensor, phases: RFFTPhases) -> Tensor:
    """Invert the RFFT weight transform (rfft.py:80-84)."""
    y = from_transformed_space(what, phases.phase_v, dim=1)
    return from_transformed_space(y, phases.phase_u, dim=0)
