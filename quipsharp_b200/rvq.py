"""Residual vector quantization decode on B200 (mirrors quipsharp/rvq.py).

`rvq_dequantize` (rvq.py:83-88) sums float32(decode_s(code_s) * s_s) over the
stages in order; the kernel (`qs_rvq_decode`) reproduces torch's float32
roundings exactly.  Stage-scale fitting and RVQ encoding (rvq.py:28-80) belong
to offline quantization and are not provided.
"""
from __future__ import annotations

from dataclasses import dataclass

import ctypes

import torch
from torch import Tensor

from . import _native as N


@dataclass
class RVQStage:
    codebook: object  # E8PCodebook / E8OneBitCodebook (or the reference's classes)
    scale: float


def codebook_kind(codebook) -> int:
    """Map a codebook object (this package's or the reference's) to its kernel kind."""
    name = type(codebook).__name__
    if name == "E8PCodebook":
        return N.QS_CB_E8P
    if name == "E8OneBitCodebook":
        return N.QS_CB_E8_1BIT
    raise TypeError(f"unsupported codebook {name}")


def rvq_dequantize(codes: list, stages: list[RVQStage]) -> Tensor:
    if not 1 <= len(stages) <= 2 or len(codes) != len(stages):
        raise NotImplementedError("the kernels handle one or two RVQ stages")
    N.require_cuda(*codes)
    shape = codes[0].shape
    cs = []
    for c in codes:
        if c.shape != shape:
            raise ValueError("all stages need codes of the same shape")
        cs.append((c if c.dtype == torch.int64 else c.to(torch.int64)).contiguous())
    out = torch.empty(*shape, 8, device=cs[0].device, dtype=torch.float32)
    kinds = N.int_array([codebook_kind(s.codebook) for s in stages])
    ptrs = (ctypes.c_void_p * len(cs))(*[c.data_ptr() for c in cs])
    scales = N.float_array([float(s.scale) for s in stages])
    N.check(N.lib().qs_rvq_decode(len(stages), kinds, ptrs, N.QS_I64, scales, cs[0].numel(),
                                  N.ptr(out), N.stream_of(cs[0])))
    return out


def _offline(*_a, **_k):
    raise NotImplementedError("RVQ scale fitting / encoding is offline quantization")


fit_stage_scale = fit_residual_stage_scale = rvq_quantize = _offline
