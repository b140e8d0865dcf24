"""Residual vector quantization on B200 (mirrors quipsharp/rvq.py).

`rvq_dequantize` (rvq.py:83-88) sums float32(decode_s(code_s) * s_s) over the
stages in order; the kernel (`qs_rvq_decode`) reproduces torch's float32
roundings exactly.  `fit_stage_scale` / `fit_residual_stage_scale` (rvq.py:28-66)
run the reference's coarse scale sweep on the GPU (`qs_fit_scale_sweep`): the
load path needs them to rebuild a 3/4-bit codebook from (bits, seed).  The
Gaussian samples come from torch's CPU generator seeded as the reference seeds
it, so both sweep the same points.  RVQ encoding of weights (rvq_quantize,
rvq.py:69-80) belongs to offline quantization and is not provided.
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


def _swept(codebook):
    """(rvq, kinds, stage_scales) of the codebook a sweep quantizes with."""
    if hasattr(codebook, "stages"):
        return 1, [codebook_kind(st.codebook) for st in codebook.stages], [float(st.scale) for st in codebook.stages]
    return 0, [codebook_kind(codebook)], None


def _sweep_device(device) -> torch.device:
    """The CUDA device a sweep runs on (a CPU `device` -- where the reference would
    compute -- runs on the current CUDA device: the result is a Python float)."""
    if device is not None and torch.device(device).type == "cuda":
        return torch.device(device)
    if not torch.cuda.is_available():
        raise RuntimeError("the stage-scale sweep runs on a CUDA device (no CPU path); pass the stage "
                           "scales or a codebook to skip it")
    return torch.device("cuda", torch.cuda.current_device())


def sweep_scale_mse(x: Tensor, codebook, candidates, prev_stages=()) -> tuple[Tensor, int]:
    """Mean squared error E||x' - s Q(x' / s)||^2 of every candidate scale s, where
    x' = x - rvq_quantize(x, prev_stages) (x' = x without previous stages), and the
    index of the first candidate with the smallest error (rvq.py:28-37).
    x: (samples, 8) float32 on a CUDA device.  Returns (mse float64 (ncand,), best)."""
    N.require_cuda(x)
    if x.dim() != 2 or x.shape[1] != 8:
        raise NotImplementedError("the sweep kernel handles 8-dimensional codebooks")
    x = x.to(torch.float32).contiguous()
    cands = [float(c) for c in (candidates.tolist() if isinstance(candidates, Tensor) else candidates)]
    rvq, kinds, sscales = _swept(codebook)
    pk = [codebook_kind(st.codebook) for st in prev_stages]
    ps = [float(st.scale) for st in prev_stages]
    S = x.shape[0]
    nb = N.lib().qs_fit_workspace_bytes(S, len(cands))
    if nb < 0:
        raise ValueError(f"bad sweep size: {S} samples, {len(cands)} candidates")
    ws = torch.empty(nb, dtype=torch.uint8, device=x.device)
    mse = torch.empty(len(cands), dtype=torch.float64, device=x.device)
    best = torch.empty(1, dtype=torch.int32, device=x.device)
    N.check(N.lib().qs_fit_scale_sweep(
        N.ptr(x), S, len(pk), N.int_array(pk) if pk else None, N.float_array(ps) if ps else None, rvq, len(kinds),
        N.int_array(kinds), N.float_array(sscales) if sscales else None, N.float_array(cands), len(cands),
        N.ptr(ws), nb, N.ptr(mse), N.ptr(best), N.stream_of(x)))
    return mse, int(best.item())


def _gaussian(n_samples: int, dim: int, seed: int, device) -> Tensor:
    g = torch.Generator().manual_seed(seed)  # the reference's sampling (rvq.py:47-49, 60-62)
    return torch.randn(n_samples, dim, generator=g).to(_sweep_device(device))


def fit_stage_scale(codebook, dim: int = 8, n_samples: int = 200_000, candidates=None, seed: int = 0,
                    device=None) -> float:
    """rvq.py:40-50: the scale in `candidates` (default linspace(0.5, 4, 71)) minimizing
    E||x - s Q(x / s)||^2 for x ~ N(0, I_dim)."""
    if candidates is None:
        candidates = torch.linspace(0.5, 4.0, 71)
    x = _gaussian(n_samples, dim, seed, device)
    _, best = sweep_scale_mse(x, codebook, candidates)
    return float(candidates[best])


def fit_residual_stage_scale(prev_stages: list, codebook, dim: int = 8, n_samples: int = 200_000, candidates=None,
                             seed: int = 0, device=None) -> float:
    """rvq.py:53-66: the same sweep (default linspace(0.05, 2, 79)) on the residual
    x - rvq_quantize(x, prev_stages)."""
    if candidates is None:
        candidates = torch.linspace(0.05, 2.0, 79)
    x = _gaussian(n_samples, dim, seed, device)
    _, best = sweep_scale_mse(x, codebook, candidates, prev_stages)
    return float(candidates[best])


def rvq_quantize(*_a, **_k):
    raise NotImplementedError("RVQ encoding of weights is offline quantization")
