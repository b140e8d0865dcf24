"""Algorithm 2 (quantized-linear inference) on B200 (mirrors quipsharp/quantize.py).

`dequantize_linear` (quantize.py:107-113) and `linear_forward` (quantize.py:116-124)
keep the reference signatures.  `linear_forward` runs the fused path of
libquipsharp_b200: input transform kernel -> fused decode+matmul kernel ->
output transform kernel; the dense weight is never materialised.  Algorithm 1
(`quantize_linear`, BlockLDLQ) is offline quantization and is not provided.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from . import _native as N
from .incoherence import IncoherenceSigns
from .rfft import RFFTPhases
from .rvq import RVQStage, codebook_kind, rvq_dequantize


@dataclass
class QuantizedLayer:
    codes: Tensor  # (..., m, n // g)
    signs: object  # IncoherenceSigns or RFFTPhases
    g: int
    shape: tuple[int, int]
    scale: float


class RVQCodebookAdapter:
    """A list of RVQ stages behind the single-codebook interface (quantize.py:31-45)."""

    def __init__(self, stages: list[RVQStage]):
        self.stages = stages

    def quantize(self, x: Tensor):
        raise NotImplementedError("RVQ encoding is offline quantization")

    def dequantize(self, code: Tensor) -> Tensor:
        return rvq_dequantize([code[i] for i in range(code.shape[0])], self.stages)


def codebook_spec(codebook):
    """(kinds, stage_scales) of a codebook: a plain codebook has no stage
    scales; an RVQ adapter (ours or the reference's) one float per stage."""
    if hasattr(codebook, "stages"):
        return [codebook_kind(s.codebook) for s in codebook.stages], [float(s.scale) for s in codebook.stages]
    return [codebook_kind(codebook)], None


def _codes_i16(codes: Tensor, stages: int, m: int, T: int) -> Tensor:
    c = codes if codes.dim() == 3 else codes.reshape(1, *codes.shape[-2:])
    if c.shape != (stages, m, T):
        raise ValueError(f"codes of shape {tuple(codes.shape)} do not match {stages} stage(s) of ({m}, {T})")
    return (c if c.dtype == torch.int16 else c.to(torch.int16)).contiguous()


def _scale_tensor(scale, device) -> Tensor:
    if isinstance(scale, Tensor):
        return scale.to(device=device, dtype=torch.float32).reshape(())
    return torch.tensor(float(scale), dtype=torch.float32, device=device)


def dequantize_linear(layer: QuantizedLayer, codebook) -> Tensor:
    """The transformed weight What (m, n) float32, bit-exact with the reference."""
    m, n = layer.shape
    kinds, ss = codebook_spec(codebook)
    N.require_cuda(layer.codes)
    codes = _codes_i16(layer.codes, len(kinds), m, n // layer.g)
    out = torch.empty(m, n, device=codes.device, dtype=torch.float32)
    scale = _scale_tensor(layer.scale, codes.device)
    N.check(N.lib().qs_dequantize_linear(N.ptr(codes), len(kinds), N.int_array(kinds),
                                         None if ss is None else N.float_array(ss), N.ptr(scale),
                                         m, n, N.ptr(out), N.stream_of(codes)))
    return out


def pack_codes(codes: Tensor, kinds, m: int, n: int) -> Tensor:
    """Kernel-ready weight stream (uint8) from int16 codes (stages, m, n/8)."""
    c = _codes_i16(codes, len(kinds), m, n // 8)
    karr = N.int_array(kinds)
    nbytes = N.lib().qs_packed_bytes(len(kinds), karr, m, n)
    if nbytes < 0:
        raise ValueError("bad layer shape for packing")
    packed = torch.empty(nbytes, dtype=torch.uint8, device=c.device)
    N.check(N.lib().qs_pack_codes(N.ptr(c), len(kinds), karr, m, n, N.ptr(packed), nbytes,
                                  N.stream_of(c)))
    return packed


class LinearKernel:
    """Everything the fused forward needs for one layer, resolved once:
    packed weight stream, codebook kinds / stage scales, transform buffers."""

    def __init__(self, codes: Tensor, codebook, m: int, n: int, scale: Tensor, transform: str,
                 su=None, sv=None, phase_u=None, phase_v=None, bias=None):
        self.m, self.n = m, n
        self.kinds, self.stage_scales = codebook_spec(codebook)
        dev = codes.device
        self.packed = pack_codes(codes, self.kinds, m, n)
        self.scale = _scale_tensor(scale, dev)
        self.transform = N.QS_RHT if transform == "rht" else N.QS_RFFT
        f32 = lambda t: None if t is None else t.to(device=dev, dtype=torch.float32).contiguous()
        c64 = lambda t: None if t is None else torch.view_as_real(
            t.to(device=dev, dtype=torch.complex64).contiguous())
        self.su, self.sv = f32(su), f32(sv)
        self.phase_u, self.phase_v = c64(phase_u), c64(phase_v)
        self.bias = f32(bias)
        self._kinds_c = N.int_array(self.kinds)
        self._ss_c = None if self.stage_scales is None else N.float_array(self.stage_scales)

    def workspace_bytes(self, batch: int) -> int:
        return N.lib().qs_linear_workspace_bytes(batch, self.m, self.n)

    # ---- the three steps, for callers that insert a collective (tensor parallel)
    def input(self, x2: Tensor, y1: Tensor | None) -> Tensor:
        """x2 (B, n) -> fp16 matmul operand workspace; zeroes y1 (B, m) if given."""
        B = x2.shape[0]
        nb = N.lib().qs_linear_input_bytes(B, self.n)
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=x2.device)
        N.check(N.lib().qs_linear_input(N.ptr(x2), N.IO_DTYPES[x2.dtype], B, self.n, self.transform,
                                        N.ptr(self.sv), N.ptr(self.phase_v), N.ptr(ws), ws.numel(),
                                        N.ptr(y1), 0 if y1 is None else self.m, N.stream_of(x2)))
        return ws

    def matmul(self, ws: Tensor, B: int, y1: Tensor) -> None:
        """y1 (B, m) float32 += x2 @ What^T (this kernel's rows)."""
        N.check(N.lib().qs_linear_matmul(N.ptr(ws), B, self.n, self.m, N.ptr(self.packed), len(self.kinds),
                                         self._kinds_c, self._ss_c, N.ptr(self.scale), N.ptr(y1),
                                         N.stream_of(y1)))

    def __call__(self, x: Tensor, out: Tensor | None = None, workspace: Tensor | None = None) -> Tensor:
        """x (..., n) of float32/float16/bfloat16 -> y (..., m) of the same dtype."""
        N.require_cuda(x)
        if x.device.index != torch.cuda.current_device():  # launch on the device that holds the layer
            with torch.cuda.device(x.device):
                return self(x, out, workspace)
        lead = x.shape[:-1]
        io_dtype = x.dtype if x.dtype in N.IO_DTYPES else torch.float32
        x2 = x.reshape(-1, self.n).to(io_dtype).contiguous()
        B = x2.shape[0]
        y = out if out is not None else torch.empty(B, self.m, device=x.device, dtype=io_dtype)
        wsb = self.workspace_bytes(B)
        ws = workspace if workspace is not None else torch.empty(max(wsb, 1), dtype=torch.uint8, device=x.device)
        N.check(N.lib().qs_linear_fwd(
            N.ptr(x2), N.IO_DTYPES[io_dtype], B, self.n, self.m, N.ptr(self.packed),
            len(self.kinds), self._kinds_c, self._ss_c, N.ptr(self.scale), self.transform,
            N.ptr(self.su), N.ptr(self.sv), N.ptr(self.phase_u), N.ptr(self.phase_v),
            N.ptr(self.bias), N.ptr(y), N.ptr(ws), ws.numel(), N.stream_of(x2)))
        return y.view(*lead, self.m).to(x.dtype)


def _signs_args(signs):
    if isinstance(signs, IncoherenceSigns) or type(signs).__name__ == "IncoherenceSigns":
        return "rht", dict(su=signs.su, sv=signs.sv)
    if isinstance(signs, RFFTPhases) or type(signs).__name__ == "RFFTPhases":
        return "rfft", dict(phase_u=signs.phase_u, phase_v=signs.phase_v)
    raise TypeError(f"unsupported transform {type(signs).__name__}")


def linear_forward(x: Tensor, layer: QuantizedLayer, codebook) -> Tensor:
    """Algorithm 2: transform_in -> x2 @ What^T -> transform_out, fused on the GPU.
    Packs the codes on every call; `QuantizedLinear` caches the packed stream."""
    m, n = layer.shape
    kind, targs = _signs_args(layer.signs)
    k = LinearKernel(layer.codes, codebook, m, n, layer.scale, kind, **targs)
    return k(x)


def quantize_linear(*_a, **_k):
    raise NotImplementedError("Algorithm 1 (BlockLDLQ quantization) is offline and not provided")
