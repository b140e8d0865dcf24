"""`QuantizedLinear` on B200 (mirrors quipsharp/checkpoint.py:80-156).

Same constructor, buffers and state_dict keys as the reference module, so a
reference checkpoint's state dict loads unchanged: `codes` int16 (m, n/8) or
(stages, m, n/8), `scale` float32 scalar, `su`/`sv` (RHT) or `phase_u`/`phase_v`
(RFFT, complex64), optional float32 `bias`.  `forward` runs the fused CUDA path:
the int16 codes are re-laid into the kernel's weight stream once and cached
(rebuilt automatically when the `codes` buffer is replaced or modified in place).
"""
from __future__ import annotations

import torch
from torch import nn, Tensor

from . import _native as N
from .incoherence import IncoherenceSigns
from .rfft import RFFTPhases
from .quantize import QuantizedLayer, LinearKernel, RVQCodebookAdapter

MANIFEST_NAME = "quip_config.json"
STATE_NAME = "quantized_state.pt"


def num_rvq_stages(bits: str) -> int:
    """checkpoint.py:56-57."""
    return 1 if bits == "2bit" else 2


class QuantizedLinear(nn.Module):
    """Drop-in quantized nn.Linear (checkpoint.py:80-146)."""

    def __init__(self, in_features: int, out_features: int, g: int, transform_kind: str,
                 num_stages: int = 1, has_bias: bool = False):
        super().__init__()
        assert transform_kind in ("rht", "rfft")
        self.in_features = in_features
        self.out_features = out_features
        self.g = g
        self.transform_kind = transform_kind
        self.num_stages = num_stages
        self.codebook = None
        self.register_buffer("bias", torch.zeros(out_features) if has_bias else None)
        T = in_features // g
        codes_shape = (out_features, T) if num_stages == 1 else (num_stages, out_features, T)
        self.register_buffer("codes", torch.zeros(codes_shape, dtype=torch.int16))
        self.register_buffer("scale", torch.zeros(()))
        if transform_kind == "rht":
            self.register_buffer("su", torch.zeros(out_features))
            self.register_buffer("sv", torch.zeros(in_features))
        else:
            self.register_buffer("phase_u", torch.zeros(out_features // 2, dtype=torch.complex64))
            self.register_buffer("phase_v", torch.zeros(in_features // 2, dtype=torch.complex64))
        self._kernel = None
        self._kernel_key = None

    @classmethod
    def from_quantized_layer(cls, layer: QuantizedLayer, bias: Tensor = None) -> "QuantizedLinear":
        m, n = layer.shape
        kind = "rht" if type(layer.signs).__name__ == "IncoherenceSigns" else "rfft"
        stages = layer.codes.shape[0] if layer.codes.dim() == 3 else 1
        mod = cls(in_features=n, out_features=m, g=layer.g, transform_kind=kind, num_stages=stages,
                  has_bias=bias is not None)
        with torch.no_grad():
            mod.codes.copy_(layer.codes)
            mod.scale.copy_(torch.as_tensor(layer.scale, dtype=torch.float32))
            if bias is not None:
                mod.bias.copy_(bias.float())
            if kind == "rht":
                mod.su.copy_(layer.signs.su)
                mod.sv.copy_(layer.signs.sv)
            else:
                mod.phase_u.copy_(layer.signs.phase_u)
                mod.phase_v.copy_(layer.signs.phase_v)
        return mod

    def _quantized_layer(self) -> QuantizedLayer:
        """checkpoint.py:132-139 (int16 -> int64 & 0xFFFF)."""
        signs = (IncoherenceSigns(su=self.su, sv=self.sv) if self.transform_kind == "rht"
                 else RFFTPhases(phase_u=self.phase_u, phase_v=self.phase_v))
        codes = self.codes.to(torch.int64) & 0xFFFF
        return QuantizedLayer(codes=codes, signs=signs, g=self.g,
                              shape=(self.out_features, self.in_features), scale=self.scale.item())

    def _buffers_key(self):
        bufs = [self.codes, self.scale, self.bias] + (
            [self.su, self.sv] if self.transform_kind == "rht" else [self.phase_u, self.phase_v])
        return (id(self.codebook),) + tuple(
            None if b is None else (b.data_ptr(), b._version, b.device) for b in bufs)

    def kernel(self) -> LinearKernel:
        """The resolved fused-forward state (packed weights etc.), rebuilt when
        a buffer or the codebook changed."""
        if self.codebook is None:
            raise RuntimeError("QuantizedLinear.codebook must be assigned before forward")
        key = self._buffers_key()
        if self._kernel is None or key != self._kernel_key:
            targs = (dict(su=self.su, sv=self.sv) if self.transform_kind == "rht"
                     else dict(phase_u=self.phase_u, phase_v=self.phase_v))
            with torch.no_grad():
                self._kernel = LinearKernel(self.codes, self.codebook, self.out_features,
                                            self.in_features, self.scale, self.transform_kind,
                                            bias=self.bias, **targs)
            self._kernel_key = key
        return self._kernel

    def forward(self, x: Tensor) -> Tensor:
        return self.kernel()(x)


def replace_with_quantized_linear_(parent: nn.Module, attr: str, layer: QuantizedLayer,
                                   codebook, bias: Tensor = None) -> QuantizedLinear:
    """checkpoint.py:149-156."""
    qlin = QuantizedLinear.from_quantized_layer(layer, bias=bias)
    qlin.codebook = codebook
    setattr(parent, attr, qlin)
    return qlin
