"""Quantized layers that read one input, run as one group.

A decoder layer's [q_proj, k_proj, v_proj] read the same hidden states, and so
do [gate_proj, up_proj] (the reference groups them the same way in
quipsharp/architectures.py:52-94, get_linear_groups).  Each layer has its own
incoherence signs or phases, so nothing of the input step can be shared; what
a group saves is time.  At decode batches every step of a quantized layer is
latency-bound (a row transform on a few CTAs, a matmul whose tail leaves SMs
idle), and `qs_linear_fwd_group` runs the group's layers on forked streams so
those steps overlap on the GPU instead of following one another.

* `LinearGroup(modules).forward(x)` returns every member's output at once.
* `fuse_linear_groups(model)` links the QuantizedLinear members of every
  [q,k,v] / [gate,up] group of a decoder, so an unmodified model's separate
  calls `q_proj(x)`, `k_proj(x)`, `v_proj(x)` are served by one group call: the
  first call with a given input tensor computes the whole group and the others
  take their outputs from it.  The input is recognised by identity (the group
  holds a reference, so its memory cannot be reused meanwhile) and version
  counter (an in-place change recomputes); tensors made under
  torch.inference_mode carry no version counter and are recognised by
  identity alone.  `unfuse_linear_groups(model)` undoes it.
"""
from __future__ import annotations

import ctypes

import torch
from torch import Tensor, nn

from . import _native as N


def _round_up(v: int, a: int) -> int:
    return (v + a - 1) // a * a


def _version(x: Tensor):
    try:
        return x._version
    except RuntimeError:  # inference tensors keep no version counter
        return None


class LinearGroup:
    """QuantizedLinear modules that read one input (equal in_features)."""

    def __init__(self, modules):
        modules = list(modules)
        if not modules or len(modules) > N.QS_GROUP_MAX_LAYERS:
            raise ValueError(f"a group has 1 to {N.QS_GROUP_MAX_LAYERS} layers, got {len(modules)}")
        if len({m.in_features for m in modules}) != 1:
            raise ValueError("the layers of a group read one input: in_features must agree")
        self.modules = modules
        self.in_features = modules[0].in_features
        self._layers, self._layers_kernels = None, None
        self._pending, self._src, self._src_key = None, None, None

    def _descriptors(self, kernels):
        """The members' qs_linear_layer array, rebuilt when a member rebuilt its
        kernel (the cached kernels are held, so a new one is never mistaken for
        a freed one at the same address)."""
        old = self._layers_kernels
        if old is None or any(a is not b for a, b in zip(old, kernels)):
            arr = (N.LinearLayer * len(kernels))()
            for d, k in zip(arr, kernels):
                d.m, d.packed, d.stages = k.m, N.ptr(k.packed), len(k.kinds)
                d.kinds = ctypes.addressof(k._kinds_c)
                d.stage_scales = None if k._ss_c is None else ctypes.addressof(k._ss_c)
                d.layer_scale, d.transform = N.ptr(k.scale), k.transform
                d.su, d.sv, d.phase_u, d.phase_v = N.ptr(k.su), N.ptr(k.sv), N.ptr(k.phase_u), N.ptr(k.phase_v)
                d.bias = N.ptr(k.bias)
            self._layers, self._layers_kernels = arr, list(kernels)
        return self._layers

    def forward(self, x: Tensor) -> list[Tensor]:
        """Every member's output for x (..., in_features), in member order."""
        N.require_cuda(x)
        if x.device.index != torch.cuda.current_device():  # launch on the device that holds the layers
            with torch.cuda.device(x.device):
                return self.forward(x)
        kernels = [m.kernel() for m in self.modules]
        n = self.in_features
        lead = x.shape[:-1]
        io_dtype = x.dtype if x.dtype in N.IO_DTYPES else torch.float32
        x2 = x.reshape(-1, n).to(io_dtype).contiguous()
        B = x2.shape[0]
        sizes = [_round_up(max(k.workspace_bytes(B), 1), 256) for k in kernels]
        ws = torch.empty(sum(sizes) + 255, dtype=torch.uint8, device=x.device)
        ys = [torch.empty(B, k.m, device=x.device, dtype=io_dtype) for k in kernels]
        tpl = self._descriptors(kernels)
        arr = type(tpl)(*tpl)  # a copy per call: concurrent calls never share output pointers
        off = _round_up(ws.data_ptr(), 256)  # every piece 256-byte aligned, as the library requires
        for d, y, size in zip(arr, ys, sizes):
            d.y, d.workspace, d.workspace_bytes = y.data_ptr(), off, size
            off += size
        N.check(N.lib().qs_linear_fwd_group(N.ptr(x2), N.IO_DTYPES[io_dtype], B, n, len(kernels), arr,
                                            N.stream_of(x2)))
        return [y.view(*lead, k.m).to(x.dtype) for y, k in zip(ys, kernels)]

    __call__ = forward

    def member_forward(self, index: int, x: Tensor) -> Tensor:
        """Member `index`'s output for x, computing the whole group when x is
        not the input of the outputs still waiting to be taken."""
        stream = torch.cuda.current_stream(x.device).cuda_stream if x.is_cuda else None
        key = (_version(x), stream)
        if not (self._pending is not None and self._src is x and self._src_key == key
                and self._pending[index] is not None):
            self._pending = self.forward(x)
            self._src, self._src_key = x, key
        y = self._pending[index]
        self._pending[index] = None
        if all(p is None for p in self._pending):
            self._pending, self._src, self._src_key = None, None, None
        return y


def linear_groups(layer: nn.Module) -> list[list[tuple[str, nn.Module]]]:
    """The QuantizedLinear groups of one decoder layer that share an input:
    [q_proj, k_proj, v_proj] of `self_attn` and [gate_proj, up_proj] of `mlp`
    (the members present; architectures.py:52-94).  Single-member groups are
    left out: they gain nothing."""
    from .checkpoint import QuantizedLinear
    groups = []
    for parent_name, names in (("self_attn", ("q_proj", "k_proj", "v_proj")), ("mlp", ("gate_proj", "up_proj"))):
        parent = getattr(layer, parent_name, None)
        if parent is None:
            continue
        members = [(f"{parent_name}.{n}", getattr(parent, n, None)) for n in names]
        members = [(name, mod) for name, mod in members if isinstance(mod, QuantizedLinear)]
        if len(members) > 1 and len({mod.in_features for _, mod in members}) == 1:
            groups.append(members)
    return groups


def fuse_linear_groups(model: nn.Module) -> int:
    """Link every [q,k,v] / [gate,up] QuantizedLinear group of `model`'s decoder
    layers so their separate calls run as one group call; returns the number of
    groups linked."""
    count = 0
    for module in model.modules():
        for members in linear_groups(module):
            group = LinearGroup([mod for _, mod in members])
            for i, (_, mod) in enumerate(members):
                mod._group, mod._group_index = group, i
            count += 1
    return count


def unfuse_linear_groups(model: nn.Module) -> None:
    from .checkpoint import QuantizedLinear
    for module in model.modules():
        if isinstance(module, QuantizedLinear):
            module._group = None
