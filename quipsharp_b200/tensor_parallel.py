"""Column-sharded tensor parallelism for `QuantizedLinear` (one process per GPU).

Rank r of P holds weight rows [r*m/P, (r+1)*m/P) (its slice of `codes`); the
input transform runs on the full activations on every rank.  Each rank's fused
decode+matmul writes its float32 y1 shard (B, m/P); NCCL all-gathers the
shards over NVLink into the rank-major buffer (P, B, m/P); the output transform
kernel reads that layout directly (element (b, c) at
((c // (m/P)) * B + b) * (m/P) + c % (m/P)), applies the full-width Hadamard /
IFFT, the row signs / conjugate phases and the bias, and every rank ends with
the full output, ready for the next layer.

The reference has no tensor parallelism (it places whole decoder layers on
devices with accelerate); this is the scale-out path for layers that do not
fit or are too slow on one B200.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn, Tensor

from . import _native as N
from .quantize import LinearKernel


def shard_rows(m: int, world: int, rank: int) -> tuple[int, int]:
    """Row range of `rank` for a column-sharded layer with m outputs."""
    if m % world:
        raise ValueError(f"out_features {m} is not divisible by world size {world}")
    mp = m // world
    return rank * mp, (rank + 1) * mp


def gathered_offset(b: int, c: int, batch: int, m: int, world: int) -> int:
    """Position of y1[b, c] in the all-gathered rank-major buffer (the index
    function the output-transform kernel uses)."""
    mp = m // world
    return ((c // mp) * batch + b) * mp + c % mp


class TPQuantizedLinear(nn.Module):
    """Tensor-parallel forward of a full `QuantizedLinear` (same output on every rank)."""

    def __init__(self, full, group=None):
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        m, n = full.out_features, full.in_features
        if full.transform_kind == "rfft" and (m // self.world) % 2:
            raise ValueError("RFFT layers need an even number of output columns per rank")
        lo, hi = shard_rows(m, self.world, self.rank)
        self.m, self.n, self.mp = m, n, hi - lo
        codes = full.codes[..., lo:hi, :].contiguous()
        targs = (dict(sv=full.sv) if full.transform_kind == "rht" else dict(phase_v=full.phase_v))
        self.local = LinearKernel(codes, full.codebook, self.mp, n, full.scale, full.transform_kind, **targs)
        dev = codes.device
        self.transform = self.local.transform
        self.su = None if full.transform_kind != "rht" else full.su.to(dev, torch.float32).contiguous()
        self.phase_u = None if full.transform_kind != "rfft" else torch.view_as_real(
            full.phase_u.to(dev, torch.complex64).contiguous())
        self.bias = None if full.bias is None else full.bias.to(dev, torch.float32).contiguous()

    def forward(self, x: Tensor) -> Tensor:
        N.require_cuda(x)
        lead = x.shape[:-1]
        io_dtype = x.dtype if x.dtype in N.IO_DTYPES else torch.float32
        x2 = x.reshape(-1, self.n).to(io_dtype).contiguous()
        B = x2.shape[0]
        y1_local = torch.empty(B, self.mp, dtype=torch.float32, device=x.device)
        ws = self.local.input(x2, y1_local)
        self.local.matmul(ws, B, y1_local)
        gathered = torch.empty(self.world * B * self.mp, dtype=torch.float32, device=x.device)
        dist.all_gather_into_tensor(gathered, y1_local.reshape(-1), group=self.group)
        y = torch.empty(B, self.m, dtype=io_dtype, device=x.device)
        N.check(N.lib().qs_linear_output(N.ptr(gathered), 0, self.world, B, self.m, self.transform,
                                         N.ptr(self.su), N.ptr(self.phase_u), N.ptr(self.bias), N.ptr(y),
                                         N.IO_DTYPES[io_dtype], N.stream_of(y)))
        return y.view(*lead, self.m).to(x.dtype)
