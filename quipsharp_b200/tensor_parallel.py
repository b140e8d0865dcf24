"""Column-sharded tensor parallelism for `QuantizedLinear` (one process per GPU).

Rank r of P holds weight rows [r*m/P, (r+1)*m/P) (its slice of `codes`).  A
forward runs, on every rank, the input transform of the full activations, the
fused decode + matmul of the local rows into a private float32 y1 shard, a push
of the shard into every rank's receive buffer over NVLink (decode batches: by
every CTA of the matmul after a grid barrier, as 8-byte words that carry the
call's sequence number, so no fence or flag is needed; prefill batches: a push
kernel, then a flag in every rank's memory), and the output transform, which
reads the gathered y1 locally once it has arrived (no collective library call on
the data path).  Every rank ends with the full output, ready for the next layer.
Layers are not grouped across streams here (groups.py): the decode matmul's grid
barrier needs every CTA of its grid resident.

The receive buffers and flags live in a `TPContext` per (process group,
device): allocated once, shared with the peers through CUDA IPC handles
exchanged over the process group.  Which of a buffer's two regions a call uses
follows a call counter kept on the device, so forwards captured in CUDA graphs
replay in any mix with eager ones (every rank must run the same sequence).  The
reference has no tensor parallelism (it places whole decoder layers on devices
with accelerate); this is the scale-out path for one layer.
"""
from __future__ import annotations

import ctypes

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
    """Position of y1[b, c] in the rank-major layout of `world` gathered shards
    ((rank, b, c % (m/world)): qs_linear_output with shards = world)."""
    mp = m // world
    return ((c // mp) * batch + b) * mp + c % mp


def exchange_floats(capacity: int, world: int) -> int:
    """float32 elements of one rank's exchange allocation: receive regions
    [2][capacity], flags [2][world] (int32, padded to 4 entries) and four uint32
    control words (16-byte aligned: capacity is a multiple of 4)."""
    return ctl_offset(capacity, world) + 4


def ctl_offset(capacity: int, world: int) -> int:
    """float32 index of the control words in an exchange allocation."""
    return 2 * capacity + (2 * world + 3) // 4 * 4


def make_peers(world: int, rank: int, bases: list[int], capacity: int) -> "N.TPPeers":
    """qs_tp_peers over exchange allocations laid out as `exchange_floats`
    describes: bases[r] is rank r's allocation as mapped in this process
    (bases[rank] is this rank's own)."""
    peers = N.TPPeers()
    peers.world, peers.rank, peers.recv_floats = world, rank, capacity
    for r, base in enumerate(bases):
        peers.recv[r] = base
        peers.flags[r] = base + 2 * capacity * 4
    peers.ctl = bases[rank] + ctl_offset(capacity, world) * 4
    return peers


class TPContext:
    """Peer-memory exchange buffers of one process group on one device."""

    _contexts: dict = {}

    @classmethod
    def get(cls, group, device) -> "TPContext":
        key = (group, torch.device(device).index)
        ctx = cls._contexts.get(key)
        if ctx is None:
            ctx = cls._contexts[key] = cls(group, torch.device(device))
        return ctx

    def __init__(self, group, device):
        self.group, self.device = group, device
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > N.QS_TP_MAX_RANKS:
            raise ValueError(f"at most {N.QS_TP_MAX_RANKS} ranks")
        self.capacity = 0  # floats per receive region (batch * m of the largest call)
        self.peers = None
        self._imported = []
        self._buffers = None

    def ensure(self, floats: int) -> None:
        """Receive regions of at least `floats` floats on every rank (collective when
        it grows: every rank makes the same calls in the same order)."""
        if floats <= self.capacity:
            return
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("tensor-parallel exchange buffers must grow outside CUDA graph capture "
                               "(run one eager forward of the largest batch first)")
        cap = (max(floats, 2 * self.capacity, 1 << 16) + 3) // 4 * 4
        self.release()
        # one allocation (one IPC handle): receive regions [2][cap] float32, flags
        # [2][world] int32, then this rank's two uint32 control words
        buf = torch.zeros(exchange_floats(cap, self.world), dtype=torch.float32, device=self.device)
        h = ctypes.create_string_buffer(64)
        off = ctypes.c_int64(0)
        N.check(N.lib().qs_ipc_export(buf.data_ptr(), h, ctypes.addressof(off)))
        every = [None] * self.world
        dist.all_gather_object(every, (h.raw, off.value), group=self.group)
        bases = []
        for r, (hr, orr) in enumerate(every):
            if r == self.rank:
                bases.append(buf.data_ptr())
            else:
                p = ctypes.c_void_p()
                N.check(N.lib().qs_ipc_import(hr, orr, ctypes.addressof(p)))
                self._imported.append((p.value, orr))
                bases.append(p.value)
        self._buffers, self.capacity = buf, cap
        self.peers = make_peers(self.world, self.rank, bases, cap)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def release(self) -> None:
        """Unmap the peers' buffers and drop this rank's (collective)."""
        if self.peers is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for ptr, off in self._imported:
            N.lib().qs_ipc_close(ptr, off)
        self._imported, self._buffers, self.peers, self.capacity = [], None, None, 0
        dist.barrier(group=self.group)


class TPQuantizedLinear(nn.Module):
    """Tensor-parallel forward of a full `QuantizedLinear` (same output on every rank)."""

    def __init__(self, full, group=None):
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        m, n = full.out_features, full.in_features
        if self.world > N.QS_TP_MAX_RANKS:
            raise ValueError(f"at most {N.QS_TP_MAX_RANKS} ranks")
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
        self.ctx = TPContext.get(group, dev)

    def forward(self, x: Tensor) -> Tensor:
        N.require_cuda(x)
        lead = x.shape[:-1]
        io_dtype = x.dtype if x.dtype in N.IO_DTYPES else torch.float32
        x2 = x.reshape(-1, self.n).to(io_dtype).contiguous()
        B = x2.shape[0]
        y = torch.empty(B, self.m, dtype=io_dtype, device=x.device)
        if B == 0:
            return y.view(*lead, self.m).to(x.dtype)
        # decode batches exchange 8-byte self-validating words, prefill batches floats
        self.ctx.ensure(B * self.m * (2 if B <= 32 else 1))
        nb = N.lib().qs_linear_tp_workspace_bytes(B, self.n, self.mp)
        ws = torch.empty(nb, dtype=torch.uint8, device=x.device)
        k = self.local
        N.check(N.lib().qs_linear_fwd_tp(
            N.ptr(x2), N.IO_DTYPES[io_dtype], B, self.n, self.m, N.ptr(k.packed), len(k.kinds), k._kinds_c,
            k._ss_c, N.ptr(k.scale), self.transform, N.ptr(self.su), N.ptr(k.sv), N.ptr(self.phase_u),
            N.ptr(k.phase_v), N.ptr(self.bias), N.ptr(y), N.ptr(ws), ws.numel(),
            ctypes.addressof(self.ctx.peers), N.stream_of(x2)))
        return y.view(*lead, self.m).to(x.dtype)
