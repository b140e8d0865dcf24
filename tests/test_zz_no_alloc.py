"""qs_linear_fwd_noalloc: the layer forward for callers that cannot allocate
device memory.

Some hosts give all device memory to their own allocator up front (serving
engines that reserve HBM for their caches, plugin hosts with a fixed budget),
or cannot afford cudaMalloc's implicit device synchronisation inside their
loop; they cannot hand qs_linear_fwd a workspace.  The no-alloc entry point
uses a built-in 8 MiB device array instead.  These tests call it through the C
ABI and check it against qs_linear_fwd (same kernels, caller workspace), twice
in a row with different inputs (the shared array keeps the previous call's
contents, which must not leak into the next result), and check that a batch
whose workspace exceeds the array is refused with a clear error.

Kept in a file pytest collects last, so a failure here cannot stop the rest of
the suite from running first."""
import numpy as np
import pytest
import torch

from quipsharp_b200 import _native as N
from quipsharp_b200 import synthetic as syn
from quipsharp_b200.checkpoint import QuantizedLinear
from quipsharp_b200.codebooks import E8PCodebook, E8OneBitCodebook
from quipsharp_b200.quantize import RVQCodebookAdapter
from quipsharp_b200.rvq import RVQStage

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_l2(a, b):
    a = a.double()
    b = b.double()
    return float((a - b).norm() / b.norm())


def _layer(m, n, kinds, seed):
    lay = syn.make_layer(m, n, kinds, seed=seed, has_bias=True)
    mod = QuantizedLinear(n, m, 8, lay.transform_kind, num_stages=len(kinds), has_bias=True)
    with torch.no_grad():
        mod.codes.copy_(lay.codes)
        mod.scale.copy_(torch.tensor(lay.layer_scale))
        if lay.transform_kind == "rht":
            mod.su.copy_(lay.su)
            mod.sv.copy_(lay.sv)
        else:
            mod.phase_u.copy_(lay.phase_u)
            mod.phase_v.copy_(lay.phase_v)
        mod.bias.copy_(lay.bias)
    cb = lambda k: E8PCodebook() if k == syn.E8P else E8OneBitCodebook()
    mod.codebook = cb(kinds[0]) if len(kinds) == 1 else RVQCodebookAdapter(
        [RVQStage(cb(k), s) for k, s in zip(kinds, lay.stage_scales)])
    return mod.to(DEV).kernel()


def _forward(k, x, noalloc):
    B = x.shape[0]
    y = torch.empty(B, k.m, dtype=x.dtype, device=DEV)
    args = [N.ptr(x), N.IO_DTYPES[x.dtype], B, k.n, k.m, N.ptr(k.packed), len(k.kinds), k._kinds_c,
            k._ss_c, N.ptr(k.scale), k.transform, N.ptr(k.su), N.ptr(k.sv), N.ptr(k.phase_u),
            N.ptr(k.phase_v), N.ptr(k.bias), N.ptr(y)]
    if noalloc:
        st = N.lib().qs_linear_fwd_noalloc(*args, N.stream_of(x))
    else:
        ws = torch.empty(k.workspace_bytes(B), dtype=torch.uint8, device=DEV)
        st = N.lib().qs_linear_fwd(*args, N.ptr(ws), ws.numel(), N.stream_of(x))
    N.check(st)
    return y


@pytest.mark.parametrize("m,n,kinds,dtype", [
    (11008, 4096, (syn.E8P, syn.E8_1BIT), torch.float16),   # benchmark layer, RFFT both sides
    (4096, 4096, (syn.E8P,), torch.bfloat16),                # RHT layer
])
def test_noalloc_matches_workspace_entry_point_twice(m, n, kinds, dtype):
    k = _layer(m, n, kinds, seed=m + n)
    tol = 2e-3 if dtype == torch.float16 else 1e-2
    for call, B in enumerate((8, 3)):  # two calls in a row, different inputs
        x = syn.make_activations(B, n, dtype=dtype, seed=100 + call).to(DEV)
        want = _forward(k, x, noalloc=False)
        got = _forward(k, x, noalloc=True)
        torch.cuda.synchronize()
        assert got.dtype == dtype and got.shape == (B, m)
        assert rel_l2(got.float(), want.float()) < tol


def test_noalloc_rejects_batches_beyond_the_builtin_workspace():
    k = _layer(4096, 4096, (syn.E8P,), seed=1)
    x = torch.zeros(1024, 4096, dtype=torch.float16, device=DEV)  # needs ~24 MiB of workspace
    y = torch.empty(1024, 4096, dtype=torch.float16, device=DEV)
    st = N.lib().qs_linear_fwd_noalloc(
        N.ptr(x), N.QS_F16, 1024, 4096, 4096, N.ptr(k.packed), 1, k._kinds_c, k._ss_c, N.ptr(k.scale),
        k.transform, N.ptr(k.su), N.ptr(k.sv), None, None, N.ptr(k.bias), N.ptr(y), N.stream_of(x))
    assert st == N.QS_ERR_WORKSPACE
    assert b"workspace" in N.lib().qs_last_error()
