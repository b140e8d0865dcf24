"""Device-side failure detection of the pipelined kernels, without a GPU fault.

Every mbarrier wait between the warps of the tcgen05 prefill GEMM is bounded; a wait
that runs out ends the kernel early (after draining its own copies and
tensor-core work in flight) and sets a device flag that qs_device_status turns
into QS_ERR_TIMEOUT.  Here the limit is lowered to 1 ns so that the first wait
that is not already satisfied gives up: the status must come back as
QS_ERR_TIMEOUT, the flag must be cleared by that read, and with the default
limit restored the next call must succeed with a correct result."""
import pytest
import torch

from quipsharp_b200 import _native as N
from quipsharp_b200 import synthetic as syn
from conftest import rel_l2
from test_gpu_linear import make_module, oracle_y, TOL

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("m,n,kinds,B", [
    (512, 1024, (syn.E8P,), 600),                 # persistent GEMM, 3 tiles per CTA on a short grid
    (256, 512, (syn.E8P, syn.E8_1BIT), 300),      # RVQ GEMM, one tile per CTA
])
def test_short_wait_limit_reports_timeout_then_recovers(m, n, kinds, B):
    lay = syn.make_layer(m, n, kinds, seed=3, transform_kind="rht")
    mod = make_module(lay)
    x = syn.make_activations(B, n, dtype=torch.float16, seed=4).to(DEV)
    lib = N.lib()
    default = lib.qs_wait_limit_ns()
    assert default == 4_000_000_000
    mod(x)  # pack and warm up with the default limit
    torch.cuda.synchronize()
    assert lib.qs_device_status(N.stream_of(x)) == N.QS_OK
    try:
        assert lib.qs_set_wait_limit_ns(1) == N.QS_OK
        assert lib.qs_wait_limit_ns() == 1
        mod(x)
        torch.cuda.synchronize()
        assert lib.qs_device_status(N.stream_of(x)) == N.QS_ERR_TIMEOUT
        assert b"timed out" in lib.qs_last_error()
        # the read cleared the flag
        assert lib.qs_device_status(N.stream_of(x)) == N.QS_OK
    finally:
        lib.qs_set_wait_limit_ns(0)
    assert lib.qs_wait_limit_ns() == default
    y = mod(x)
    torch.cuda.synchronize()
    assert lib.qs_device_status(N.stream_of(x)) == N.QS_OK
    assert rel_l2(y.float().cpu().numpy(), oracle_y(lay, x.cpu())) < TOL[torch.float16]
