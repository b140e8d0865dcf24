"""The output step's shard-aware layout on one GPU.

Column-sharded tensor parallelism all-gathers each rank's float32 y1 shard
(batch, m/P) into a rank-major buffer (P, batch, m/P), which qs_linear_output
reads in place (shards = P).  Here the full y1 of one layer is computed once on
one GPU, laid out exactly as all_gather_into_tensor would lay out P shards, and
the shard-aware output step must give the same result as the unsharded one,
for the Hadamard (RHT) and FFT (RFFT) output transforms, few and many rows."""
import pytest
import torch

from quipsharp_b200 import _native as N
from quipsharp_b200 import synthetic as syn
from quipsharp_b200.tensor_parallel import gathered_offset
from conftest import rel_l2
from test_gpu_linear import make_module, TOL

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _y1(mod, x):
    """y1 = x2 @ What^T of the whole layer (input step + matmul)."""
    k = mod.kernel()
    B = x.shape[0]
    y1 = torch.empty(B, k.m, dtype=torch.float32, device=DEV)
    ws = k.input(x, y1)
    k.matmul(ws, B, y1)
    return y1


def _output(mod, y1_buf, shards, B, dt):
    k = mod.kernel()
    y = torch.empty(B, k.m, dtype=dt, device=DEV)
    N.check(N.lib().qs_linear_output(N.ptr(y1_buf), k.m, shards, B, k.m, k.transform, N.ptr(k.su),
                                     N.ptr(k.phase_u), N.ptr(k.bias), N.ptr(y), N.IO_DTYPES[dt], N.stream_of(y)))
    return y


@pytest.mark.parametrize("m,n,transform,B,dt", [
    (4096, 1024, "rht", 1, torch.float16),
    (4096, 1024, "rht", 64, torch.bfloat16),
    (11008, 1024, "rfft", 3, torch.float16),     # 5504-point IFFT (43 x 128)
    (28672, 512, "rfft", 2, torch.bfloat16),    # 14336-point IFFT (7 x 2048), config-5 gate width
    (2048, 512, "rfft", 40, torch.float32),
])
@pytest.mark.parametrize("P", [2, 4, 8])
def test_rank_major_gathered_layout_matches_unsharded(m, n, transform, B, dt, P):
    if transform == "rfft" and (m // P) % 2:
        pytest.skip("RFFT shards need an even number of columns")
    lay = syn.make_layer(m, n, (syn.E8P,), seed=m + P, transform_kind=transform, has_bias=True)
    mod = make_module(lay)
    x = syn.make_activations(B, n, dtype=dt, seed=B).to(DEV)
    y1 = _y1(mod, x)
    mp = m // P
    # rank-major buffer of P gathered shards: (P, B, m/P)
    gathered = y1.reshape(B, P, mp).permute(1, 0, 2).contiguous().reshape(-1)
    # the index rule the kernels use
    b, c = B - 1, m - 3
    assert gathered[gathered_offset(b, c, B, m, P)].item() == y1[b, c].item()
    y_ref = _output(mod, y1.clone(), 1, B, dt)
    y_tp = _output(mod, gathered, P, B, dt)
    torch.cuda.synchronize()
    assert rel_l2(y_tp.float().cpu().numpy(), y_ref.float().cpu().numpy()) < TOL[dt] / 4
