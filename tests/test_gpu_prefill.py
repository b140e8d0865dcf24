"""GPU parity of the prefill matmul (fused decode + tcgen05 GEMM, batches of
33 tokens and more) through the public module, against the CPU oracle.

Same tolerance as the decode-regime tests (relative L2 against the float32
oracle: 1e-3 fp32 out, 2e-3 fp16 out, 1e-2 bf16 out): the weights are exact in
fp16, activations are rounded to fp16 once, accumulation is float32 in TMEM."""
import pytest
import torch

from quipsharp_b200 import _native as N
from quipsharp_b200 import synthetic as syn
from conftest import rel_l2
from test_gpu_linear import make_module, oracle_y, TOL

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("m,n,kinds,B,dt", [
    (384, 512, (syn.E8P,), 300, torch.bfloat16),                   # RFFT both sides, ragged token tile
    (256, 1024, (syn.E8P,), 2048, torch.bfloat16),                 # RHT, 8 token tiles
    (200, 256, (syn.E8P, syn.E8_1BIT), 100, torch.float16),        # 3-bit RVQ, ragged row tile
    (128, 256, (syn.E8P, syn.E8P), 33, torch.float32),             # 4-bit RVQ at the threshold batch
    (1792, 3584, (syn.E8P,), 64, torch.bfloat16),                  # Qwen2.5-7B hidden width
])
def test_prefill_matmul_vs_oracle(m, n, kinds, B, dt):
    lay = syn.make_layer(m, n, kinds, seed=m * 7 + n + B, has_bias=True)
    x = syn.make_activations(B, n, dtype=dt, seed=B + 3)
    y = make_module(lay)(x.to(DEV))
    torch.cuda.synchronize()
    N.check(N.lib().qs_device_status(N.stream_of(y)))
    assert y.shape == (B, m) and y.dtype == dt
    assert rel_l2(y.float().cpu().numpy(), oracle_y(lay, x)) < TOL[dt]


# Many rows of RFFT layers whose half-width N = P * 2^a (P an odd prime) is at
# least 4096: the input / output transforms run in two passes (per-column P-point
# DFTs, then per-block power-of-two FFTs with a warp (N1 <= 512) or the whole
# CTA (N1 > 512) per block).
@pytest.mark.parametrize("m,n,kinds,B,dt", [
    (11008, 1024, (syn.E8P,), 100, torch.bfloat16),               # output 5504 = 43 * 128 (warp blocks)
    (512, 11008, (syn.E8P, syn.E8_1BIT), 96, torch.float16),      # input 5504 (warp blocks), RVQ
    (14336, 256, (syn.E8P,), 80, torch.float32),                  # output 7168 = 7 * 1024 (CTA blocks), fp32 out
    (256, 14336, (syn.E8P,), 77, torch.bfloat16),                 # input 7168 (CTA blocks)
    (14336, 256, (syn.E8P,), 40, torch.float16),                  # GEMM batch, few rows: spread two-pass output
    (256, 14336, (syn.E8P, syn.E8_1BIT), 48, torch.bfloat16),     # GEMM batch, few rows: spread two-pass input
])
def test_prefill_two_pass_transforms_vs_oracle(m, n, kinds, B, dt):
    lay = syn.make_layer(m, n, kinds, seed=m + 3 * n + B, transform_kind="rfft", has_bias=True)
    x = syn.make_activations(B, n, dtype=dt, seed=B + 7)
    y = make_module(lay)(x.to(DEV))
    torch.cuda.synchronize()
    N.check(N.lib().qs_device_status(N.stream_of(y)))
    assert y.shape == (B, m) and y.dtype == dt
    assert rel_l2(y.float().cpu().numpy(), oracle_y(lay, x)) < TOL[dt]
    # the same rows through the few-row (one-pass) transforms agree
    y_few = make_module(lay)(x[:8].to(DEV))
    assert rel_l2(y[:8].float().cpu().numpy(), y_few.float().cpu().numpy()) < TOL[dt]


def test_prefill_and_decode_paths_agree():
    """The same layer through the decode-regime kernel (32 tokens: two passes
    of 16) and the prefill GEMM (33 tokens): the shared 32 rows agree."""
    lay = syn.make_layer(512, 1024, (syn.E8P, syn.E8_1BIT), seed=42)
    mod = make_module(lay)
    x = syn.make_activations(33, 1024, dtype=torch.float16, seed=5).to(DEV)
    y_tc = mod(x)[:32].float()
    y_mma = mod(x[:32]).float()
    assert rel_l2(y_tc.cpu().numpy(), y_mma.cpu().numpy()) < 2e-3


# Grids with more output tiles than SMs.  One-stage codebooks run the persistent
# GEMM (one CTA per SM looping over tiles): several tiles per CTA exercise the
# second TMEM accumulator, the accumulator-empty handshake and the ring phases
# that carry over from tile to tile.  Two-stage RVQ runs one tile per CTA over
# a grid far larger than the GPU.  The whole batch runs on the GPU; a seeded
# subset of token rows is compared with the oracle (rows are independent).
@pytest.mark.parametrize("m,n,kinds,B,dt,transform", [
    (18944, 3584, (syn.E8P,), 2048, torch.bfloat16, "rfft"),    # config-4 gate: 1184 tiles, 8 per CTA
    (4096, 256, (syn.E8P,), 2567, torch.float16, "rht"),        # 352 tiles (2-3 per CTA), ragged token tile
    (8192, 8192, (syn.E8P, syn.E8_1BIT), 4096, torch.bfloat16, "rht"),  # config-5 q, RVQ-3bit: 1024 CTAs
])
def test_prefill_multi_tile_grid_vs_oracle(m, n, kinds, B, dt, transform):
    lay = syn.make_layer(m, n, kinds, seed=m + n + B, transform_kind=transform, has_bias=True)
    x = syn.make_activations(B, n, dtype=dt, seed=B + 11)
    y = make_module(lay)(x.to(DEV))
    torch.cuda.synchronize()
    N.check(N.lib().qs_device_status(N.stream_of(y)))
    assert y.shape == (B, m) and y.dtype == dt
    g = torch.Generator().manual_seed(B)
    rows = torch.randperm(B, generator=g)[:48].sort().values
    rows = torch.cat([rows, torch.tensor([0, B - 1])])  # first and last (ragged) token tile too
    got = y[rows.to(DEV)].float().cpu().numpy()
    assert rel_l2(got, oracle_y(lay, x[rows])) < TOL[dt]
    assert torch.isfinite(y).all()
