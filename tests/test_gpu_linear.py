"""GPU parity of the fused quantized-linear forward (input transform ->
decode+matmul -> output transform) against the oracle and the reference's
golden outputs.

Tolerance (relative L2 against the float32 oracle before the output cast):
the matmul rounds the transformed activations x2 to fp16 (weights are exact
in fp16, accumulation is float32), which costs ~1.5e-4; the final cast to the
caller's dtype adds at most half an ulp.  Bounds: 1e-3 for float32 outputs,
2e-3 for float16 outputs, 1e-2 for bfloat16 outputs."""
import numpy as np
import pytest
import torch

from oracle import quipsharp_oracle as O
from quipsharp_b200 import synthetic as syn
from conftest import rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = {torch.float32: 1e-3, torch.float16: 2e-3, torch.bfloat16: 1e-2}


def make_module(lay, device=DEV):
    from quipsharp_b200.checkpoint import QuantizedLinear
    from quipsharp_b200.codebooks import E8PCodebook, E8OneBitCodebook
    from quipsharp_b200.quantize import RVQCodebookAdapter
    from quipsharp_b200.rvq import RVQStage
    mod = QuantizedLinear(lay.n, lay.m, 8, lay.transform_kind, num_stages=lay.num_stages,
                          has_bias=lay.bias is not None)
    with torch.no_grad():
        mod.codes.copy_(lay.codes)
        mod.scale.copy_(torch.tensor(lay.layer_scale))
        if lay.transform_kind == "rht":
            mod.su.copy_(lay.su)
            mod.sv.copy_(lay.sv)
        else:
            mod.phase_u.copy_(lay.phase_u)
            mod.phase_v.copy_(lay.phase_v)
        if lay.bias is not None:
            mod.bias.copy_(lay.bias)
    cb = lambda k: E8PCodebook() if k == syn.E8P else E8OneBitCodebook()
    mod.codebook = cb(lay.kinds[0]) if lay.num_stages == 1 else RVQCodebookAdapter(
        [RVQStage(cb(k), s) for k, s in zip(lay.kinds, lay.stage_scales)])
    return mod.to(device)


def oracle_y(lay, x):
    ss = None if lay.num_stages == 1 else list(lay.stage_scales)
    t = lambda v: None if v is None else v.numpy()
    return O.linear_forward(x.float().numpy(), lay.codes.numpy(), list(lay.kinds), ss, lay.layer_scale,
                            lay.transform_kind, su=t(lay.su), sv=t(lay.sv), phase_u=t(lay.phase_u),
                            phase_v=t(lay.phase_v), bias=t(lay.bias))


FORWARD_CASES = ["fw_e8p_rht_f32_bias", "fw_e8p_rht_f16", "fw_e8p_rht_bf16", "fw_rvq3_rfft_bf16_bias",
                 "fw_e8p_rfft_f32", "fw_rvq4_rht_f16", "fw_rvq3_rht_f32", "fw_e8p_rfft_f16_odd"]


@pytest.mark.parametrize("name", FORWARD_CASES)
def test_forward_small_layers_vs_reference(golden, name):
    m, n, lseed, xseed, B, bias = (int(v) for v in golden[name + "_meta"])
    kinds = tuple(str(k) for k in golden[name + "_kinds"])
    dt = getattr(torch, str(golden[name + "_dtype"]))
    lay = syn.make_layer(m, n, kinds, seed=lseed, has_bias=bool(bias))
    x = syn.make_activations(B, n, dtype=dt, seed=xseed)
    y = make_module(lay)(x.to(DEV))
    assert y.dtype == dt and y.shape == (B, m)
    assert rel_l2(y.float().cpu().numpy(), oracle_y(lay, x)) < TOL[dt]
    assert rel_l2(y.float().cpu().numpy(), golden[name + "_y"]) < TOL[dt]


@pytest.mark.parametrize("cfg", ["c1", "c2"])
def test_forward_config_shapes_vs_reference(golden_configs, cfg):
    m, n, lseed, xseed, B = (int(v) for v in golden_configs[cfg + "_meta"])
    kinds = (syn.E8P,) if cfg == "c1" else (syn.E8P, syn.E8_1BIT)
    lay = syn.make_layer(m, n, kinds, seed=lseed)
    x = syn.make_activations(B, n, dtype=torch.float16, seed=xseed)
    mod = make_module(lay)
    y = mod(x.to(DEV)).float().cpu().numpy()
    assert rel_l2(y, golden_configs[cfg + "_y"]) < 2e-3
    # every token row independently (batch 1 and batch B give the same rows)
    y1 = mod(x[:1].to(DEV)).float().cpu().numpy()
    assert rel_l2(y1, y[:1]) < 1e-3


@pytest.mark.parametrize("m,n,kinds,B,dt", [
    (11008, 4096, (syn.E8P, syn.E8_1BIT), 32, torch.float16),     # config 2, batch 32
    (1024, 4096, (syn.E8P,), 16, torch.bfloat16),                 # Llama-3-8B k/v, batch 16
    (4096, 14336, (syn.E8P,), 3, torch.bfloat16),                 # Llama-3-8B down (RFFT 7168 in)
    (18944, 3584, (syn.E8P,), 2, torch.bfloat16),                 # Qwen2.5-7B gate (RFFT 9472 out)
    (8192, 28672, (syn.E8P, syn.E8_1BIT), 1, torch.bfloat16),     # Llama-3-70B down (14336 in)
    (256, 512, (syn.E8P, syn.E8P), 5, torch.float32),             # 4-bit RVQ
    (40, 24, (syn.E8P,), 9, torch.float16),                       # ragged: m, n not tile multiples
    (2048, 1024, (syn.E8P, syn.E8_1BIT), 12, torch.float16),      # 3-bit RVQ, 9..16 tokens in one pass
    (512, 1024, (syn.E8_1BIT, syn.E8P), 11, torch.bfloat16),      # 1-bit first stage, one pass
    (384, 512, (syn.E8P, syn.E8P), 16, torch.float32),            # 4-bit RVQ at the one-pass limit
    (11008, 1024, (syn.E8P,), 1, torch.float32),                  # output 5504 = 43 x 128: warp-per-column pass A
    (4096, 11008, (syn.E8P, syn.E8_1BIT), 4, torch.float16),      # input 5504: warp-per-column pass A + L1 scale
    (3584, 18944, (syn.E8P,), 2, torch.bfloat16),                 # input 9472 = 37 x 256
    (640, 2048, (syn.E8P,), 17, torch.float16),                   # 32 token columns, one stage
    (300, 768, (syn.E8_1BIT, syn.E8_1BIT), 24, torch.bfloat16),   # ragged rows, 1-bit stages, 32 columns
    (8192, 8192, (syn.E8P, syn.E8_1BIT), 1, torch.bfloat16),      # Llama-3-70B q: chunk ranges cross row tiles
    (1024, 8192, (syn.E8P, syn.E8_1BIT), 2, torch.bfloat16),      # Llama-3-70B k: few chunks per CTA
    (128, 256, (syn.E8P,), 1, torch.float32),                     # fewer chunks than SMs
])
def test_forward_shapes_vs_oracle(m, n, kinds, B, dt):
    lay = syn.make_layer(m, n, kinds, seed=m + n + B, has_bias=True)
    x = syn.make_activations(B, n, dtype=dt, seed=B)
    y = make_module(lay)(x.to(DEV))
    assert rel_l2(y.float().cpu().numpy(), oracle_y(lay, x)) < TOL[dt]


def test_forward_leading_dims_and_large_activations():
    lay = syn.make_layer(64, 128, (syn.E8P,), seed=3)
    mod = make_module(lay)
    x = syn.make_activations(6, 128, dtype=torch.float32, seed=4).reshape(2, 3, 128) * 3.0e4
    y = mod(x.to(DEV))
    assert y.shape == (2, 3, 64)
    assert rel_l2(y.cpu().numpy().reshape(6, 64), oracle_y(lay, x.reshape(6, 128))) < 1e-3


def test_forward_empty_batch_and_cache_invalidation():
    lay = syn.make_layer(64, 128, (syn.E8P,), seed=5)
    mod = make_module(lay)
    assert mod(torch.empty(0, 128, device=DEV, dtype=torch.float16)).shape == (0, 64)
    x = syn.make_activations(2, 128, dtype=torch.float32, seed=6)
    y0 = mod(x.to(DEV)).cpu()
    lay2 = syn.make_layer(64, 128, (syn.E8P,), seed=7)
    with torch.no_grad():
        mod.codes.copy_(lay2.codes.to(DEV))     # in-place update must invalidate the packed cache
    lay2.su, lay2.sv, lay2.layer_scale = lay.su, lay.sv, lay.layer_scale
    y1 = mod(x.to(DEV)).cpu().numpy()
    assert rel_l2(y1, oracle_y(lay2, x)) < 1e-3
    assert rel_l2(y1, y0.numpy()) > 0.1


def test_state_dict_round_trip_and_functional_path():
    from quipsharp_b200.checkpoint import QuantizedLinear
    from quipsharp_b200.quantize import linear_forward
    lay = syn.make_layer(48, 144, (syn.E8P, syn.E8_1BIT), seed=8, has_bias=True)
    mod = make_module(lay)
    x = syn.make_activations(4, 144, dtype=torch.float32, seed=9).to(DEV)
    fresh = QuantizedLinear(144, 48, 8, "rfft", num_stages=2, has_bias=True).to(DEV)
    fresh.load_state_dict(mod.state_dict())
    fresh.codebook = mod.codebook
    assert torch.allclose(fresh(x), mod(x), atol=1e-6)
    yf = linear_forward(x, mod._quantized_layer(), mod.codebook) + mod.bias
    assert torch.allclose(yf, mod(x), atol=1e-5)


def test_reference_codebook_objects_are_accepted():
    """A codebook built by name-compatible classes (the reference's) drives the
    same kernels: only the class name and `.stages` / `.scale` are used."""
    class E8PCodebook:  # stand-in with the reference's class name
        pass

    lay = syn.make_layer(32, 64, (syn.E8P,), seed=10)
    mod = make_module(lay)
    x = syn.make_activations(2, 64, dtype=torch.float32, seed=11).to(DEV)
    y = mod(x)
    mod.codebook = E8PCodebook()
    assert torch.allclose(mod(x), y)
