"""Generate the golden fixtures in this directory by running the REFERENCE
implementation (numbersletter/quipsharp) on seeded inputs.

Usage (needs a checkout of the reference; it is not needed to run the tests):

    python tests/golden/make_golden.py /path/to/quipsharp-reference

The reference is pure Python + torch, so it is imported directly and its own
public functions are called: `build_abs_table`, `E8PCodebook.dequantize`,
`E8OneBitCodebook.dequantize`, `rvq_dequantize`, `dequantize_linear`, `fwht`,
`transform_input/output`, `to/from_transformed_space` and
`QuantizedLinear.forward`.  Inputs come from `quipsharp_b200.synthetic` (seeded,
CPU), so the tests can regenerate the large inputs bit-identically and only the
outputs need to be stored.
"""
from __future__ import annotations

import hashlib
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def main(ref_root: str):
    sys.path.insert(0, ref_root)
    sys.path.insert(0, REPO)
    from quipsharp.codebooks import e8p as ref_e8p
    from quipsharp.codebooks.e8_1bit import E8OneBitCodebook, build_table
    from quipsharp.rvq import RVQStage, rvq_dequantize
    from quipsharp.quantize import RVQCodebookAdapter, dequantize_linear, QuantizedLayer
    from quipsharp.hadamard import fwht
    from quipsharp.incoherence import transform_input, transform_output, IncoherenceSigns
    from quipsharp.rfft import to_transformed_space, from_transformed_space, RFFTPhases
    from quipsharp.checkpoint import QuantizedLinear
    from quipsharp_b200 import synthetic as syn

    torch.set_num_threads(os.cpu_count() or 1)
    out = {}

    # --- tables (e8p.py:84-89, e8_1bit.py:67-71)
    out["abs_table"] = ref_e8p.build_abs_table().numpy()
    out["raw227"] = ref_e8p._enumerate_d8hat_abs_le_norm10().numpy()
    out["onebit_table"] = build_table().numpy()

    # --- E8P decode: a sample with edge codes, plus a digest over all 2^16 codes
    g = torch.Generator().manual_seed(1234)
    sample = torch.cat([torch.tensor([0, 1, 2, 255, 256, 32767, 32768, 65534, 65535]),
                        torch.randint(0, 65536, (4087,), generator=g)])
    cb = ref_e8p.E8PCodebook()
    out["e8p_codes"] = sample.numpy()
    out["e8p_decoded"] = cb.dequantize(sample).numpy()
    allc = torch.arange(65536, dtype=torch.int64)
    full = cb.dequantize(allc).numpy().astype(np.float32)
    out["e8p_all_sha256"] = np.frombuffer(hashlib.sha256(full.tobytes()).digest(), dtype=np.uint8)
    # negative int64 codes as produced without the & 0xFFFF mask
    negs = torch.tensor([-1, -2, -256, -32768, -12345])
    out["e8p_neg_codes"] = negs.numpy()
    out["e8p_neg_decoded"] = cb.dequantize(negs).numpy()
    ob = E8OneBitCodebook()
    idx = torch.tensor([0, 1, 5, 128, 240, 241, 255, -1, -256])
    out["onebit_idx"] = idx.numpy()
    out["onebit_decoded"] = ob.dequantize(idx).numpy()

    # --- RVQ decode (rvq.py:83-88) with python-float stage scales
    g = torch.Generator().manual_seed(99)
    c0 = torch.randint(0, 65536, (777,), generator=g)
    c1 = torch.randint(0, 256, (777,), generator=g)
    s0, s1 = 1.0312345678901, 0.4123456789
    out["rvq_c0"], out["rvq_c1"] = c0.numpy(), c1.numpy()
    out["rvq_scales"] = np.array([s0, s1], dtype=np.float64)
    out["rvq_decoded"] = rvq_dequantize([c0, c1], [RVQStage(cb, s0), RVQStage(ob, s1)]).numpy()

    # --- dequantize_linear via QuantizedLinear._quantized_layer (int16 storage)
    for name, m, n, kinds in [("dq_e8p", 32, 64, (syn.E8P,)), ("dq_rvq3", 24, 48, (syn.E8P, syn.E8_1BIT)),
                              ("dq_rvq4", 16, 32, (syn.E8P, syn.E8P))]:
        lay = syn.make_layer(m, n, kinds, seed=len(name) * 7 + m)
        mod, codebook = _ref_module(lay, QuantizedLinear, ref_e8p, E8OneBitCodebook, RVQStage, RVQCodebookAdapter)
        q = mod._quantized_layer()
        out[name + "_codes"] = lay.codes.numpy()
        out[name + "_stage_scales"] = np.array([s if s is not None else np.nan for s in lay.stage_scales])
        out[name + "_layer_scale"] = np.array(lay.layer_scale, dtype=np.float32)
        out[name + "_w"] = dequantize_linear(q, codebook).numpy()

    # --- FWHT (hadamard.py:17-40)
    g = torch.Generator().manual_seed(7)
    for n in (1, 2, 4, 8, 16, 32, 128, 1024, 4096):
        x = torch.randn(3 if n < 4096 else 1, n, generator=g)
        out[f"fwht_x_{n}"] = x.numpy()
        out[f"fwht_y_{n}"] = fwht(x).numpy()
    # RHT transforms (incoherence.py:86-93)
    x = torch.randn(4, 64, generator=g)
    sv = torch.randint(0, 2, (64,), generator=g).float() * 2 - 1
    su = torch.randint(0, 2, (64,), generator=g).float() * 2 - 1
    out["rht_x"], out["rht_sv"], out["rht_su"] = x.numpy(), sv.numpy(), su.numpy()
    out["rht_in"] = transform_input(x, sv).numpy()
    out["rht_out"] = transform_output(x, su).numpy()

    # --- RFFT transforms (rfft.py:37-60)
    for n in (2, 10, 12, 18, 24, 144, 1152, 4096, 11008, 3584):
        x = torch.randn(3 if n < 4096 else 1, n, generator=g)
        th = torch.rand(n // 2, generator=g) * (2 * torch.pi)
        ph = torch.polar(torch.ones_like(th), th)
        out[f"rfft_x_{n}"], out[f"rfft_phase_{n}"] = x.numpy(), ph.numpy()
        out[f"rfft_to_{n}"] = to_transformed_space(x, ph).numpy()
        out[f"rfft_from_{n}"] = from_transformed_space(x, ph).numpy()

    # --- QuantizedLinear.forward on small layers (checkpoint.py:141-146)
    cases = [
        ("fw_e8p_rht_f32_bias", 64, 128, (syn.E8P,), torch.float32, True, 5),
        ("fw_e8p_rht_f16", 64, 128, (syn.E8P,), torch.float16, False, 3),
        ("fw_e8p_rht_bf16", 32, 256, (syn.E8P,), torch.bfloat16, True, 7),
        ("fw_rvq3_rfft_bf16_bias", 48, 144, (syn.E8P, syn.E8_1BIT), torch.bfloat16, True, 4),
        ("fw_e8p_rfft_f32", 16, 24, (syn.E8P,), torch.float32, False, 2),
        ("fw_rvq4_rht_f16", 32, 64, (syn.E8P, syn.E8P), torch.float16, False, 9),
        ("fw_rvq3_rht_f32", 128, 64, (syn.E8P, syn.E8_1BIT), torch.float32, True, 1),
        ("fw_e8p_rfft_f16_odd", 40, 1152, (syn.E8P,), torch.float16, True, 3),
    ]
    for i, (name, m, n, kinds, dt, bias, B) in enumerate(cases):
        lay = syn.make_layer(m, n, kinds, seed=1000 + i, has_bias=bias)
        x = syn.make_activations(B, n, dtype=dt, seed=2000 + i)
        mod, _ = _ref_module(lay, QuantizedLinear, ref_e8p, E8OneBitCodebook, RVQStage, RVQCodebookAdapter)
        with torch.no_grad():
            y = mod(x)
        assert y.dtype == dt
        out[name + "_meta"] = np.array([m, n, 1000 + i, 2000 + i, B, int(bias)], dtype=np.int64)
        out[name + "_kinds"] = np.array([k for k in kinds])
        out[name + "_dtype"] = np.array(str(dt).replace("torch.", ""))
        out[name + "_y"] = y.float().numpy()

    np.savez_compressed(os.path.join(HERE, "reference_small.npz"), **out)
    print("wrote reference_small.npz with", len(out), "arrays")

    # --- config-shaped forwards (slow in the reference: decode-bound Python loop)
    big = {}
    for name, m, n, kinds, dt, B, lseed, xseed in [
        ("c1", 4096, 4096, (syn.E8P,), torch.float16, 1, 11, 12),
        ("c2", 11008, 4096, (syn.E8P, syn.E8_1BIT), torch.float16, 8, 21, 22),
    ]:
        lay = syn.make_layer(m, n, kinds, seed=lseed)
        x = syn.make_activations(B, n, dtype=dt, seed=xseed)
        mod, _ = _ref_module(lay, QuantizedLinear, ref_e8p, E8OneBitCodebook, RVQStage, RVQCodebookAdapter)
        t0 = time.time()
        with torch.no_grad():
            y = mod(x)
        print(f"{name}: reference forward {time.time() - t0:.1f}s")
        big[name + "_meta"] = np.array([m, n, lseed, xseed, B], dtype=np.int64)
        big[name + "_y"] = y.float().numpy()
    np.savez_compressed(os.path.join(HERE, "reference_configs.npz"), **big)
    print("wrote reference_configs.npz")


def _ref_module(lay, QuantizedLinear, ref_e8p, E8OneBitCodebook, RVQStage, RVQCodebookAdapter):
    """Build the reference's QuantizedLinear holding the synthetic layer's buffers."""
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

    def cb_for(kind):
        return ref_e8p.E8PCodebook() if kind == "e8p" else E8OneBitCodebook()

    if lay.num_stages == 1:
        codebook = cb_for(lay.kinds[0])
    else:
        codebook = RVQCodebookAdapter([RVQStage(cb_for(k), s) for k, s in zip(lay.kinds, lay.stage_scales)])
    mod.codebook = codebook
    return mod, codebook


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QUIPSHARP_REF", ""))
