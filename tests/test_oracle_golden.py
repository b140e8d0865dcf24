"""Pin the CPU oracle against the reference's own outputs (tests/golden/*.npz,
written by tests/golden/make_golden.py from the reference implementation).

Bit-exact for the tables and every decode; tight tolerances for the float
transforms (the oracle computes FFTs in complex128, the reference in
complex64 pocketfft)."""
import hashlib

import numpy as np
import pytest

from oracle import quipsharp_oracle as O
from quipsharp_b200 import synthetic as syn
from conftest import rel_l2


def test_tables_bit_exact(golden):
    assert np.array_equal(O.e8p_abs_table(), golden["abs_table"])
    assert np.array_equal(O.e8_1bit_table(), golden["onebit_table"])
    raw = np.abs(O.e8p_abs_table()[:227])
    assert np.array_equal(raw, golden["raw227"])


def test_e8p_decode_sample_bit_exact(golden):
    assert np.array_equal(O.e8p_decode_bits(golden["e8p_codes"]), golden["e8p_decoded"])
    got = O.e8p_decode(golden["e8p_codes"])
    assert got.dtype == np.float32
    assert np.array_equal(got, golden["e8p_decoded"])


def test_e8p_decode_all_codes_digest(golden):
    full = O.e8p_decode_bits(np.arange(65536)).astype(np.float32)
    digest = np.frombuffer(hashlib.sha256(full.tobytes()).digest(), dtype=np.uint8)
    assert np.array_equal(digest, golden["e8p_all_sha256"])


def test_e8p_decode_negative_int64_codes(golden):
    assert np.array_equal(O.e8p_decode(golden["e8p_neg_codes"]), golden["e8p_neg_decoded"])
    assert np.array_equal(O.e8p_decode_bits(golden["e8p_neg_codes"]), golden["e8p_neg_decoded"])


def test_1bit_decode_with_negative_indices(golden):
    assert np.array_equal(O.e8_1bit_decode(golden["onebit_idx"]), golden["onebit_decoded"])
    with pytest.raises(IndexError):
        O.e8_1bit_decode(np.array([256]))


def test_rvq_decode_bit_exact(golden):
    s0, s1 = golden["rvq_scales"]
    got = O.rvq_decode([golden["rvq_c0"], golden["rvq_c1"]], [O.E8P, O.E8_1BIT], [s0, s1])
    assert np.array_equal(got, golden["rvq_decoded"])


@pytest.mark.parametrize("name,kinds", [("dq_e8p", (O.E8P,)), ("dq_rvq3", (O.E8P, O.E8_1BIT)),
                                        ("dq_rvq4", (O.E8P, O.E8P))])
def test_dequantize_linear_bit_exact(golden, name, kinds):
    codes = golden[name + "_codes"]
    ss = golden[name + "_stage_scales"]
    ss = None if np.isnan(ss).all() else list(ss)
    w = golden[name + "_w"]
    got = O.dequantize_linear(codes, kinds, ss, float(golden[name + "_layer_scale"]), *w.shape)
    assert np.array_equal(got, w)


@pytest.mark.parametrize("n", [1, 2, 4, 8, 16, 32, 128, 1024, 4096])
def test_fwht(golden, n):
    got = O.fwht(golden[f"fwht_x_{n}"])
    np.testing.assert_allclose(got, golden[f"fwht_y_{n}"], rtol=0, atol=1e-6)


def test_fwht_rejects_non_pow2():
    with pytest.raises(ValueError):
        O.fwht(np.zeros(3, np.float32))


def test_rht_transforms(golden):
    x, sv, su = golden["rht_x"], golden["rht_sv"], golden["rht_su"]
    np.testing.assert_allclose(O.rht_transform_input(x, sv), golden["rht_in"], atol=1e-6)
    np.testing.assert_allclose(O.rht_transform_output(x, su), golden["rht_out"], atol=1e-6)


@pytest.mark.parametrize("n", [2, 10, 12, 18, 24, 144, 1152, 4096, 11008, 3584])
def test_rfft_transforms(golden, n):
    x, ph = golden[f"rfft_x_{n}"], golden[f"rfft_phase_{n}"]
    assert rel_l2(O.rfft_to_transformed(x, ph), golden[f"rfft_to_{n}"]) < 2e-6
    assert rel_l2(O.rfft_from_transformed(x, ph), golden[f"rfft_from_{n}"]) < 2e-6


FORWARD_CASES = ["fw_e8p_rht_f32_bias", "fw_e8p_rht_f16", "fw_e8p_rht_bf16", "fw_rvq3_rfft_bf16_bias",
                 "fw_e8p_rfft_f32", "fw_rvq4_rht_f16", "fw_rvq3_rht_f32", "fw_e8p_rfft_f16_odd"]


def oracle_forward(lay, x_np):
    ss = None if lay.num_stages == 1 else list(lay.stage_scales)
    t = lambda v: None if v is None else v.numpy()
    return O.linear_forward(x_np, lay.codes.numpy(), list(lay.kinds), ss, lay.layer_scale,
                            lay.transform_kind, su=t(lay.su), sv=t(lay.sv), phase_u=t(lay.phase_u),
                            phase_v=t(lay.phase_v), bias=t(lay.bias))


@pytest.mark.parametrize("name", FORWARD_CASES)
def test_forward_matches_reference(golden, name):
    import torch
    m, n, lseed, xseed, B, bias = golden[name + "_meta"]
    kinds = tuple(str(k) for k in golden[name + "_kinds"])
    dt = getattr(torch, str(golden[name + "_dtype"]))
    lay = syn.make_layer(int(m), int(n), kinds, seed=int(lseed), has_bias=bool(bias))
    x = syn.make_activations(int(B), int(n), dtype=dt, seed=int(xseed))
    y32 = oracle_forward(lay, x.float().numpy())
    y = torch.from_numpy(y32).to(dt).float().numpy()  # same final cast as the reference
    ref = golden[name + "_y"]
    tol = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 1e-2}[dt]
    assert rel_l2(y, ref) < tol, rel_l2(y, ref)


@pytest.mark.parametrize("cfg", ["c1", "c2"])
def test_config_forward_matches_reference(golden_configs, cfg):
    import torch
    m, n, lseed, xseed, B = golden_configs[cfg + "_meta"]
    kinds = (syn.E8P,) if cfg == "c1" else (syn.E8P, syn.E8_1BIT)
    lay = syn.make_layer(int(m), int(n), kinds, seed=int(lseed))
    x = syn.make_activations(int(B), int(n), dtype=torch.float16, seed=int(xseed))
    y = torch.from_numpy(oracle_forward(lay, x.float().numpy())).half().float().numpy()
    assert rel_l2(y, golden_configs[cfg + "_y"]) < 1e-3
