"""GPU parity: codebook decode kernels vs the oracle (bit-exact)."""
import hashlib

import numpy as np
import pytest
import torch

from oracle import quipsharp_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_e8p_decode_all_codes_bit_exact(golden):
    from quipsharp_b200.codebooks import E8PCodebook
    cb = E8PCodebook(device=DEV)
    out = cb.dequantize(torch.arange(65536, device=DEV)).cpu().numpy()
    digest = np.frombuffer(hashlib.sha256(out.astype(np.float32).tobytes()).digest(), np.uint8)
    assert np.array_equal(digest, golden["e8p_all_sha256"])
    assert np.array_equal(out, O.e8p_decode(np.arange(65536)))


@pytest.mark.parametrize("dt", [torch.int16, torch.int32, torch.int64])
def test_e8p_decode_code_dtypes(golden, dt):
    from quipsharp_b200.codebooks import E8PCodebook
    codes = torch.from_numpy(golden["e8p_codes"]).to(dt)  # int16 wraps to negative values
    got = E8PCodebook(device=DEV).dequantize(codes.to(DEV).reshape(64, -1)).cpu().numpy()
    assert np.array_equal(got.reshape(-1, 8), golden["e8p_decoded"])


def test_e8p_decode_negative_and_empty(golden):
    from quipsharp_b200.codebooks import E8PCodebook
    cb = E8PCodebook(device=DEV)
    got = cb.dequantize(torch.from_numpy(golden["e8p_neg_codes"]).to(DEV)).cpu().numpy()
    assert np.array_equal(got, golden["e8p_neg_decoded"])
    assert cb.dequantize(torch.empty(0, 3, dtype=torch.int64, device=DEV)).shape == (0, 3, 8)


def test_1bit_decode_and_index_error(golden):
    from quipsharp_b200.codebooks import E8OneBitCodebook
    cb = E8OneBitCodebook(device=DEV)
    got = cb.dequantize(torch.from_numpy(golden["onebit_idx"]).to(DEV)).cpu().numpy()
    assert np.array_equal(got, golden["onebit_decoded"])
    with pytest.raises(IndexError):
        cb.dequantize(torch.tensor([3, 256], device=DEV))
    with pytest.raises(IndexError):
        cb.dequantize(torch.tensor([-257], device=DEV))
    # the context stays usable after the reported error
    assert cb.dequantize(torch.tensor([1], device=DEV)).shape == (1, 8)


def test_rvq_decode_bit_exact(golden):
    from quipsharp_b200.codebooks import E8PCodebook, E8OneBitCodebook
    from quipsharp_b200.rvq import RVQStage, rvq_dequantize
    s0, s1 = golden["rvq_scales"]
    got = rvq_dequantize([torch.from_numpy(golden["rvq_c0"]).to(DEV), torch.from_numpy(golden["rvq_c1"]).to(DEV)],
                         [RVQStage(E8PCodebook(), float(s0)), RVQStage(E8OneBitCodebook(), float(s1))])
    assert np.array_equal(got.cpu().numpy(), golden["rvq_decoded"])


@pytest.mark.parametrize("name,nst", [("dq_e8p", 1), ("dq_rvq3", 2), ("dq_rvq4", 2)])
def test_dequantize_linear_bit_exact(golden, name, nst):
    from quipsharp_b200.codebooks import E8PCodebook, E8OneBitCodebook
    from quipsharp_b200.rvq import RVQStage
    from quipsharp_b200.quantize import QuantizedLayer, RVQCodebookAdapter, dequantize_linear
    from quipsharp_b200.incoherence import IncoherenceSigns
    codes = torch.from_numpy(golden[name + "_codes"]).to(DEV)
    w = golden[name + "_w"]
    ss = golden[name + "_stage_scales"]
    if nst == 1:
        cb = E8PCodebook()
    else:
        second = E8OneBitCodebook() if name == "dq_rvq3" else E8PCodebook()
        cb = RVQCodebookAdapter([RVQStage(E8PCodebook(), float(ss[0])), RVQStage(second, float(ss[1]))])
    layer = QuantizedLayer(codes=codes.to(torch.int64) & 0xFFFF, signs=None, g=8, shape=w.shape,
                           scale=float(golden[name + "_layer_scale"]))
    got = dequantize_linear(layer, cb).cpu().numpy()
    assert np.array_equal(got, w)


def test_pack_rejects_out_of_range_1bit_codes():
    from quipsharp_b200.quantize import pack_codes
    codes = torch.zeros(2, 16, 32, dtype=torch.int16, device=DEV)
    codes[1, 3, 5] = 300
    with pytest.raises(IndexError):
        pack_codes(codes, [0, 1], 16, 256)
