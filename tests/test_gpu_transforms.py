"""GPU parity: FWHT / RHT and RFFT transform kernels vs the oracle and the
reference's golden outputs."""
import numpy as np
import pytest
import torch

from oracle import quipsharp_oracle as O
from conftest import rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("n", [1, 2, 4, 8, 16, 32, 128, 1024, 4096])
def test_fwht_golden(golden, n):
    from quipsharp_b200.hadamard import fwht
    x = torch.from_numpy(golden[f"fwht_x_{n}"]).to(DEV)
    np.testing.assert_allclose(fwht(x).cpu().numpy(), golden[f"fwht_y_{n}"], atol=2e-6, rtol=1e-5)


@pytest.mark.parametrize("n", [64, 512, 2048, 8192, 16384, 32768])
def test_fwht_sizes_vs_oracle(n):
    from quipsharp_b200.hadamard import fwht
    g = torch.Generator().manual_seed(n)
    x = torch.randn(5, n, generator=g)
    got = fwht(x.to(DEV)).cpu().numpy()
    assert rel_l2(got, O.fwht(x.numpy())) < 1e-6
    # involution (tests/test_hadamard.py:27-31 of the reference)
    assert rel_l2(fwht(fwht(x.to(DEV))).cpu().numpy(), x.numpy()) < 1e-6


def test_fwht_along_dim_and_dtypes():
    from quipsharp_b200.hadamard import fwht
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4, 8, 6, generator=g)
    got = fwht(x.to(DEV), dim=1).cpu()
    want = torch.stack([torch.from_numpy(O.fwht(x[:, :, j].numpy())) for j in range(6)], dim=-1)
    assert torch.allclose(got, want, atol=1e-5)
    for dt, tol in [(torch.float16, 2e-3), (torch.bfloat16, 1e-2)]:
        xh = torch.randn(3, 256, generator=g).to(dt)
        y = fwht(xh.to(DEV))
        assert y.dtype == dt
        assert rel_l2(y.float().cpu().numpy(), O.fwht(xh.float().numpy())) < tol


def test_rht_transforms(golden):
    from quipsharp_b200.incoherence import transform_input, transform_output, IncoherenceSigns
    x, sv, su = (torch.from_numpy(golden[k]).to(DEV) for k in ("rht_x", "rht_sv", "rht_su"))
    np.testing.assert_allclose(transform_input(x, sv).cpu().numpy(), golden["rht_in"], atol=2e-6)
    np.testing.assert_allclose(IncoherenceSigns(su, sv).transform_output(x).cpu().numpy(),
                               golden["rht_out"], atol=2e-6)


@pytest.mark.parametrize("n", [2, 10, 12, 18, 24, 144, 1152, 4096, 11008, 3584])
def test_rfft_golden(golden, n):
    from quipsharp_b200.rfft import to_transformed_space, from_transformed_space
    x = torch.from_numpy(golden[f"rfft_x_{n}"]).to(DEV)
    ph = torch.from_numpy(golden[f"rfft_phase_{n}"]).to(DEV)
    assert rel_l2(to_transformed_space(x, ph).cpu().numpy(), golden[f"rfft_to_{n}"]) < 5e-6
    assert rel_l2(from_transformed_space(x, ph).cpu().numpy(), golden[f"rfft_from_{n}"]) < 5e-6


# half-lengths covering every radix: primes 11..43, 3/5/7, powers of two,
# lengths whose two row buffers need a cluster of CTAs even for many rows
# (above 12800 points), and the largest supported length (32768)
@pytest.mark.parametrize("n", [22, 26, 34, 38, 46, 58, 62, 74, 82, 86, 30, 98, 250, 1792, 3584, 5504 * 2,
                               9472 * 2, 2 * 14336, 2 * 16384, 2 * 12288, 2 * 4096 * 3, 2 * 43 * 512,
                               2 * 32768])
def test_rfft_sizes_vs_oracle(n):
    from quipsharp_b200.rfft import to_transformed_space, from_transformed_space
    g = torch.Generator().manual_seed(n)
    x = torch.randn(3, n, generator=g)
    th = torch.rand(n // 2, generator=g) * 6.283185307179586
    ph = torch.polar(torch.ones_like(th), th)
    fw = to_transformed_space(x.to(DEV), ph.to(DEV)).cpu().numpy()
    assert rel_l2(fw, O.rfft_to_transformed(x.numpy(), ph.numpy())) < 5e-6
    bw = from_transformed_space(x.to(DEV), ph.to(DEV)).cpu().numpy()
    assert rel_l2(bw, O.rfft_from_transformed(x.numpy(), ph.numpy())) < 5e-6
    # round trip (tests/test_rfft.py:11-19 of the reference)
    rt = from_transformed_space(to_transformed_space(x.to(DEV), ph.to(DEV)), ph.to(DEV)).cpu().numpy()
    assert rel_l2(rt, x.numpy()) < 5e-6


# Many rows: one CTA per row (or a 2-CTA cluster for the largest rows) instead
# of a cluster per row.
@pytest.mark.parametrize("n", [3584, 11008, 18944, 8192, 2 * 14336, 2 * 43 * 512])
def test_rfft_many_rows_vs_oracle(n):
    from quipsharp_b200.rfft import to_transformed_space, from_transformed_space
    g = torch.Generator().manual_seed(n + 1)
    x = torch.randn(300, n, generator=g)
    th = torch.rand(n // 2, generator=g) * 6.283185307179586
    ph = torch.polar(torch.ones_like(th), th)
    fw = to_transformed_space(x.to(DEV), ph.to(DEV)).cpu().numpy()
    assert rel_l2(fw, O.rfft_to_transformed(x.numpy(), ph.numpy())) < 5e-6
    bw = from_transformed_space(x.to(DEV), ph.to(DEV)).cpu().numpy()
    assert rel_l2(bw, O.rfft_from_transformed(x.numpy(), ph.numpy())) < 5e-6


@pytest.mark.parametrize("n", [32, 4096, 32768])
def test_fwht_many_rows_vs_oracle(n):
    from quipsharp_b200.hadamard import fwht
    g = torch.Generator().manual_seed(n + 2)
    x = torch.randn(300, n, generator=g)
    assert rel_l2(fwht(x.to(DEV)).cpu().numpy(), O.fwht(x.numpy())) < 1e-6


def test_rfft_unsupported_and_errors():
    from quipsharp_b200.rfft import to_transformed_space
    with pytest.raises(NotImplementedError):
        to_transformed_space(torch.randn(1, 2 * 47, device=DEV), torch.ones(47, dtype=torch.complex64, device=DEV))
    with pytest.raises(AssertionError):
        to_transformed_space(torch.randn(1, 10, device=DEV), torch.ones(4, dtype=torch.complex64, device=DEV))
