"""The RHT and RFFT input and output steps of the fused forward at every power-of-two
width from 2^10 to 2^14 and decode batches (1 to 32 rows: the one-CTA row
kernels) plus a batch above them (the general row engine), through the split
C ABI, against the oracle (quipsharp/incoherence.py:86-93, quipsharp/rfft.py:37-60):
  input:  x2 = fwht(x * sv) / sqrt(n), or view_as_real(fft(x * phase_v, ortho)),
          stored as fp16 times a power-of-two row scale, with y1 zeroed;
  output: y = fwht(y1) / sqrt(m) * su + bias, or view_as_real(ifft(y1, ortho) *
          conj(phase_u)) + bias, cast; also from the rank-major layout of P
          gathered shards."""
import numpy as np
import pytest
import torch

from oracle import quipsharp_oracle as O
from quipsharp_b200 import _native as N
from conftest import rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _signs(n, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randint(0, 2, (n,), generator=g) * 2 - 1).float()


@pytest.mark.parametrize("lg", [10, 11, 12, 13, 14])
@pytest.mark.parametrize("B,dt", [(1, torch.bfloat16), (5, torch.float16), (32, torch.float32), (40, torch.float16)])
def test_rht_input_step(lg, B, dt):
    n, m_local = 1 << lg, 300
    g = torch.Generator().manual_seed(lg * 100 + B)
    x = torch.randn(B, n, generator=g).to(dt)
    sv = _signs(n, lg)
    nb = N.lib().qs_linear_input_bytes(B, n)
    ws = torch.empty(nb, dtype=torch.uint8, device=DEV)
    y1 = torch.full((B, m_local), 7.0, device=DEV)
    xd, svd = x.to(DEV), sv.to(DEV)
    N.check(N.lib().qs_linear_input(N.ptr(xd), N.IO_DTYPES[dt], B, n, N.QS_RHT, N.ptr(svd), None, N.ptr(ws), nb,
                                    N.ptr(y1), m_local, N.stream_of(xd)))
    torch.cuda.synchronize()
    n_pad = n  # powers of two >= 256 need no padding
    x2h = ws[: B * n_pad * 2].view(torch.float16).reshape(B, n_pad).float().cpu().numpy()
    off = (B * n_pad * 2 + 255) // 256 * 256
    inv = ws[off: off + 4 * B].view(torch.float32).cpu().numpy()
    got = x2h[:, :n] * inv[:, None]
    ref = O.rht_transform_input(x.float().numpy(), sv.numpy())
    assert rel_l2(got, ref) < 1e-3
    # the operand fills the fp16 range: max |x2h| in [2^11, 2^12)
    mx = np.abs(x2h).max(axis=1)
    assert np.all((mx >= 2048) & (mx < 4096))
    assert torch.count_nonzero(y1).item() == 0


@pytest.mark.parametrize("lg", [10, 11, 12, 13, 14])
@pytest.mark.parametrize("B,dt,P", [(1, torch.bfloat16, 1), (3, torch.float32, 1), (32, torch.float16, 1),
                                    (40, torch.float32, 1), (1, torch.float32, 2), (2, torch.float32, 8)])
def test_rht_output_step(lg, B, dt, P):
    m = 1 << lg
    g = torch.Generator().manual_seed(lg * 10 + B + P)
    y1 = torch.randn(B, m, generator=g) * 30
    su = _signs(m, lg + 1)
    bias = torch.randn(m, generator=g)
    mp = m // P
    buf = y1.reshape(B, P, mp).permute(1, 0, 2).contiguous().reshape(-1) if P > 1 else y1.reshape(-1)
    bd, sud, biasd = buf.to(DEV), su.to(DEV), bias.to(DEV)
    y = torch.empty(B, m, dtype=dt, device=DEV)
    N.check(N.lib().qs_linear_output(N.ptr(bd), m, P, B, m, N.QS_RHT, N.ptr(sud), None, N.ptr(biasd), N.ptr(y),
                                     N.IO_DTYPES[dt], N.stream_of(y)))
    torch.cuda.synchronize()
    ref = O.rht_transform_output(y1.numpy(), su.numpy()) + bias.numpy()
    tol = {torch.float32: 1e-5, torch.float16: 1e-3, torch.bfloat16: 8e-3}[dt]
    assert rel_l2(y.float().cpu().numpy(), ref) < tol


def _phase(N, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.rand(N, generator=g, dtype=torch.float64) * 2 * np.pi
    return torch.polar(torch.ones(N, dtype=torch.float64), a).to(torch.complex64)


@pytest.mark.parametrize("lg", [11, 12, 13, 14])
@pytest.mark.parametrize("B,dt", [(1, torch.bfloat16), (5, torch.float16), (32, torch.float32), (40, torch.float16)])
def test_rfft_input_step(lg, B, dt):
    """RFFT input step (quipsharp/rfft.py:37-49): x2 = view_as_real(fft(x * phase_v) / sqrt(n/2))."""
    n, m_local = 1 << lg, 200
    g = torch.Generator().manual_seed(lg * 7 + B)
    x = torch.randn(B, n, generator=g).to(dt)
    ph = _phase(n // 2, lg)
    nb = N.lib().qs_linear_input_bytes(B, n)
    ws = torch.empty(nb, dtype=torch.uint8, device=DEV)
    y1 = torch.full((B, m_local), 3.0, device=DEV)
    xd, phd = x.to(DEV), torch.view_as_real(ph).to(DEV)
    N.check(N.lib().qs_linear_input(N.ptr(xd), N.IO_DTYPES[dt], B, n, N.QS_RFFT, None, N.ptr(phd), N.ptr(ws), nb,
                                    N.ptr(y1), m_local, N.stream_of(xd)))
    torch.cuda.synchronize()
    x2h = ws[: B * n * 2].view(torch.float16).reshape(B, n).float().cpu().numpy()
    off = (B * n * 2 + 255) // 256 * 256
    inv = ws[off: off + 4 * B].view(torch.float32).cpu().numpy()
    ref = O.rfft_to_transformed(x.float().numpy(), ph.numpy())
    assert rel_l2(x2h * inv[:, None], ref) < 1e-3
    mx = np.abs(x2h).max(axis=1)
    assert np.all((mx >= 2048) & (mx < 4096))
    assert torch.count_nonzero(y1).item() == 0


@pytest.mark.parametrize("lg", [11, 12, 13, 14])
@pytest.mark.parametrize("B,dt,P", [(1, torch.bfloat16, 1), (3, torch.float32, 1), (32, torch.float16, 1),
                                    (40, torch.float32, 1), (1, torch.float32, 2), (2, torch.float32, 8)])
def test_rfft_output_step(lg, B, dt, P):
    """RFFT output step (quipsharp/rfft.py:52-60): y = view_as_real(ifft(y1) * sqrt(m/2) conj(phase_u)) + bias."""
    m = 1 << lg
    g = torch.Generator().manual_seed(lg * 13 + B + P)
    y1 = torch.randn(B, m, generator=g) * 30
    ph = _phase(m // 2, lg + 3)
    bias = torch.randn(m, generator=g)
    mp = m // P
    buf = y1.reshape(B, P, mp).permute(1, 0, 2).contiguous().reshape(-1) if P > 1 else y1.reshape(-1)
    bd, phd, biasd = buf.to(DEV), torch.view_as_real(ph).to(DEV), bias.to(DEV)
    y = torch.empty(B, m, dtype=dt, device=DEV)
    N.check(N.lib().qs_linear_output(N.ptr(bd), m, P, B, m, N.QS_RFFT, None, N.ptr(phd), N.ptr(biasd), N.ptr(y),
                                     N.IO_DTYPES[dt], N.stream_of(y)))
    torch.cuda.synchronize()
    ref = O.rfft_from_transformed(y1.numpy(), ph.numpy()) + bias.numpy()
    tol = {torch.float32: 1e-5, torch.float16: 1e-3, torch.bfloat16: 8e-3}[dt]
    assert rel_l2(y.float().cpu().numpy(), ref) < tol
