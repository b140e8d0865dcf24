"""The peer-memory exchange of column-sharded tensor parallelism on ONE GPU.

P ranks are emulated in one process on one stream: each rank's exchange
allocation is an ordinary device buffer, and every "rank" runs the input step,
the matmul of its row shard and the push (qs_tp_push after qs_linear_matmul, or
the fused qs_linear_matmul_tp), which stores into all ranks' receive buffers,
before any rank runs qs_linear_output_peers.  Kernels therefore run strictly one
after another, so no kernel ever waits for one that has not been launched;
every output step finds its data already there.  This checks the
gathered layout, the device-side call counter that picks the receive region,
and CUDA graph replay in any mix with direct calls, for P = 2, 4, 8; the
multi-process path over NVLink is covered by test_gpu_tp.py."""
import sys
import os

import pytest
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from conftest import rel_l2  # noqa: E402

pytestmark = pytest.mark.gpu


class Emulated:
    def __init__(self, full, world):
        from quipsharp_b200 import _native as N
        from quipsharp_b200.quantize import LinearKernel
        from quipsharp_b200.tensor_parallel import exchange_floats, make_peers, shard_rows, ctl_offset
        self.ctl_at = ctl_offset
        self.N, self.world = N, world
        m, n = full.out_features, full.in_features
        self.m, self.n, self.mp = m, n, m // world
        self.full = full
        targs = dict(sv=full.sv) if full.transform_kind == "rht" else dict(phase_v=full.phase_v)
        self.shards = []
        for r in range(world):
            lo, hi = shard_rows(m, world, r)
            self.shards.append(LinearKernel(full.codes[..., lo:hi, :].contiguous(), full.codebook, hi - lo, n,
                                            full.scale, full.transform_kind, **targs))
        dev = full.codes.device
        self.su = None if full.transform_kind != "rht" else full.su.to(dev, torch.float32).contiguous()
        self.phase_u = None if full.transform_kind != "rfft" else torch.view_as_real(
            full.phase_u.to(dev, torch.complex64).contiguous())
        self.bias = None if full.bias is None else full.bias.to(dev, torch.float32).contiguous()
        self.cap = 1 << 18  # receive region (floats): >= batch * m of every case
        self.bufs = [torch.zeros(exchange_floats(self.cap, world), dtype=torch.float32, device=dev)
                     for _ in range(world)]
        bases = [b.data_ptr() for b in self.bufs]
        self.peers = [make_peers(world, r, bases, self.cap) for r in range(world)]

    def __call__(self, x, ys, fused=False):
        """One call of every rank; ys[r] receives rank r's full output.  fused: the
        matmul's CTAs push after a grid barrier (qs_linear_matmul_tp), else
        qs_linear_matmul then qs_tp_push."""
        import ctypes
        N = self.N
        B = x.shape[0]
        assert B * self.m <= self.cap
        for r, k in enumerate(self.shards):
            y1 = torch.empty(B, self.mp, dtype=torch.float32, device=x.device)
            ws = k.input(x, None if B >= 33 else y1)
            pr = ctypes.addressof(self.peers[r])
            if fused:
                N.check(N.lib().qs_linear_matmul_tp(N.ptr(ws), B, k.n, k.m, N.ptr(k.packed), len(k.kinds),
                                                    k._kinds_c, k._ss_c, N.ptr(k.scale), N.ptr(y1), pr,
                                                    N.stream_of(x)))
            else:
                k.matmul(ws, B, y1)
                N.check(N.lib().qs_tp_push(pr, N.ptr(y1), B, self.mp, N.stream_of(x)))
        for r in range(self.world):
            N.check(N.lib().qs_linear_output_peers(
                ctypes.addressof(self.peers[r]), B, self.m, self.shards[r].transform, N.ptr(self.su),
                N.ptr(self.phase_u), N.ptr(self.bias), N.ptr(ys[r]), N.IO_DTYPES[x.dtype], N.stream_of(x)))

    def sequence(self):
        return [int(b[self.ctl_at(self.cap, self.world)].view(torch.int32).item()) for b in self.bufs]


def _module(m, n, kinds, transform):
    from quipsharp_b200 import synthetic as syn
    from test_gpu_linear import make_module
    lay = syn.make_layer(m, n, kinds, seed=21, transform_kind=transform, has_bias=True)
    return make_module(lay)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("m,n,kinds,transform,B", [
    (4096, 4096, ("e8p",), "rht", 1),                 # decode regime, RHT
    (11008, 4096, ("e8p", "e8_1bit"), "rfft", 3),     # config-2 shape, RVQ, RFFT
    (2048, 1024, ("e8p",), "rfft", 40),               # prefill regime (tcgen05 GEMM)
])
def test_emulated_ranks_match_unsharded(world, m, n, kinds, transform, B):
    from quipsharp_b200 import synthetic as syn
    from quipsharp_b200 import _native as N
    full = _module(m, n, kinds, transform)
    em = Emulated(full, world)
    for call in range(4):  # successive calls alternate receive regions and push routes
        x = syn.make_activations(B, n, dtype=torch.float16, seed=30 + call).cuda()
        y_ref = full(x)
        ys = [torch.empty(B, m, dtype=torch.float16, device="cuda") for _ in range(world)]
        em(x, ys, fused=call % 2 == 1)
        torch.cuda.synchronize()
        assert N.lib().qs_device_status(N.stream_of(ys[0])) == 0
        for r in range(world):
            err = rel_l2(ys[r].float().cpu().numpy(), y_ref.float().cpu().numpy())
            assert err < 2e-3, (call, r, err)
            assert torch.equal(ys[r], ys[0]), (call, r)
    assert em.sequence() == [4] * world


def test_emulated_graph_replay_mixed_with_direct_calls():
    """A graph holding ONE call per rank (odd) replayed between direct calls:
    the receive region follows the device-side counter, not the capture."""
    from quipsharp_b200 import synthetic as syn
    from quipsharp_b200 import _native as N
    m, n, world, B = 4096, 2048, 4, 2
    full = _module(m, n, ("e8p",), "rfft")
    em = Emulated(full, world)
    xg = syn.make_activations(B, n, dtype=torch.float16, seed=40).cuda()
    yg = [torch.empty(B, m, dtype=torch.float16, device="cuda") for _ in range(world)]
    em(xg, yg, fused=True)  # warm-up outside capture (call 1)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            em(xg, yg, fused=True)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    calls = 1
    for step in range(5):
        x_new = syn.make_activations(B, n, dtype=torch.float16, seed=50 + step)
        xg.copy_(x_new)
        g.replay()
        calls += 1
        if step % 2 == 0:  # a direct call in between: the parity of later replays flips
            yd = [torch.empty(B, m, dtype=torch.float16, device="cuda") for _ in range(world)]
            em(xg, yd)
            calls += 1
        torch.cuda.synchronize()
        assert N.lib().qs_device_status(N.stream_of(yg[0])) == 0
        y_ref = full(xg)
        for r in range(world):
            err = rel_l2(yg[r].float().cpu().numpy(), y_ref.float().cpu().numpy())
            assert err < 2e-3, (step, r, err)
            if step % 2 == 0:  # split-K atomics: equal up to the summation order
                err_d = rel_l2(yd[r].float().cpu().numpy(), y_ref.float().cpu().numpy())
                assert err_d < 2e-3, (step, r, err_d)
    assert em.sequence() == [calls] * world
