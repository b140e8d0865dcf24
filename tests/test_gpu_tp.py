"""Tensor parallelism on GPUs: two ranks (one process per GPU) run
TPQuantizedLinear (column-sharded fused matmul, push of the float32 y1 shards
into every rank's receive buffer over NVLink, flags in peer memory, gathered
output transform) and must reproduce the unsharded QuantizedLinear forward on
every rank, over several calls (alternating receive regions) and through a
CUDA graph replayed between eager calls.  Needs two GPUs; skipped otherwise."""
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, m, n, kinds, transform, B, dtype_name, q):
    try:
        import datetime
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        import torch.distributed as dist
        from conftest import rel_l2
        from test_gpu_linear import make_module
        from quipsharp_b200 import synthetic as syn
        from quipsharp_b200.tensor_parallel import TPQuantizedLinear
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                timeout=datetime.timedelta(seconds=60))
        dt = getattr(torch, dtype_name)
        lay = syn.make_layer(m, n, kinds, seed=11, transform_kind=transform, has_bias=True)
        x = syn.make_activations(B, n, dtype=dt, seed=12).cuda()
        full = make_module(lay)          # on cuda:rank (current device)
        tp = TPQuantizedLinear(full)
        err, same = 0.0, True

        def check(y_tp, xin):
            nonlocal err, same
            y_ref = full(xin)
            torch.cuda.synchronize()
            err = max(err, rel_l2(y_tp.float().cpu().numpy(), y_ref.float().cpu().numpy()))
            ys = [torch.empty_like(y_tp) for _ in range(world)]  # every rank holds the same output
            dist.all_gather(ys, y_tp)
            same = same and all(torch.equal(ys[0], t) for t in ys[1:])

        for call in range(3):
            xc = syn.make_activations(B, n, dtype=dt, seed=12 + call).cuda()
            check(tp(xc), xc)
        # one captured call (odd), replayed between eager calls
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
            yg = tp(x)
        torch.cuda.current_stream().wait_stream(s)
        for step in range(3):
            x.copy_(syn.make_activations(B, n, dtype=dt, seed=40 + step).cuda())
            g.replay()
            check(yg, x)
            if step != 1:
                check(tp(x), x)
        from quipsharp_b200 import _native as N
        torch.cuda.synchronize()
        if N.lib().qs_device_status(N.stream_of(x)) != 0:
            err = "device status flag set"
        del g
        q.put((rank, err, same))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e), False))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("m,n,kinds,transform,B,dt", [
    (4096, 4096, ("e8p",), "rht", 1, "float16"),                  # decode, RHT, mma.sync path
    (11008, 4096, ("e8p", "e8_1bit"), "rfft", 4, "float16"),      # config-2 shape, RVQ, RFFT
    (2048, 1024, ("e8p",), "rfft", 40, "bfloat16"),               # prefill batch: tcgen05 path
])
def test_tp_two_ranks_match_unsharded(m, n, kinds, transform, B, dt):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, m, n, kinds, transform, B, dt, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, err, same = q.get(timeout=240)
        results[rank] = (err, same)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    tol = 2e-3 if dt == "float16" else 1e-2
    for rank, (err, same) in results.items():
        assert not isinstance(err, str), f"rank {rank}: {err}"
        assert err < tol, (rank, err)
        assert same, f"rank {rank}: outputs differ across ranks"
