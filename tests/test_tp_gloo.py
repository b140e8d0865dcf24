"""Tensor-parallel host logic on CPU with world_size 2 over gloo.

Each rank computes its row shard of y1 with the oracle, the shards are
gathered in the layout TPQuantizedLinear's push kernels write into every
rank's receive buffer (rank-major, one flat buffer),
the gathered buffer is read through `gathered_offset` (the index function of
the output-transform kernel), and the output transform is applied; the result
must equal the unsharded forward.  A second test kills one rank before the
collective and checks the survivor gets an error instead of hanging."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=60):
    import datetime
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _sharded_forward(rank, world, port, m, n, transform, B, q):
    try:
        _init(rank, world, port)
        from oracle import quipsharp_oracle as O
        from quipsharp_b200 import synthetic as syn
        from quipsharp_b200.tensor_parallel import shard_rows, gathered_offset
        lay = syn.make_layer(m, n, (syn.E8P, syn.E8_1BIT), seed=5, transform_kind=transform, has_bias=True)
        x = syn.make_activations(B, n, dtype=torch.float32, seed=6).numpy()
        lo, hi = shard_rows(m, world, rank)
        w = O.dequantize_linear(lay.codes.numpy()[:, lo:hi], list(lay.kinds), list(lay.stage_scales),
                                lay.layer_scale, hi - lo, n)
        x2 = O.rht_transform_input(x, lay.sv.numpy()) if transform == "rht" else \
            O.rfft_to_transformed(x, lay.phase_v.numpy())
        y1_local = torch.from_numpy((x2 @ w.T).astype(np.float32))
        gathered = torch.empty(world * B * (hi - lo), dtype=torch.float32)
        dist.all_gather_into_tensor(gathered, y1_local.reshape(-1))
        g = gathered.numpy()
        y1 = np.array([[g[gathered_offset(b, c, B, m, world)] for c in range(m)] for b in range(B)],
                      dtype=np.float32)
        y = O.rht_transform_output(y1, lay.su.numpy()) if transform == "rht" else \
            O.rfft_from_transformed(y1, lay.phase_u.numpy())
        y = y + lay.bias.numpy()
        full = O.linear_forward(x, lay.codes.numpy(), list(lay.kinds), list(lay.stage_scales), lay.layer_scale,
                                transform, su=None if lay.su is None else lay.su.numpy(),
                                sv=None if lay.sv is None else lay.sv.numpy(),
                                phase_u=None if lay.phase_u is None else lay.phase_u.numpy(),
                                phase_v=None if lay.phase_v is None else lay.phase_v.numpy(),
                                bias=lay.bias.numpy())
        err = float(np.linalg.norm(y - full) / np.linalg.norm(full))
        q.put((rank, err))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))


@pytest.mark.parametrize("m,n,transform,B", [(64, 128, "rht", 3), (48, 144, "rfft", 2)])
def test_column_sharded_forward_matches_unsharded(m, n, transform, B):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_forward, args=(r, 2, port, m, n, transform, B, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert isinstance(res[r], float), res[r]
        assert res[r] < 1e-5, res


def _rank_fails_before_collective(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        os._exit(3)  # dies between steps, never reaches the all-gather
    try:
        t = torch.ones(4)
        out = torch.empty(8)
        dist.all_gather_into_tensor(out, t)
        q.put((rank, "no error"))
    except Exception as e:
        q.put((rank, type(e).__name__))


def test_lost_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_fails_before_collective, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert rank == 0 and outcome != "no error"


def test_shard_rows_and_offsets():
    from quipsharp_b200.tensor_parallel import shard_rows, gathered_offset
    assert shard_rows(28672, 8, 3) == (10752, 14336)
    with pytest.raises(ValueError):
        shard_rows(100, 8, 0)
    # the rank-major layout is a permutation of (B, m)
    B, m, P = 3, 16, 4
    offs = sorted(gathered_offset(b, c, B, m, P) for b in range(B) for c in range(m))
    assert offs == list(range(B * m))
