"""qs_linear_fwd_group through groups.LinearGroup and fuse_linear_groups: the
layers of a group run on forked streams and must give what each member's own
forward gives (and what the oracle gives), eagerly, under CUDA-graph replay and
through an unmodified decoder's separate q/k/v and gate/up calls."""
import os
import sys

import numpy as np
import pytest
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from conftest import rel_l2  # noqa: E402
from test_gpu_linear import make_module, oracle_y  # noqa: E402

pytestmark = pytest.mark.gpu


def _group(shapes, kinds, transform, seed=0, bias=False):
    from quipsharp_b200 import synthetic as syn
    lays = [syn.make_layer(m, n, kinds, seed=seed + i, transform_kind=transform, has_bias=bias)
            for i, (m, n) in enumerate(shapes)]
    return lays, [make_module(lay) for lay in lays]


@pytest.mark.parametrize("shapes,kinds,transform,B,dtype", [
    ([(4096, 4096), (1024, 4096), (1024, 4096)], ("e8p",), "rht", 1, torch.float16),     # q, k, v
    ([(4096, 4096), (1024, 4096), (1024, 4096)], ("e8p", "e8_1bit"), "rht", 5, torch.bfloat16),
    ([(11008, 4096), (11008, 4096)], ("e8p", "e8_1bit"), "rfft", 1, torch.float16),     # gate, up
    ([(5504, 2048), (5504, 2048)], ("e8p", "e8p"), "rfft", 17, torch.float16),
    ([(2048, 1024), (512, 1024), (512, 1024)], ("e8p",), "rfft", 40, torch.bfloat16),    # prefill matmul
])
def test_group_matches_members_and_oracle(shapes, kinds, transform, B, dtype):
    from quipsharp_b200 import synthetic as syn
    from quipsharp_b200 import _native as N
    from quipsharp_b200.groups import LinearGroup
    lays, mods = _group(shapes, kinds, transform, bias=True)
    x = syn.make_activations(B, shapes[0][1], dtype=dtype, seed=7).cuda()
    group = LinearGroup(mods)
    own = [mod(x).float().cpu().numpy() for mod in mods]
    refs = [oracle_y(lay, x.cpu()) for lay in lays]
    tol = 2e-3 if dtype == torch.float16 else 1e-2
    for call in range(3):  # the side streams are reused by every call
        ys = group(x)
        torch.cuda.synchronize()
        assert N.lib().qs_device_status(N.stream_of(x)) == 0
        for lay, y, o, ref in zip(lays, ys, own, refs):
            assert y.shape == (B, lay.m) and y.dtype == dtype
            assert rel_l2(y.float().cpu().numpy(), o) < 1e-3, call
            assert rel_l2(y.float().cpu().numpy(), ref) < tol, call


def test_group_graph_replay_with_new_inputs():
    from quipsharp_b200 import synthetic as syn
    from quipsharp_b200.groups import LinearGroup
    shapes = [(4096, 4096), (1024, 4096), (1024, 4096)]
    lays, mods = _group(shapes, ("e8p", "e8_1bit"), "rht", seed=3)
    group = LinearGroup(mods)
    x = syn.make_activations(2, 4096, seed=11).cuda()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        group(x)  # first call outside capture: creates the side streams
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            ys = group(x)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    for step in range(3):
        x.copy_(syn.make_activations(2, 4096, seed=20 + step))
        g.replay()
        torch.cuda.synchronize()
        for lay, y in zip(lays, ys):
            ref = oracle_y(lay, x.cpu())
            assert rel_l2(y.float().cpu().numpy(), ref) < 2e-3, step


def test_group_outputs_are_ordered_before_later_work():
    """Work queued on the caller's stream after the call sees every output
    (the side streams join back), here a reduction launched right after."""
    from quipsharp_b200 import synthetic as syn
    from quipsharp_b200.groups import LinearGroup
    lays, mods = _group([(2048, 2048), (4096, 2048), (2048, 2048)], ("e8p",), "rht", seed=9)
    group = LinearGroup(mods)
    x = syn.make_activations(1, 2048, seed=4).cuda()
    sums = []
    for _ in range(5):
        ys = group(x)
        sums.append(torch.stack([y.float().sum() for y in ys]))  # queued, not synchronised
    torch.cuda.synchronize()
    want = torch.stack([m(x).float().sum() for m in mods]).cpu()
    for s in sums:
        assert torch.allclose(s.cpu(), want, rtol=1e-3, atol=1e-2)


def _tiny_quantized_llama(seed=0):
    """A 2-layer Llama whose projections are random QuantizedLinear layers:
    q/k/v/o RHT (power-of-two widths), gate/up/down RFFT (width 384)."""
    pytest.importorskip("transformers")
    from transformers import LlamaConfig, LlamaForCausalLM
    from quipsharp_b200 import synthetic as syn
    torch.manual_seed(seed)
    cfg = LlamaConfig(vocab_size=128, hidden_size=256, intermediate_size=384, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=64)
    model = LlamaForCausalLM(cfg).to(torch.float16)
    i = 0
    for name, mod in list(model.named_modules()):
        if isinstance(mod, torch.nn.Linear) and ".layers." in name:
            lay = syn.make_layer(mod.out_features, mod.in_features, ("e8p", "e8_1bit"), seed=100 + i,
                                 layer_scale=0.5 / mod.in_features ** 0.5)
            i += 1
            parent, _, attr = name.rpartition(".")
            setattr(model.get_submodule(parent), attr, make_module(lay, device="cpu"))
    return model.cuda().eval()


def test_fused_decoder_matches_unfused():
    from quipsharp_b200.groups import fuse_linear_groups, unfuse_linear_groups
    model = _tiny_quantized_llama()
    ids = torch.randint(0, 128, (2, 9), generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad():
        want = model(ids).logits.float()
        assert fuse_linear_groups(model) == 4  # [q,k,v] and [gate,up] of each of the 2 layers
        got = model(ids).logits.float()
        got2 = model(ids).logits.float()  # a second step reuses nothing stale
        with torch.inference_mode():
            got3 = model(ids).logits.float()  # inference tensors: no version counter
        unfuse_linear_groups(model)
        back = model(ids).logits.float()
    for g in (got, got2, got3, back):
        assert torch.isfinite(g).all()
        assert (g - want).norm() / want.norm() < 2e-3


def test_member_calls_in_any_order_and_after_in_place_change():
    from quipsharp_b200 import synthetic as syn
    from quipsharp_b200.groups import LinearGroup
    lays, mods = _group([(1024, 2048), (512, 2048), (512, 2048)], ("e8p",), "rht", seed=5)
    group = LinearGroup(mods)
    for i, m in enumerate(mods):
        m._group, m._group_index = group, i
    x = syn.make_activations(3, 2048, seed=6).cuda()
    order = [2, 0, 1]
    ys = {i: mods[i](x) for i in order}
    for i, lay in enumerate(lays):
        ref = oracle_y(lay, x.cpu())
        assert rel_l2(ys[i].float().cpu().numpy(), ref) < 2e-3
    y0 = mods[0](x)      # computes the group again
    x.mul_(-1.0)         # in place: the pending outputs no longer apply
    y1 = mods[1](x)
    ref1 = oracle_y(lays[1], x.cpu())
    assert rel_l2(y1.float().cpu().numpy(), ref1) < 2e-3
    assert not np.allclose(y1.float().cpu().numpy(), ys[1].float().cpu().numpy())
    assert y0.shape == (3, 1024)
