"""Host logic of groups.py (no GPU): which layers of a decoder form groups, and
when a member call reuses the group's outputs or computes the group again."""
import pytest
import torch
from torch import nn

from quipsharp_b200.checkpoint import QuantizedLinear
from quipsharp_b200.groups import LinearGroup, fuse_linear_groups, linear_groups, unfuse_linear_groups


class CountingGroup(LinearGroup):
    """forward() replaced by a host computation that counts its calls."""

    def __init__(self, modules):
        super().__init__(modules)
        self.calls = 0

    def forward(self, x):
        self.calls += 1
        return [x.sum(-1, keepdim=True) * (i + 1) + self.calls for i in range(len(self.modules))]


def _qlin(n, m, kind="rht"):
    return QuantizedLinear(n, m, 8, kind)


def _decoder_layer(n=64, kv=32, inter=96):
    layer = nn.Module()
    layer.self_attn = nn.Module()
    layer.self_attn.q_proj, layer.self_attn.k_proj = _qlin(n, n), _qlin(n, kv)
    layer.self_attn.v_proj, layer.self_attn.o_proj = _qlin(n, kv), _qlin(n, n)
    layer.mlp = nn.Module()
    layer.mlp.gate_proj, layer.mlp.up_proj = _qlin(n, inter, "rfft"), _qlin(n, inter, "rfft")
    layer.mlp.down_proj = _qlin(inter, n, "rfft")
    return layer


def test_linear_groups_follow_the_reference_grouping():
    layer = _decoder_layer()
    groups = linear_groups(layer)
    assert [[name for name, _ in g] for g in groups] == [
        ["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"], ["mlp.gate_proj", "mlp.up_proj"]]
    layer.self_attn.k_proj = nn.Linear(64, 32)  # not quantized: left out of the group
    layer.self_attn.v_proj = None                # absent (KV-shared layers)
    assert linear_groups(layer) == [linear_groups(layer)[0]]
    assert [n for n, _ in linear_groups(layer)[0]] == ["mlp.gate_proj", "mlp.up_proj"]


def test_fuse_links_every_decoder_layer_and_unfuse_undoes_it():
    model = nn.Module()
    model.layers = nn.ModuleList([_decoder_layer(), _decoder_layer()])
    assert fuse_linear_groups(model) == 4
    q, k = model.layers[1].self_attn.q_proj, model.layers[1].self_attn.k_proj
    assert q._group is k._group and (q._group_index, k._group_index) == (0, 1)
    assert model.layers[0].mlp.down_proj._group is None and model.layers[0].self_attn.o_proj._group is None
    assert q._group is not model.layers[0].self_attn.q_proj._group
    assert "_group" not in "".join(model.state_dict())  # no state: checkpoints unchanged
    unfuse_linear_groups(model)
    assert all(m._group is None for m in model.modules() if isinstance(m, QuantizedLinear))


def test_group_rejects_mismatched_inputs():
    with pytest.raises(ValueError):
        LinearGroup([_qlin(64, 64), _qlin(128, 64)])
    with pytest.raises(ValueError):
        LinearGroup([])
    with pytest.raises(ValueError):
        LinearGroup([_qlin(64, 64) for _ in range(9)])


def test_member_calls_share_one_group_call_per_input():
    mods = [_qlin(64, 64), _qlin(64, 32), _qlin(64, 32)]
    g = CountingGroup(mods)
    x = torch.randn(2, 64)
    outs = [g.member_forward(i, x) for i in (0, 1, 2)]
    assert g.calls == 1
    assert torch.equal(outs[1], x.sum(-1, keepdim=True) * 2 + 1)
    assert g._pending is None and g._src is None  # all taken: nothing held
    g.member_forward(1, x)  # the same input again: a new step
    assert g.calls == 2
    g.member_forward(1, x)  # member 1 asked twice before the others: computes again
    assert g.calls == 3
    g.member_forward(0, x)
    assert g.calls == 3     # member 0's output from that call is still pending
    x.add_(1.0)             # in-place change: pending outputs no longer apply
    g.member_forward(2, x)
    assert g.calls == 4
    y = torch.randn(2, 64)  # another tensor with the same contents is another input
    y.copy_(x)
    g.member_forward(0, y)
    assert g.calls == 5
    with torch.inference_mode():  # no version counter: identity alone
        z = torch.randn(2, 64)
        g.member_forward(0, z)
        g.member_forward(1, z)
    assert g.calls == 6


def test_descriptors_follow_rebuilt_kernels():
    """A member whose kernel was rebuilt (new packed weights) gets a new
    descriptor array; unchanged kernels reuse the cached one."""
    import ctypes
    from types import SimpleNamespace
    from quipsharp_b200 import _native as N

    def fake_kernel(base):
        t = lambda off: SimpleNamespace(data_ptr=lambda: base + off)
        return SimpleNamespace(m=64, packed=t(0), kinds=[N.QS_CB_E8P], _kinds_c=N.int_array([N.QS_CB_E8P]),
                               _ss_c=None, scale=t(256), transform=N.QS_RHT, su=t(512), sv=t(768),
                               phase_u=None, phase_v=None, bias=None)

    g = LinearGroup([_qlin(64, 64), _qlin(64, 64)])
    k1, k2 = fake_kernel(0x100000), fake_kernel(0x200000)
    a = g._descriptors([k1, k2])
    assert g._descriptors([k1, k2]) is a
    assert a[1].packed == 0x200000 and a[0].sv == 0x100000 + 768
    assert a[0].kinds == ctypes.addressof(k1._kinds_c) and a[0].stage_scales is None
    k2b = fake_kernel(0x300000)
    b = g._descriptors([k1, k2b])
    assert b is not a and b[1].packed == 0x300000


def test_group_forward_host_side(monkeypatch):
    """LinearGroup.forward's host logic with the library call replaced by a
    recorder: one workspace carved into 256-byte aligned, disjoint per-layer
    pieces of the sizes the library asks for, one output per member, and a fresh
    descriptor array per call (the cached template is never written)."""
    import ctypes
    from types import SimpleNamespace
    from quipsharp_b200 import _native as N
    from quipsharp_b200 import checkpoint as C

    class FakeKernel:
        def __init__(self, codes, codebook, m, n, *a, **k):
            self.m, self.n = m, n
            self.packed = self.scale = self.su = self.sv = torch.zeros(4)
            self.phase_u = self.phase_v = self.bias = None
            self.kinds, self._kinds_c, self._ss_c, self.transform = [0], N.int_array([0]), None, N.QS_RHT

        def workspace_bytes(self, B):
            return 1000 * self.m + B

    calls = []

    class FakeLib:
        def qs_linear_fwd_group(self, x, dtype, B, n, count, arr, stream):
            calls.append((x, dtype, B, n, count, [(d.m, d.y, d.workspace, d.workspace_bytes) for d in arr[:count]],
                          ctypes.addressof(arr)))
            return N.QS_OK

    monkeypatch.setattr(C, "LinearKernel", FakeKernel)
    monkeypatch.setattr(N, "lib", lambda: FakeLib())
    monkeypatch.setattr(N, "require_cuda", lambda *t: None)
    monkeypatch.setattr(N, "stream_of", lambda t: 0)
    monkeypatch.setattr(torch.cuda, "current_device", lambda: None)  # a CPU tensor's device index
    mods = [_qlin(64, 64), _qlin(64, 32), _qlin(64, 32)]
    for m in mods:
        m.codebook = object()
    g = LinearGroup(mods)
    x = torch.randn(2, 3, 64, dtype=torch.bfloat16)
    ys = g(x)
    assert [tuple(y.shape) for y in ys] == [(2, 3, 64), (2, 3, 32), (2, 3, 32)]
    assert all(y.dtype == torch.bfloat16 for y in ys)
    _, dtype, B, n, count, layers, addr1 = calls[0]
    assert (dtype, B, n, count) == (N.QS_BF16, 6, 64, 3)
    for (m, y, ws, wb), want_m in zip(layers, (64, 32, 32)):
        assert m == want_m and ws % 256 == 0 and wb >= 1000 * m + 6
    spans = sorted((ws, ws + wb) for _, _, ws, wb in layers)
    assert all(a[1] <= b[0] for a, b in zip(spans, spans[1:]))
    assert len({y for _, y, _, _ in layers}) == 3
    g(x)
    assert calls[1][6] != ctypes.addressof(g._layers)  # a copy, not the template
    assert all(d.y is None and d.workspace is None for d in g._layers)
