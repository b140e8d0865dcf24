"""Checkpoint format (quipsharp/checkpoint.py:159-275) on the host: checkpoints
written by the REFERENCE's save_quantized_checkpoint (fixtures made by
tests/golden/make_ckpt_fixture.py) load into this package's modules with every
buffer intact, and this package's own save / load round-trips, including the
optional RVQ stage scales that let the loader rebuild a 3-bit codebook."""
import json
import os
import sys

import pytest
import torch

from quipsharp_b200 import checkpoint as C
from quipsharp_b200.codebooks import E8PCodebook, E8OneBitCodebook

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLDEN)
from make_ckpt_fixture import toy_decoder, LAYERS  # noqa: E402


def _check_against_state(model, ckpt_dir):
    state = torch.load(os.path.join(ckpt_dir, C.STATE_NAME), map_location="cpu")
    got = model.state_dict()
    assert set(got) == set(state)
    for k, v in state.items():
        assert got[k].dtype == v.dtype and got[k].shape == v.shape, k
        assert torch.equal(got[k].cpu(), v), k
    for name, n, m, has_bias in LAYERS:
        q = model.get_submodule(name)
        assert isinstance(q, C.QuantizedLinear)
        assert (q.in_features, q.out_features) == (n, m) and (q.bias is not None) == has_bias


def test_reference_2bit_checkpoint_loads():
    d = os.path.join(GOLDEN, "ckpt_ref_2bit")
    assert C.is_quantized_checkpoint(d)
    model = C.load_quantized_checkpoint(d, device="cpu", model=toy_decoder())
    _check_against_state(model, d)
    assert not model.training
    for name, *_ in LAYERS:
        assert isinstance(model.get_submodule(name).codebook, E8PCodebook)


def test_reference_3bit_checkpoint_with_given_stage_scales():
    d = os.path.join(GOLDEN, "ckpt_ref_3bit")
    if not torch.cuda.is_available():  # no scales: the seeded sweep needs the GPU
        with pytest.raises(RuntimeError, match="CUDA"):
            C.load_quantized_checkpoint(d, device="cpu", model=toy_decoder())
    scales = json.load(open(os.path.join(d, "stage_scales.json")))
    model = C.load_quantized_checkpoint(d, device="cpu", model=toy_decoder(),
                                        codebook=C.codebook_for("3bit", scales))
    _check_against_state(model, d)
    cb = model.get_submodule(LAYERS[0][0]).codebook
    assert [type(s.codebook) for s in cb.stages] == [E8PCodebook, E8OneBitCodebook]
    assert [s.scale for s in cb.stages] == [float(v) for v in scales]
    assert model.get_submodule(LAYERS[1][0]).codes.shape == (2, 384, 32)


def test_round_trip_records_stage_scales_and_loads_onto_meta(tmp_path):
    src = os.path.join(GOLDEN, "ckpt_ref_3bit")
    scales = json.load(open(os.path.join(src, "stage_scales.json")))
    model = C.load_quantized_checkpoint(src, device="cpu", model=toy_decoder(),
                                        codebook=C.codebook_for("3bit", scales))
    manifest = json.load(open(os.path.join(src, C.MANIFEST_NAME)))
    out = tmp_path / "ckpt"
    C.save_quantized_checkpoint(model, manifest["model_id"], out, "3bit", 8, manifest["seed"],
                                manifest["quantized_modules"], stage_scales=scales)
    written = json.load(open(out / C.MANIFEST_NAME))
    # the reference's keys unchanged, plus the stage scales
    assert {k: written[k] for k in manifest} == manifest and written["stage_scales"] == scales
    with torch.device("meta"):
        skeleton = toy_decoder()
    back = C.load_quantized_checkpoint(out, device="cpu", model=skeleton)
    _check_against_state(back, out)
    assert [s.scale for s in back.get_submodule(LAYERS[2][0]).codebook.stages] == scales


def test_unknown_architecture_asks_for_a_skeleton():
    with pytest.raises(RuntimeError, match="model="):
        C.load_quantized_checkpoint(os.path.join(GOLDEN, "ckpt_ref_2bit"), device="cpu")


def test_codebook_for_rejects_bad_bits():
    with pytest.raises(ValueError):
        C.codebook_for("5bit")
    assert isinstance(C.codebook_for("2bit"), E8PCodebook)


def test_split_layers_is_contiguous_and_proportional():
    from quipsharp_b200.checkpoint import split_layers
    where = split_layers([10] * 8, [100, 100])
    assert where == [0, 0, 0, 0, 1, 1, 1, 1]
    # budgets 3:1 -> three quarters of the bytes on the first device
    where = split_layers([10] * 8, [300, 100])
    assert where == [0] * 6 + [1] * 2
    # contiguous, non-decreasing device order
    where = split_layers([5, 30, 5, 5, 30, 5, 5, 30], [60, 60, 60])
    assert where == sorted(where) and set(where) == {0, 1, 2}
    with pytest.raises(ValueError):
        split_layers([10] * 8, [30, 30])          # does not fit at all
    with pytest.raises(ValueError):
        split_layers([50, 50, 20], [60, 60])      # fits in total, not contiguously


def test_place_decoder_layers_moves_inputs_between_devices():
    """Placement over two (host) devices: every placed module receives its inputs on
    its own device and the forward result is unchanged."""
    import torch.nn as nn
    from quipsharp_b200.checkpoint import place_decoder_layers

    class Body(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed_tokens = nn.Embedding(10, 4)
            self.layers = nn.ModuleList([nn.Linear(4, 4) for _ in range(4)])
            self.norm = nn.LayerNorm(4)

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.model = Body()
            self.lm_head = nn.Linear(4, 10)

        def forward(self, ids):
            h = self.model.embed_tokens(ids)
            for layer in self.model.layers:
                h = layer(h)
            return self.lm_head(self.model.norm(h))

    torch.manual_seed(0)
    model = Model()
    ids = torch.tensor([[1, 2, 3]])
    ref = model(ids)
    seen = []
    for layer in model.model.layers:
        layer.register_forward_pre_hook(lambda m, a: seen.append(a[0].device))
    place_decoder_layers(model, model.state_dict(), ["cpu", "cpu"], [10**6, 10**6])
    assert torch.allclose(model(ids), ref)
    assert len(seen) == 4 and all(d.type == "cpu" for d in seen)


def test_kernel_cache_follows_codebook_and_buffers(monkeypatch):
    """QuantizedLinear.kernel() rebuilds its fused-forward state when the codebook
    object or a buffer changes, and reuses it otherwise (LinearKernel replaced by
    a host fake: building the real one packs codes on the GPU)."""
    built = []

    class FakeKernel:
        def __init__(self, codes, codebook, *a, **k):
            built.append(codebook)

    monkeypatch.setattr(C, "LinearKernel", FakeKernel)
    q = C.QuantizedLinear(64, 32, 8, "rht")
    q.codebook = E8PCodebook()
    k = q.kernel()
    assert q.kernel() is k and len(built) == 1
    q.codebook = E8PCodebook()            # another codebook object
    assert q.kernel() is not k and len(built) == 2
    q.codes.add_(1)                       # in-place change of a buffer
    q.kernel()
    assert len(built) == 3
    q.kernel()
    assert len(built) == 3
    assert "_kernel_codebook" not in dict(q.named_modules()) and set(q.state_dict()) == {
        "codes", "scale", "su", "sv"}
