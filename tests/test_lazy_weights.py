"""lazy_weights (quipsharp/lazy_weights.py): tensor-at-a-time checkpoint access,
the skeleton <-> checkpoint name map, materialize / release of submodules and the
multi-device dense loader, on tiny random Llama checkpoints written here as
sharded safetensors (plain, and with the decoder wrapped one level deeper as
multimodal checkpoints store it)."""
import json
import os

import pytest
import torch

transformers = pytest.importorskip("transformers")
safetensors_torch = pytest.importorskip("safetensors.torch")

from quipsharp_b200 import lazy_weights as L  # noqa: E402

TINY = dict(vocab_size=96, hidden_size=32, intermediate_size=64, num_hidden_layers=3, num_attention_heads=4,
            num_key_value_heads=2, max_position_embeddings=64, tie_word_embeddings=False)


def _tiny_model(dtype=torch.bfloat16, **over):
    """Built in `dtype` the way the loader builds its skeleton (computed buffers
    such as the rotary frequencies stay float32)."""
    from transformers import AutoModelForCausalLM, LlamaConfig
    torch.manual_seed(0)
    cfg = LlamaConfig(**{**TINY, **over})
    model = AutoModelForCausalLM.from_config(cfg, dtype=dtype).eval()
    return model, model.config


def _write_shards(path, state, nshards):
    """safetensors shards plus model.safetensors.index.json (or one file)."""
    names = sorted(state)
    if nshards == 1:
        safetensors_torch.save_file({k: state[k].contiguous() for k in names}, os.path.join(path, "model.safetensors"))
        return
    weight_map = {}
    for s in range(nshards):
        part = names[s::nshards]
        fname = f"model-{s + 1:05d}-of-{nshards:05d}.safetensors"
        safetensors_torch.save_file({k: state[k].contiguous() for k in part}, os.path.join(path, fname))
        weight_map.update({k: fname for k in part})
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)


@pytest.fixture(scope="module")
def plain_ckpt(tmp_path_factory):
    path = tmp_path_factory.mktemp("plain")
    model, cfg = _tiny_model()
    cfg.save_pretrained(path)
    _write_shards(str(path), model.state_dict(), 2)
    return str(path), model


@pytest.fixture(scope="module")
def wrapped_ckpt(tmp_path_factory):
    """A multimodal-style checkpoint: decoder under "model.language_model.", a
    vision branch the text skeleton lacks, the head at the top level."""
    from transformers import LlavaConfig
    path = tmp_path_factory.mktemp("wrapped")
    model, cfg = _tiny_model()
    full = LlavaConfig(text_config=cfg.to_dict(), vision_config=dict(hidden_size=16, intermediate_size=32,
                                                                     num_hidden_layers=1, num_attention_heads=2,
                                                                     image_size=28, patch_size=14))
    full.dtype = torch.bfloat16
    full.save_pretrained(path)
    state = {}
    for k, v in model.state_dict().items():
        state[k.replace("model.", "model.language_model.", 1) if k.startswith("model.") else k] = v
    state["model.vision_tower.patch.weight"] = torch.ones(4, 4, dtype=torch.bfloat16)
    state["model.multi_modal_projector.weight"] = torch.ones(2, 2, dtype=torch.bfloat16)
    _write_shards(str(path), state, 3)
    return str(path), model


def test_lazy_checkpoint_reads_single_tensors(plain_ckpt):
    path, model = plain_ckpt
    ck = L.LazyCheckpoint(path)
    state = model.state_dict()
    assert set(ck.keys()) == set(state)
    for name, t in state.items():
        assert name in ck
        assert ck.tensor_nbytes(name) == t.numel() * t.element_size()
        got = ck.get_tensor(name)
        assert got.dtype == t.dtype and torch.equal(got, t)
    assert ck.get_tensor("lm_head.weight", device="cpu").device.type == "cpu"
    assert "model.nonexistent" not in ck
    ck.close()


def test_lazy_checkpoint_single_file_and_missing(tmp_path):
    safetensors_torch.save_file({"a.layers.0.w": torch.arange(6, dtype=torch.float32).reshape(2, 3)},
                                str(tmp_path / "model.safetensors"))
    ck = L.LazyCheckpoint(str(tmp_path))
    assert list(ck.keys()) == ["a.layers.0.w"] and ck.tensor_nbytes("a.layers.0.w") == 24
    empty = tmp_path / "empty"
    empty.mkdir()
    with pytest.raises(FileNotFoundError):
        L.LazyCheckpoint(str(empty))


def test_wrap_prefix_and_key_map():
    assert L._wrap_prefix(["lm_head.weight", "model.layers.0.mlp.up_proj.weight"]) == "model."
    assert L._wrap_prefix(["model.language_model.layers.0.x"]) == "model.language_model."
    with pytest.raises(ValueError):
        L._wrap_prefix(["model.embed_tokens.weight"])
    km = L.KeyMap(["model.language_model.layers.0.a", "model.vision_tower.b", "lm_head.weight"],
                  ["model.layers.0.a", "lm_head.weight"])
    assert km.to_checkpoint("model.layers.3.self_attn.q_proj.weight") == \
        "model.language_model.layers.3.self_attn.q_proj.weight"
    assert km.to_checkpoint("model.embed_tokens.weight") == "model.language_model.embed_tokens.weight"
    assert km.to_checkpoint("lm_head.weight") == "lm_head.weight"
    assert km.to_skeleton("model.language_model.norm.weight") == "model.norm.weight"
    assert km.to_skeleton("model.vision_tower.b") is None
    assert km.to_skeleton("lm_head.weight") == "lm_head.weight"
    same = L.KeyMap(["model.layers.0.a"], ["model.layers.0.a"])
    for name in ("model.layers.1.b", "model.norm.weight", "lm_head.weight"):
        assert same.to_checkpoint(name) == name and same.to_skeleton(name) == name


@pytest.mark.parametrize("which", ["plain", "wrapped"])
def test_meta_skeleton_materialize_release(which, plain_ckpt, wrapped_ckpt):
    path, model = plain_ckpt if which == "plain" else wrapped_ckpt
    skel, text_cfg, full_cfg, ck = L.build_text_skeleton(path)
    assert type(skel).__name__ == "LlamaForCausalLM" and text_cfg.num_hidden_layers == 3
    assert all(p.device.type == "meta" for p in skel.parameters())
    assert all(p.dtype == torch.bfloat16 for p in skel.parameters())  # the checkpoint's dtype, not fp32
    names = [n for n, _ in skel.named_parameters()] + [n for n, _ in skel.named_buffers()]
    km = L.KeyMap(list(ck.keys()), names)
    layer = skel.model.layers[1]
    assert L._layer_nbytes(layer, 1, ck, km) == sum(p.numel() * 2 for p in model.model.layers[1].parameters())
    L.materialize_module_(layer, "model.layers.1", ck, km, "cpu")
    ref = model.model.layers[1].state_dict()
    for n, p in layer.named_parameters():
        assert isinstance(p, torch.nn.Parameter) and p.device.type == "cpu"
        assert torch.equal(p, ref[n]), n
    assert all(p.device.type == "meta" for p in skel.model.layers[0].parameters())
    L.release_module_(layer)
    assert all(p.device.type == "meta" for p in layer.parameters())


def test_materialize_casts_to_the_skeleton_dtype(plain_ckpt):
    path, model = plain_ckpt
    skel, _, _, ck = L.build_text_skeleton(path)
    skel.model.norm.to(dtype=torch.float32)
    km = L.KeyMap(list(ck.keys()), [n for n, _ in skel.named_parameters()])
    L.materialize_module_(skel.model.norm, "model.norm", ck, km, "cpu")
    assert skel.model.norm.weight.dtype == torch.float32
    assert torch.equal(skel.model.norm.weight, model.model.norm.weight.float())


def test_fill_in_order_matches_the_greedy_rule():
    assert L._fill_in_order([3, 3, 3, 3, 3], [7, 5, 100]) == [0, 0, 1, 2, 2]
    assert L._fill_in_order([4, 4, 4], [4, 4]) == [0, 1, 1]  # the last device takes the rest
    assert L._fill_in_order([10, 1], [5, 5]) == [1, 1]  # a layer over a budget skips the device
    assert L._fill_in_order([], [1]) == []


@pytest.mark.parametrize("which", ["plain", "wrapped"])
def test_load_dense_causal_lm_matches_the_model(which, plain_ckpt, wrapped_ckpt):
    path, model = plain_ckpt if which == "plain" else wrapped_ckpt
    loaded = L.load_dense_causal_lm(path, [], 0, cpu_budget_bytes=1 << 30)
    assert not loaded.training
    assert all(p.device.type == "cpu" for p in loaded.parameters())
    ids = torch.randint(0, TINY["vocab_size"], (2, 7), generator=torch.Generator().manual_seed(3))
    with torch.no_grad():
        want = model(ids).logits
        got = loaded(ids).logits
    assert torch.equal(got, want)


def test_load_dense_causal_lm_ties_the_head(tmp_path):
    model, cfg = _tiny_model(tie_word_embeddings=True)
    cfg.save_pretrained(tmp_path)
    state = {k: v for k, v in model.state_dict().items() if k != "lm_head.weight"}  # tied: stored once
    _write_shards(str(tmp_path), state, 1)
    loaded = L.load_dense_causal_lm(str(tmp_path), [], 0, cpu_budget_bytes=1 << 30)
    assert loaded.lm_head.weight.data_ptr() == loaded.model.embed_tokens.weight.data_ptr()
    ids = torch.arange(5).unsqueeze(0)
    with torch.no_grad():
        assert torch.equal(loaded(ids).logits, model(ids).logits)


def test_load_dense_causal_lm_needs_a_device(plain_ckpt):
    with pytest.raises(ValueError):
        L.load_dense_causal_lm(plain_ckpt[0], [], 0)


@pytest.mark.gpu
def test_load_dense_causal_lm_spreads_over_gpu_and_host(plain_ckpt):
    """Layers 0.. on cuda:0 within its budget, the rest on the host; the head
    and embeddings on cuda:0; the call moves activations between them."""
    path, model = plain_ckpt
    layer_bytes = sum(p.numel() * 2 for p in model.model.layers[0].parameters())
    loaded = L.load_dense_causal_lm(path, ["cuda:0"], layer_bytes, cpu_budget_bytes=1 << 30)
    devs = [next(layer.parameters()).device.type for layer in loaded.model.layers]
    assert devs == ["cuda", "cpu", "cpu"]
    assert loaded.lm_head.weight.device.type == "cuda" and loaded.model.embed_tokens.weight.device.type == "cuda"
    assert loaded.model.rotary_emb.inv_freq.device.type == "cuda"
    ids = torch.randint(0, TINY["vocab_size"], (1, 6), generator=torch.Generator().manual_seed(4))
    with torch.no_grad():
        got = loaded(ids.cuda()).logits.float().cpu()
        want = model(ids).logits.float()
    assert (got - want).norm() / want.norm() < 2e-2


def test_quantized_checkpoint_loads_onto_the_architecture_of_its_model_id(plain_ckpt, tmp_path):
    """checkpoint.load_quantized_checkpoint without model=: the skeleton comes from
    build_meta_model(manifest model_id), so the rotary frequencies (computed,
    never saved) are real and the whole model moves to its device."""
    from quipsharp_b200 import checkpoint as C
    from quipsharp_b200.codebooks import E8PCodebook
    path, model = plain_ckpt
    skel, _, _ = L.build_meta_model(path)
    names = []
    g = torch.Generator().manual_seed(5)
    for name, mod in list(skel.named_modules()):
        if isinstance(mod, torch.nn.Linear) and ".layers." in name:
            q = C.QuantizedLinear(mod.in_features, mod.out_features, 8, "rht")
            q.codes.copy_(torch.randint(-2 ** 15, 2 ** 15, q.codes.shape, generator=g, dtype=torch.int16))
            q.scale.fill_(0.5)
            parent, _, attr = name.rpartition(".")
            setattr(skel.get_submodule(parent), attr, q)
            names.append({"name": name, "in_features": mod.in_features, "out_features": mod.out_features,
                          "transform_kind": "rht"})
    rest = {k: v for k, v in model.state_dict().items() if "proj" not in k}
    skel.load_state_dict({**rest, **{k: v for k, v in skel.state_dict().items() if k not in rest}},
                         strict=True, assign=True)
    out = tmp_path / "q"
    C.save_quantized_checkpoint(skel, path, out, "2bit", 8, 0, names)
    back = C.load_quantized_checkpoint(out, device="cpu", codebook=E8PCodebook())
    assert back.model.rotary_emb.inv_freq.device.type == "cpu"
    assert torch.equal(back.model.rotary_emb.inv_freq, model.model.rotary_emb.inv_freq)
    got = back.state_dict()
    for k, v in torch.load(out / C.STATE_NAME, map_location="cpu").items():
        assert torch.equal(got[k], v), k
    assert isinstance(back.model.layers[2].mlp.down_proj, C.QuantizedLinear)
