"""Tensor-at-a-time loading of full-precision causal-LM checkpoints (mirrors
quipsharp/lazy_weights.py: LazyCheckpoint, KeyMap, build_meta_model,
build_text_skeleton, materialize_module_, release_module_, load_dense_causal_lm).

A 70B-class bf16 checkpoint does not fit in host memory, so nothing here reads
more than one tensor at a time:

* `LazyCheckpoint` indexes a safetensors checkpoint (one file, or shards with
  `model.safetensors.index.json`) and reads single tensors from the memory-mapped
  shards; `tensor_nbytes` reads only a shard's header.
* `build_meta_model` builds the text decoder of a config with its parameters on
  the meta device (no memory for weights; computed buffers stay real),
  unwrapping multimodal configs with `get_text_config()`.
* `KeyMap` translates skeleton names to checkpoint names and back when a
  checkpoint nests its decoder one level deeper (a multimodal wrapper: decoder
  weights under "model.language_model." for a "model." skeleton); the wrapping
  prefix is found as whatever precedes ".layers.0." on each side.
* `materialize_module_` fills one submodule from the checkpoint onto a device
  (casting to the skeleton's dtype) and `release_module_` returns it to the meta
  device, so callers can walk the decoder layers of any size one at a time.
* `load_dense_causal_lm` places a whole model over GPUs by decoder layer, then
  the host, and makes each placed module move its inputs to its own device, so
  `model(input_ids)` works as for a single-device model.

Differences from the reference: the model id may be a local directory (the
Hugging Face hub is asked only for an id that is not one); the meta-device
skeleton, the tensor replacement and the cross-device hooks are this package's
own (no `accelerate`).
"""
from __future__ import annotations

import contextlib
import json
import os
from pathlib import Path

import torch
from torch import nn


def _resolve_dir(model_id: str, revision: str | None) -> Path:
    if os.path.isdir(model_id):
        return Path(model_id)
    from huggingface_hub import snapshot_download
    return Path(snapshot_download(model_id, revision=revision,
                                  allow_patterns=["*.safetensors", "*.safetensors.index.json", "*.json"]))


class LazyCheckpoint:
    """Name -> tensor access over a (possibly sharded) safetensors checkpoint,
    one tensor in memory at a time (lazy_weights.py:45-99)."""

    _NBYTES = {"F64": 8, "I64": 8, "F32": 4, "I32": 4, "F16": 2, "BF16": 2, "I16": 2, "I8": 1, "U8": 1,
               "BOOL": 1, "F8_E4M3": 1, "F8_E5M2": 1}

    def __init__(self, model_id: str, revision: str | None = None):
        self.local_dir = _resolve_dir(model_id, revision)
        index = self.local_dir / "model.safetensors.index.json"
        if index.exists():
            self.weight_map: dict[str, str] = dict(json.loads(index.read_text())["weight_map"])
        else:
            single = self.local_dir / "model.safetensors"
            if not single.exists():
                raise FileNotFoundError(f"no safetensors weights under {self.local_dir}")
            self.weight_map = {name: "model.safetensors" for name in self._header(single)}
        self._files: dict[str, object] = {}

    @staticmethod
    def _header(path: Path) -> dict:
        """The JSON header of a safetensors file: name -> {dtype, shape, offsets}."""
        with open(path, "rb") as f:
            n = int.from_bytes(f.read(8), "little")
            head = json.loads(f.read(n))
        head.pop("__metadata__", None)
        return head

    def keys(self):
        return self.weight_map.keys()

    def __contains__(self, name: str) -> bool:
        return name in self.weight_map

    def _file(self, name: str):
        shard = self.weight_map[name]
        f = self._files.get(shard)
        if f is None:
            from safetensors import safe_open
            f = self._files[shard] = safe_open(str(self.local_dir / shard), framework="pt", device="cpu")
        return f

    def tensor_nbytes(self, name: str) -> int:
        """Bytes of tensor `name`, from its shard's header (no tensor data read)."""
        sl = self._file(name).get_slice(name)
        count = 1
        for d in sl.get_shape():
            count *= int(d)
        return count * self._NBYTES.get(sl.get_dtype(), 4)

    def get_tensor(self, name: str, device=None) -> torch.Tensor:
        t = self._file(name).get_tensor(name)
        return t if device is None else t.to(device)

    def close(self) -> None:
        self._files.clear()


def _wrap_prefix(names) -> str:
    """What precedes "layers.0." in the first name that has ".layers.0." (e.g.
    "model." or "model.language_model."); the same wrapping holds for the
    decoder's other top-level modules (embeddings, final norm)."""
    for name in names:
        i = name.find(".layers.0.")
        if i >= 0:
            return name[: i + 1]
    raise ValueError("no name contains '.layers.0.': not a decoder-style causal LM")


class KeyMap:
    """Skeleton <-> checkpoint names across a differing decoder wrap prefix
    (lazy_weights.py:120-139).  Names outside the wrap (lm_head) are the same on
    both sides; checkpoint branches the text skeleton lacks (a vision tower under
    the same top-level module) map to None."""

    def __init__(self, checkpoint_names, skeleton_names):
        self.src_wrap = _wrap_prefix(checkpoint_names)
        self.dst_wrap = _wrap_prefix(skeleton_names)

    def to_checkpoint(self, skeleton_name: str) -> str:
        if skeleton_name.startswith(self.dst_wrap):
            return self.src_wrap + skeleton_name[len(self.dst_wrap):]
        return skeleton_name

    def to_skeleton(self, checkpoint_name: str) -> str | None:
        if checkpoint_name.startswith(self.src_wrap):
            return self.dst_wrap + checkpoint_name[len(self.src_wrap):]
        top = self.src_wrap.split(".", 1)[0] + "."
        return None if checkpoint_name.startswith(top) else checkpoint_name


@contextlib.contextmanager
def _parameters_on_meta():
    """Modules built inside have every parameter on the meta device while their
    buffers stay real: computed, unsaved buffers (rotary frequencies) keep
    their values, as they must, since no checkpoint holds them.  A parameter is
    moved as it is registered, before any initialiser touches it, so building a
    70B-class architecture allocates one parameter's storage at a time and
    initialises nothing."""
    register = nn.Module.register_parameter

    def to_meta(module, name, param):
        if param is not None and param.device.type != "meta":
            param = nn.Parameter(param.to("meta"), requires_grad=param.requires_grad)
        register(module, name, param)

    nn.Module.register_parameter = to_meta
    try:
        yield
    finally:
        nn.Module.register_parameter = register


def build_meta_model(model_id: str):
    """(model, text_config, full_config): the text decoder of `model_id`'s config
    with its parameters on the meta device, in the checkpoint's own dtype
    (lazy_weights.py:149-179; a float32 skeleton would double the memory of
    every bf16 tensor it receives).  `get_text_config()` unwraps a multimodal
    config to its decoder; the dtype is read from the full config, which may
    be the only one that carries it."""
    from transformers import AutoConfig, AutoModelForCausalLM
    full_config = AutoConfig.from_pretrained(model_id)
    text_config = full_config.get_text_config()
    dtype = getattr(full_config, "dtype", None) or getattr(full_config, "torch_dtype", None) or torch.bfloat16
    with _parameters_on_meta():
        model = AutoModelForCausalLM.from_config(text_config, dtype=dtype)
    return model, text_config, full_config


def build_text_skeleton(model_id: str):
    """(model, text_config, full_config, checkpoint): `build_meta_model` plus a
    `LazyCheckpoint` to fill it from (lazy_weights.py:180-187)."""
    model, text_config, full_config = build_meta_model(model_id)
    return model, text_config, full_config, LazyCheckpoint(model_id)


def _set_tensor(module: nn.Module, local_name: str, value: torch.Tensor) -> None:
    owner_name, _, attr = local_name.rpartition(".")
    owner = module.get_submodule(owner_name) if owner_name else module
    old = owner._parameters.get(attr) if attr in owner._parameters else owner._buffers.get(attr)
    if old is not None and old.dtype != value.dtype and value.is_floating_point():
        value = value.to(old.dtype)
    if attr in owner._parameters:
        owner._parameters[attr] = nn.Parameter(value, requires_grad=old.requires_grad if old is not None else False)
    else:
        owner._buffers[attr] = value


def materialize_module_(module: nn.Module, module_prefix: str, checkpoint: LazyCheckpoint, key_map: KeyMap,
                        device) -> None:
    """Fill every parameter and buffer of `module` (reached from the skeleton's
    root by `module_prefix`) from the checkpoint onto `device`, one tensor at a
    time, cast to the skeleton's dtype; names the checkpoint lacks (computed
    buffers) are left as they are (lazy_weights.py:190-208)."""
    names = [n for n, _ in module.named_parameters(recurse=True)]
    names += [n for n, _ in module.named_buffers(recurse=True)]
    for local in names:
        full = f"{module_prefix}.{local}" if module_prefix else local
        src = key_map.to_checkpoint(full)
        if src in checkpoint:
            _set_tensor(module, local, checkpoint.get_tensor(src, device=device))


def release_module_(module: nn.Module) -> None:
    """Return every tensor of `module` to the meta device (its memory is freed)."""
    module.to("meta")


def _layer_nbytes(layer: nn.Module, index: int, checkpoint: LazyCheckpoint, key_map: KeyMap) -> int:
    """Bytes of decoder layer `index` from the checkpoint's shard headers (no data
    read): the layer's real projection shapes, whatever the architecture."""
    total = 0
    for local, _ in layer.named_parameters(recurse=True):
        src = key_map.to_checkpoint(f"model.layers.{index}.{local}")
        if src in checkpoint:
            total += checkpoint.tensor_nbytes(src)
    return total


def _fill_in_order(sizes: list[int], budgets: list[int]) -> list[int]:
    """Device index of each layer: layers go in order to the current device
    until the next would pass its budget, then to the next device; the last
    device takes the rest, over budget or not (lazy_weights.py:279-288)."""
    out, d, used = [], 0, 0
    for size in sizes:
        while d < len(budgets) - 1 and used + size > budgets[d]:
            d, used = d + 1, 0
        out.append(d)
        used += size
    return out


def load_dense_causal_lm(model_id: str, gpu_devices: list, gpu_budget_bytes: int, cpu_budget_bytes: int | None = None):
    """The full-precision text decoder of `model_id`, decoder layers placed in
    order on `gpu_devices` (each filled to `gpu_budget_bytes` before the next),
    then on the host (`cpu_budget_bytes`); the last device takes whatever does
    not fit.  Embeddings, final norm and head go on the first GPU, which with
    several GPUs keeps half its budget for them and the logits
    (lazy_weights.py:237-306).  Every placed module moves its inputs to its own
    device first, so the model is called like a single-device one."""
    from .checkpoint import _follow_inputs
    model, _, _ = build_meta_model(model_id)
    checkpoint = LazyCheckpoint(model_id)
    skeleton_names = [n for n, _ in model.named_parameters()] + [n for n, _ in model.named_buffers()]
    key_map = KeyMap(list(checkpoint.keys()), skeleton_names)

    devices = list(gpu_devices) + (["cpu"] if cpu_budget_bytes else [])
    budgets = [gpu_budget_bytes] * len(gpu_devices) + ([cpu_budget_bytes] if cpu_budget_bytes else [])
    if not devices:
        raise ValueError("no device: give gpu_devices or a cpu_budget_bytes")
    main = gpu_devices[0] if gpu_devices else "cpu"
    if len(gpu_devices) > 1:
        budgets[0] = gpu_budget_bytes // 2

    layers = model.get_submodule("model.layers")
    where = _fill_in_order([_layer_nbytes(layer, i, checkpoint, key_map) for i, layer in enumerate(layers)],
                           budgets)
    placed = {}
    for i, layer in enumerate(layers):
        materialize_module_(layer, f"model.layers.{i}", checkpoint, key_map, devices[where[i]])
        placed[layer] = devices[where[i]]
    for name, child in model.model.named_children():
        if name != "layers":
            materialize_module_(child, f"model.{name}", checkpoint, key_map, main)
            placed[child] = main
    if hasattr(model, "lm_head"):
        materialize_module_(model.lm_head, "lm_head", checkpoint, key_map, main)
        placed[model.lm_head] = main
    model.tie_weights()  # replaced tensors broke e.g. the head <-> embedding tie
    checkpoint.close()
    for module, dev in placed.items():
        module.to(dev)  # computed buffers (not in the checkpoint) join their module's device
        _follow_inputs(module, dev)
    model.eval()
    return model
