"""`QuantizedLinear` on B200 (mirrors quipsharp/checkpoint.py:80-156) and the
compact checkpoint format (checkpoint.py:159-275).

Same constructor, buffers and state_dict keys as the reference module, so a
reference checkpoint's state dict loads unchanged: `codes` int16 (m, n/8) or
(stages, m, n/8), `scale` float32 scalar, `su`/`sv` (RHT) or `phase_u`/`phase_v`
(RFFT, complex64), optional float32 `bias`.  `forward` runs the fused CUDA path:
the int16 codes are re-laid into the kernel's weight stream once and cached
(rebuilt automatically when the `codes` buffer is replaced or modified in place).

Checkpoints: a directory with the model's state dict (`quantized_state.pt`) and a
JSON manifest (`quip_config.json`: model_id, bits, block_size, seed and one entry per
quantized module), written and read exactly as the reference does, so checkpoints
saved by either side load in the other.  A 3/4-bit RVQ codebook is rebuilt at load
time as the reference does: `build_codebook` re-runs the seeded stage-scale sweeps
(on the GPU, `quipsharp_b200.rvq.fit_stage_scale`); a `stage_scales` manifest entry
(written by this package's `save_quantized_checkpoint`, ignored by the reference's
loader) or the caller's codebook skips the sweep.  A 2-bit codebook needs no scales.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch
from torch import nn, Tensor

from . import _native as N
from .incoherence import IncoherenceSigns
from .rfft import RFFTPhases
from .quantize import QuantizedLayer, LinearKernel, RVQCodebookAdapter

MANIFEST_NAME = "quip_config.json"
STATE_NAME = "quantized_state.pt"


def num_rvq_stages(bits: str) -> int:
    """checkpoint.py:56-57."""
    return 1 if bits == "2bit" else 2


class QuantizedLinear(nn.Module):
    """Drop-in quantized nn.Linear (checkpoint.py:80-146)."""

    def __init__(self, in_features: int, out_features: int, g: int, transform_kind: str,
                 num_stages: int = 1, has_bias: bool = False):
        super().__init__()
        assert transform_kind in ("rht", "rfft")
        self.in_features = in_features
        self.out_features = out_features
        self.g = g
        self.transform_kind = transform_kind
        self.num_stages = num_stages
        self.codebook = None
        self.register_buffer("bias", torch.zeros(out_features) if has_bias else None)
        T = in_features // g
        codes_shape = (out_features, T) if num_stages == 1 else (num_stages, out_features, T)
        self.register_buffer("codes", torch.zeros(codes_shape, dtype=torch.int16))
        self.register_buffer("scale", torch.zeros(()))
        if transform_kind == "rht":
            self.register_buffer("su", torch.zeros(out_features))
            self.register_buffer("sv", torch.zeros(in_features))
        else:
            self.register_buffer("phase_u", torch.zeros(out_features // 2, dtype=torch.complex64))
            self.register_buffer("phase_v", torch.zeros(in_features // 2, dtype=torch.complex64))
        self._kernel = None
        self._kernel_key = None
        self._kernel_codebook = None  # held: a new codebook at a freed one's address is still new
        self._group = None  # a groups.LinearGroup this layer is a member of (fuse_linear_groups)
        self._group_index = 0

    @classmethod
    def from_quantized_layer(cls, layer: QuantizedLayer, bias: Tensor = None) -> "QuantizedLinear":
        m, n = layer.shape
        kind = "rht" if type(layer.signs).__name__ == "IncoherenceSigns" else "rfft"
        stages = layer.codes.shape[0] if layer.codes.dim() == 3 else 1
        mod = cls(in_features=n, out_features=m, g=layer.g, transform_kind=kind, num_stages=stages,
                  has_bias=bias is not None)
        with torch.no_grad():
            mod.codes.copy_(layer.codes)
            mod.scale.copy_(torch.as_tensor(layer.scale, dtype=torch.float32))
            if bias is not None:
                mod.bias.copy_(bias.float())
            if kind == "rht":
                mod.su.copy_(layer.signs.su)
                mod.sv.copy_(layer.signs.sv)
            else:
                mod.phase_u.copy_(layer.signs.phase_u)
                mod.phase_v.copy_(layer.signs.phase_v)
        return mod

    def _quantized_layer(self) -> QuantizedLayer:
        """checkpoint.py:132-139 (int16 -> int64 & 0xFFFF)."""
        signs = (IncoherenceSigns(su=self.su, sv=self.sv) if self.transform_kind == "rht"
                 else RFFTPhases(phase_u=self.phase_u, phase_v=self.phase_v))
        codes = self.codes.to(torch.int64) & 0xFFFF
        return QuantizedLayer(codes=codes, signs=signs, g=self.g,
                              shape=(self.out_features, self.in_features), scale=self.scale.item())

    def _buffers_key(self):
        bufs = [self.codes, self.scale, self.bias] + (
            [self.su, self.sv] if self.transform_kind == "rht" else [self.phase_u, self.phase_v])
        return (id(self.codebook),) + tuple(
            None if b is None else (b.data_ptr(), b._version, b.device) for b in bufs)

    def kernel(self) -> LinearKernel:
        """The resolved fused-forward state (packed weights etc.), rebuilt when
        a buffer or the codebook changed."""
        if self.codebook is None:
            raise RuntimeError("QuantizedLinear.codebook must be assigned before forward")
        key = self._buffers_key()
        if self._kernel is None or key != self._kernel_key or self.codebook is not self._kernel_codebook:
            targs = (dict(su=self.su, sv=self.sv) if self.transform_kind == "rht"
                     else dict(phase_u=self.phase_u, phase_v=self.phase_v))
            with torch.no_grad():
                self._kernel = LinearKernel(self.codes, self.codebook, self.out_features,
                                            self.in_features, self.scale, self.transform_kind,
                                            bias=self.bias, **targs)
            self._kernel_key = key
            self.__dict__["_kernel_codebook"] = self.codebook  # a plain reference, never a submodule
        return self._kernel

    def forward(self, x: Tensor) -> Tensor:
        if self._group is not None:
            return self._group.member_forward(self._group_index, x)
        return self.kernel()(x)


def replace_with_quantized_linear_(parent: nn.Module, attr: str, layer: QuantizedLayer,
                                   codebook, bias: Tensor = None) -> QuantizedLinear:
    """checkpoint.py:149-156."""
    qlin = QuantizedLinear.from_quantized_layer(layer, bias=bias)
    qlin.codebook = codebook
    setattr(parent, attr, qlin)
    return qlin


def build_codebook(bits: str, device=None, seed: int = 0):
    """checkpoint.py:60-77: the codebook of `bits` and its fitted input scale,
    deterministic given `seed`: E8P (2-bit) or an RVQ of [E8P, E8-1bit] (3-bit) /
    [E8P, E8P] (4-bit) whose stage scales come from the reference's sweeps (E8P on
    N(0, I) with seed; the second stage on stage 1's residuals with seed + 1; the
    returned scale for the whole RVQ with seed + 2; 20,000 samples each).  The
    sweeps run on `device` when it is a CUDA device, else on the current one."""
    from .codebooks import E8PCodebook, E8OneBitCodebook
    from .rvq import RVQStage, fit_stage_scale, fit_residual_stage_scale
    if bits not in ("2bit", "3bit", "4bit"):
        raise ValueError(f"unknown bits {bits!r}")
    e8p = E8PCodebook()
    e8p_scale = fit_stage_scale(e8p, seed=seed, device=device, n_samples=20_000)
    if bits == "2bit":
        return e8p, e8p_scale
    second = E8OneBitCodebook() if bits == "3bit" else E8PCodebook()
    second_scale = fit_residual_stage_scale([RVQStage(e8p, e8p_scale)], second, seed=seed + 1, device=device,
                                            n_samples=20_000)
    rvq_cb = RVQCodebookAdapter([RVQStage(e8p, e8p_scale), RVQStage(second, second_scale)])
    rvq_scale = fit_stage_scale(rvq_cb, seed=seed + 2, device=device, n_samples=20_000)
    return rvq_cb, rvq_scale


def codebook_for(bits: str, stage_scales=None, seed: int = 0, device=None):
    """The codebook a `bits` checkpoint decodes with (checkpoint.py:60-77 builds the
    same objects): 2-bit: E8P; 3-bit: RVQ [E8P, E8-1bit]; 4-bit: RVQ [E8P, E8P].
    The two RVQ stage scales are `stage_scales` when given, else rebuilt from the
    manifest's `seed` by `build_codebook`'s sweeps."""
    from .codebooks import E8PCodebook, E8OneBitCodebook
    from .rvq import RVQStage
    if bits == "2bit":
        return E8PCodebook()
    if bits not in ("3bit", "4bit"):
        raise ValueError(f"unknown bits {bits!r}")
    if stage_scales is None:
        return build_codebook(bits, device, seed)[0]
    if len(stage_scales) != 2:
        raise ValueError(f"a {bits} codebook has two RVQ stage scales, got {len(stage_scales)}")
    second = E8OneBitCodebook() if bits == "3bit" else E8PCodebook()
    return RVQCodebookAdapter([RVQStage(E8PCodebook(), float(stage_scales[0])),
                               RVQStage(second, float(stage_scales[1]))])


def save_quantized_checkpoint(model: nn.Module, model_id: str, save_path, bits: str, block_size: int,
                              seed: int, quantized_modules: list, tokenizer=None, stage_scales=None) -> None:
    """checkpoint.py:159-185: the state dict and the manifest.  `quantized_modules`:
    one {"name", "in_features", "out_features", "transform_kind"[, "has_bias"]} per
    QuantizedLinear.  `stage_scales` (RVQ only) is recorded so this package's loader
    can rebuild the codebook without refitting."""
    save_path = Path(save_path)
    save_path.mkdir(parents=True, exist_ok=True)
    torch.save(model.state_dict(), save_path / STATE_NAME)
    manifest = {"model_id": model_id, "bits": bits, "block_size": block_size, "seed": seed,
                "quantized_modules": quantized_modules}
    if stage_scales is not None:
        manifest["stage_scales"] = [float(v) for v in stage_scales]
    (save_path / MANIFEST_NAME).write_text(json.dumps(manifest, indent=2))
    if tokenizer is not None:
        tokenizer.save_pretrained(save_path)


def is_quantized_checkpoint(path) -> bool:
    """checkpoint.py:188-189."""
    return (Path(path) / MANIFEST_NAME).exists()


def _meta_skeleton(model_id: str) -> nn.Module:
    """The architecture of `model_id` with its parameters on the meta device and
    its computed buffers real (lazy_weights.build_meta_model, as
    checkpoint.py:206-209 uses it); needs the model's config locally (a
    directory or the Hugging Face cache: there is no download here)."""
    try:
        from .lazy_weights import build_meta_model
        return build_meta_model(model_id)[0]
    except Exception as e:  # no transformers, no local config, unknown architecture
        raise RuntimeError(f"cannot build the architecture of {model_id!r} ({e}); pass model= "
                           "(a skeleton whose quantized submodules will be replaced)") from e


def split_layers(layer_bytes: list[int], budgets: list[int]) -> list[int]:
    """Device index of each decoder layer: contiguous runs whose sizes are
    proportional to the device budgets.  Layer i goes to the device whose share
    of the cumulative byte range holds the layer's midpoint; a device that would
    exceed its budget raises (the checkpoint does not fit)."""
    total = float(sum(layer_bytes))
    cap = float(sum(budgets))
    if total > cap:
        raise ValueError(f"decoder layers need {int(total)} bytes, budgets allow {int(cap)}")
    edges, acc = [], 0.0
    for b in budgets:  # cumulative share boundaries of each device in [0, total]
        acc += b
        edges.append(total * acc / cap)
    out, before, load = [], 0.0, [0] * len(budgets)
    for size in layer_bytes:
        mid = before + size / 2.0
        d = next(i for i, e in enumerate(edges) if mid <= e or i == len(edges) - 1)
        out.append(d)
        load[d] += size
        before += size
    for d, (l, b) in enumerate(zip(load, budgets)):
        if l > b:
            raise ValueError(f"device {d} would hold {l} bytes of decoder layers, over its budget {b}")
    return out


def _move(obj, dev):
    if torch.is_tensor(obj):
        return obj.to(dev)
    if isinstance(obj, (tuple, list)):
        return type(obj)(_move(o, dev) for o in obj)
    if isinstance(obj, dict):
        return {k: _move(v, dev) for k, v in obj.items()}
    return obj


def _follow_inputs(module: nn.Module, dev) -> None:
    """Move every tensor argument of module's forward onto `dev` first."""
    module.register_forward_pre_hook(lambda _m, args, kwargs: (_move(args, dev), _move(kwargs, dev)),
                                     with_kwargs=True)


def place_decoder_layers(model: nn.Module, state: dict, devices: list, budgets: list[int]) -> None:
    """Spread a decoder-only model over `devices` by decoder layer (split_layers
    on the state dict's per-layer bytes).  The embeddings stay with the first
    layer, the final norm and head go with the last; every placed module moves
    its inputs to its own device, so the forward runs unchanged."""
    body = getattr(model, "model", None)
    layers = getattr(body, "layers", None)
    if layers is None:
        raise NotImplementedError("multi-device placement needs a model with model.layers (decoder-only)")
    sizes = [0] * len(layers)
    for key, t in state.items():
        parts = key.split(".")
        if len(parts) > 2 and parts[0] == "model" and parts[1] == "layers":
            sizes[int(parts[2])] += t.numel() * t.element_size()
    where = split_layers(sizes, budgets)
    for i, layer in enumerate(layers):
        layer.to(devices[where[i]])
        _follow_inputs(layer, devices[where[i]])
    first, last = devices[where[0]], devices[where[-1]]
    for name, child in body.named_children():
        if name != "layers":
            child.to(first if "embed" in name else last)
            _follow_inputs(child, first if "embed" in name else last)
    head = getattr(model, "lm_head", None)
    if head is not None:
        head.to(last)
        _follow_inputs(head, last)


def load_quantized_checkpoint(save_path, device="cuda", gpu_devices=None, gpu_budget_bytes=None,
                              cpu_budget_bytes=0, *, model: nn.Module | None = None, codebook=None,
                              prepack: bool = True):
    """checkpoint.py:192-275: rebuild the architecture (or take `model`, a skeleton
    on any device, meta included), swap in QuantizedLinear modules of the manifest's
    shapes, load the state dict with assign=True, place it, give every quantized
    module its codebook and return the model in eval mode.

    Placement: everything on `device` (or gpu_devices[0]) when it fits; a checkpoint
    above `gpu_budget_bytes` is split over `gpu_devices` (and the host, with
    `cpu_budget_bytes`) by decoder layer, see place_decoder_layers.
    Codebook: `codebook` if given, else built from the manifest's bits (RVQ: its
    stage_scales when present, else the seeded sweeps of build_codebook, run on the
    first CUDA device the model uses; see codebook_for).  prepack: modules placed on a GPU re-lay
    their codes into the kernels' weight stream (stage 2 of a 3-bit layer at one byte
    per code) now rather than at their first forward."""
    save_path = Path(save_path)
    manifest = json.loads((save_path / MANIFEST_NAME).read_text())
    state = torch.load(save_path / STATE_NAME, map_location="cpu")
    if model is None:
        model = _meta_skeleton(manifest["model_id"])
    stages = num_rvq_stages(manifest["bits"])
    for info in manifest["quantized_modules"]:
        parent_name, _, attr = info["name"].rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, attr, QuantizedLinear(info["in_features"], info["out_features"], manifest["block_size"],
                                              info["transform_kind"], num_stages=stages,
                                              has_bias=info.get("has_bias", False)))
    model.load_state_dict(state, strict=True, assign=True)

    total_bytes = sum(t.numel() * t.element_size() for t in state.values())
    if gpu_devices is None or gpu_budget_bytes is None or total_bytes <= gpu_budget_bytes:
        target = gpu_devices[0] if gpu_devices else device
        model.to(target)
    else:
        devices = list(gpu_devices) + (["cpu"] if cpu_budget_bytes else [])
        budgets = [gpu_budget_bytes] * len(gpu_devices) + ([cpu_budget_bytes] if cpu_budget_bytes else [])
        place_decoder_layers(model, state, devices, budgets)

    if codebook is None:
        cuda = [d for d in ([device] + list(gpu_devices or [])) if torch.device(d).type == "cuda"]
        codebook = codebook_for(manifest["bits"], manifest.get("stage_scales"), manifest.get("seed", 0),
                                cuda[0] if cuda else None)
    shared = codebook
    for info in manifest["quantized_modules"]:
        # the kernels carry their own tables: one codebook object serves every device
        q = model.get_submodule(info["name"])
        q.codebook = shared
        if prepack and q.codes.is_cuda:
            q.kernel()
    model.eval()
    return model
