"""Generate the checkpoint fixtures in this directory with the REFERENCE's own
`save_quantized_checkpoint` (numbersletter/quipsharp, checkpoint.py:159-185).

Usage (needs a checkout of the reference; it is not needed to run the tests):

    python tests/golden/make_ckpt_fixture.py /path/to/quipsharp-reference

Writes ckpt_ref_2bit/ (E8P, RHT and RFFT layers, one with a bias) and
ckpt_ref_3bit/ (RVQ E8P + E8-1bit; the reference's manifest carries no stage
scales, so ckpt_ref_3bit/stage_scales.json records the ones used) for a toy
decoder whose module names follow the Hugging Face layout.  Layer contents come
from quipsharp_b200.synthetic (seeded, CPU).
"""
from __future__ import annotations

import json
import os
import sys

import torch
from torch import nn

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def toy_decoder(n_hidden: int = 256, n_inter: int = 384) -> nn.Module:
    """model.layers.0.{self_attn.q_proj, mlp.up_proj, mlp.down_proj} + an embedding."""
    root = nn.Module()
    root.model = nn.Module()
    root.model.embed_tokens = nn.Embedding(16, n_hidden)
    layer = nn.Module()
    layer.self_attn = nn.Module()
    layer.self_attn.q_proj = nn.Linear(n_hidden, n_hidden, bias=False)
    layer.mlp = nn.Module()
    layer.mlp.up_proj = nn.Linear(n_hidden, n_inter, bias=True)
    layer.mlp.down_proj = nn.Linear(n_inter, n_hidden, bias=False)
    root.model.layers = nn.ModuleList([layer])
    return root


LAYERS = [  # name, in, out, has_bias
    ("model.layers.0.self_attn.q_proj", 256, 256, False),   # RHT (both powers of two)
    ("model.layers.0.mlp.up_proj", 256, 384, True),         # RFFT (384 is not a power of two)
    ("model.layers.0.mlp.down_proj", 384, 256, False),      # RFFT
]


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    sys.path.insert(0, REPO)
    from quipsharp import checkpoint as RC
    from quipsharp.quantize import QuantizedLayer
    from quipsharp.incoherence import IncoherenceSigns
    from quipsharp.rfft import RFFTPhases
    from quipsharp.codebooks.e8p import E8PCodebook
    from quipsharp_b200 import synthetic as syn

    for bits, kinds in (("2bit", (syn.E8P,)), ("3bit", (syn.E8P, syn.E8_1BIT))):
        torch.manual_seed(0)
        model = toy_decoder()
        infos, scales = [], None
        for i, (name, n, m, has_bias) in enumerate(LAYERS):
            lay = syn.make_layer(m, n, kinds, seed=100 + i, has_bias=has_bias)
            scales = list(lay.stage_scales) if len(kinds) == 2 else None
            signs = (IncoherenceSigns(su=lay.su, sv=lay.sv) if lay.transform_kind == "rht"
                     else RFFTPhases(phase_u=lay.phase_u, phase_v=lay.phase_v))
            ql = QuantizedLayer(codes=lay.codes, signs=signs, g=8, shape=(m, n), scale=lay.layer_scale)
            parent_name, _, attr = name.rpartition(".")
            RC.replace_with_quantized_linear_(model.get_submodule(parent_name), attr, ql, E8PCodebook(),
                                              bias=lay.bias)
            infos.append({"name": name, "in_features": n, "out_features": m,
                          "transform_kind": lay.transform_kind, "has_bias": has_bias})
        out = os.path.join(HERE, f"ckpt_ref_{bits}")
        RC.save_quantized_checkpoint(model, "toy-decoder", out, bits, 8, 0, infos)
        if scales is not None:
            with open(os.path.join(out, "stage_scales.json"), "w") as f:
                json.dump(scales, f)
        print("wrote", out, sorted(os.listdir(out)))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QUIPSHARP_REF", ""))
