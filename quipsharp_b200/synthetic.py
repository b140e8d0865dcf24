"""Seeded synthetic quantized layers with the shapes and value distributions of
the benchmark configurations (no checkpoints or datasets are involved).

Distributions follow how the reference's buffers are filled:
  * E8P codes: uniform over all 65,536 16-bit values (every code is valid),
    stored as int16 like `QuantizedLinear.codes` (quipsharp/checkpoint.py:99-103);
  * second-stage 1-bit indices: uniform in [0, 256);
  * sign vectors: Rademacher +-1 (quipsharp/hadamard.py:43-46);
  * RFFT phases: unit-modulus with uniform angle (quipsharp/rfft.py:31-34);
  * stage scales near the fitted values (s0 in [0.9, 1.2], s1 in [0.3, 0.6]);
  * activations N(0, 1).
Everything is drawn on the CPU from one `torch.Generator`, so the same seed
gives bit-identical tensors on every machine with this torch build.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from .hadamard import is_pow2

E8P = "e8p"
E8_1BIT = "e8_1bit"


@dataclass
class SyntheticLayer:
    m: int                      # out_features
    n: int                      # in_features
    kinds: tuple                # codebook kind per RVQ stage
    codes: torch.Tensor         # int16 (m, n/8) or (stages, m, n/8)
    stage_scales: tuple         # python floats (one per stage; (None,) for a plain codebook)
    layer_scale: float
    transform_kind: str
    su: torch.Tensor = None
    sv: torch.Tensor = None
    phase_u: torch.Tensor = None
    phase_v: torch.Tensor = None
    bias: torch.Tensor = None
    extra: dict = field(default_factory=dict)

    @property
    def num_stages(self) -> int:
        return len(self.kinds)


def make_layer(m: int, n: int, kinds=(E8P,), seed: int = 0, transform_kind: str | None = None,
               layer_scale: float | None = None, has_bias: bool = False) -> SyntheticLayer:
    g = torch.Generator().manual_seed(seed)
    T = n // 8
    stage_codes = []
    for kind in kinds:
        if kind == E8P:
            c = torch.randint(-32768, 32768, (m, T), generator=g, dtype=torch.int32)
        elif kind == E8_1BIT:
            c = torch.randint(0, 256, (m, T), generator=g, dtype=torch.int32)
        else:
            raise ValueError(kind)
        stage_codes.append(c.to(torch.int16))
    codes = stage_codes[0] if len(kinds) == 1 else torch.stack(stage_codes, 0)
    u = torch.rand(3, generator=g, dtype=torch.float64).tolist()
    if len(kinds) == 1:
        stage_scales = (None,)
    else:
        stage_scales = (0.9 + 0.3 * u[0], 0.3 + 0.3 * u[1]) if len(kinds) == 2 else \
            tuple(0.9 * (0.5 ** i) for i in range(len(kinds)))
    if layer_scale is None:
        layer_scale = 1.0 if len(kinds) == 1 else 0.5 + u[2]
    if transform_kind is None:
        transform_kind = "rht" if (is_pow2(m) and is_pow2(n)) else "rfft"
    lay = SyntheticLayer(m=m, n=n, kinds=tuple(kinds), codes=codes, stage_scales=stage_scales,
                         layer_scale=float(torch.tensor(layer_scale, dtype=torch.float32).item()),
                         transform_kind=transform_kind)
    if transform_kind == "rht":
        lay.su = torch.randint(0, 2, (m,), generator=g).to(torch.float32) * 2 - 1
        lay.sv = torch.randint(0, 2, (n,), generator=g).to(torch.float32) * 2 - 1
    else:
        th_u = torch.rand(m // 2, generator=g) * (2 * math.pi)
        th_v = torch.rand(n // 2, generator=g) * (2 * math.pi)
        lay.phase_u = torch.polar(torch.ones_like(th_u), th_u)
        lay.phase_v = torch.polar(torch.ones_like(th_v), th_v)
    if has_bias:
        lay.bias = torch.randn(m, generator=g) * 0.1
    return lay


def make_activations(batch: int, n: int, dtype=torch.float16, seed: int = 1) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(batch, n, generator=g).to(dtype)


# Benchmark configurations (BASELINE.json "configs"), as (name, [(layer, m, n), ...], kinds, dtype, batches)
LLAMA3_8B = [("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
             ("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336)]
QWEN25_7B = [("gate", 18944, 3584), ("up", 18944, 3584), ("down", 3584, 18944)]
LLAMA3_70B = [("q", 8192, 8192), ("k", 1024, 8192), ("v", 1024, 8192), ("o", 8192, 8192),
              ("gate", 28672, 8192), ("up", 28672, 8192), ("down", 8192, 28672)]

CONFIGS = {
    "c1_e8p_4096x4096": dict(layers=[("l", 4096, 4096)], kinds=(E8P,), dtype=torch.float16, batches=(1,)),
    "c2_rvq3_4096to11008": dict(layers=[("l", 11008, 4096)], kinds=(E8P, E8_1BIT), dtype=torch.float16,
                                batches=(1, 8, 32)),
    "c3_llama3_8b_layer": dict(layers=LLAMA3_8B, kinds=(E8P,), dtype=torch.bfloat16, batches=tuple(range(1, 17))),
    "c4_qwen25_7b_prefill": dict(layers=QWEN25_7B, kinds=(E8P,), dtype=torch.bfloat16, batches=(2048, 8192)),
    "c5_llama3_70b_rvq3": dict(layers=LLAMA3_70B, kinds=(E8P, E8_1BIT), dtype=torch.bfloat16, batches=(1, 4096)),
}
