"""Codebook construction on the GPU (qs_fit_scale_sweep): the stage-scale sweeps
of quipsharp/rvq.py:28-66 and build_codebook (quipsharp/checkpoint.py:60-77),
against the reference's own results (tests/golden/reference_codebook_scales.json,
written by tests/golden/make_codebook_scales.py) and the oracle; and a
reference-written 3-bit checkpoint loaded with no stage scales supplied."""
import json
import os
import sys

import numpy as np
import pytest
import torch

from oracle import quipsharp_oracle as O
from quipsharp_b200 import checkpoint as C
from quipsharp_b200 import _native as N
from quipsharp_b200 import synthetic as syn
from quipsharp_b200.codebooks import E8PCodebook, E8OneBitCodebook
from quipsharp_b200.quantize import RVQCodebookAdapter
from quipsharp_b200.rvq import RVQStage, sweep_scale_mse
from conftest import rel_l2

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLDEN)
from make_ckpt_fixture import toy_decoder, LAYERS  # noqa: E402

with open(os.path.join(GOLDEN, "reference_codebook_scales.json")) as _f:
    REF = json.load(_f)
CB = {"e8p": E8PCodebook, "e8_1bit": E8OneBitCodebook}


def _codebook(stages):
    if len(stages) == 1:
        return CB[stages[0][0]]()
    return RVQCodebookAdapter([RVQStage(CB[k](), s) for k, s in stages])


@pytest.mark.parametrize("i", range(5))
def test_sweep_errors_match_reference(i):
    sw = REF["sweeps"][i]
    g = torch.Generator().manual_seed(sw["seed"])
    x = torch.randn(sw["n_samples"], 8, generator=g).cuda()
    cands = torch.linspace(0.5, 4.0, 71) if sw["kind"] == "stage" else torch.linspace(0.05, 2.0, 79)
    prev = [RVQStage(CB[k](), s) for k, s in sw["prev"]]
    mse, best = sweep_scale_mse(x, _codebook(sw["stages"]), cands, prev)
    ref = np.array(sw["mse"])
    np.testing.assert_allclose(mse.cpu().numpy(), ref, rtol=2e-5)
    assert float(cands[best]) == sw["best"]


def test_sweep_matches_oracle_on_every_candidate():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(512, 8, generator=g)
    cands = torch.linspace(0.05, 2.0, 79)
    prev = [RVQStage(E8PCodebook(), 0.949999988079071)]
    mse, _ = sweep_scale_mse(x.cuda(), RVQCodebookAdapter([RVQStage(E8PCodebook(), 1.25),
                                                           RVQStage(E8OneBitCodebook(), 0.5)]), cands, prev)
    ref = O.sweep_scale_mse(x.numpy(), [("e8p", 1.25), ("e8_1bit", 0.5)], cands.numpy(), True,
                            prev=[("e8p", 0.949999988079071)])
    np.testing.assert_allclose(mse.cpu().numpy(), ref, rtol=1e-5)


@pytest.mark.parametrize("key", ["3bit/0", "4bit/0", "3bit/1"])
def test_build_codebook_matches_reference(key):
    bits, seed = key.split("/")
    cb, scale = C.build_codebook(bits, "cuda", int(seed))
    rec = REF["build_codebook"][key]
    assert [st.scale for st in cb.stages] == rec["stage_scales"]
    assert scale == rec["scale"]


def test_reference_3bit_checkpoint_loads_without_stage_scales():
    d = os.path.join(GOLDEN, "ckpt_ref_3bit")
    assert "stage_scales" not in json.load(open(os.path.join(d, "quip_config.json")))
    model = C.load_quantized_checkpoint(d, device="cuda", model=toy_decoder())
    scales = REF["build_codebook"]["3bit/0"]["stage_scales"]
    kinds = [syn.E8P, syn.E8_1BIT]
    for i, (name, n, m, _) in enumerate(LAYERS):
        q = model.get_submodule(name)
        assert [st.scale for st in q.codebook.stages] == scales
        x = syn.make_activations(2, n, dtype=torch.float16, seed=60 + i)
        y = q(x.cuda())
        torch.cuda.synchronize()
        N.check(N.lib().qs_device_status(N.stream_of(y)))
        t = lambda v: None if v is None else v.detach().cpu().numpy()
        rht = q.transform_kind == "rht"
        ref = O.linear_forward(x.float().numpy(), q.codes.cpu().numpy(), kinds, scales, float(q.scale.item()),
                               q.transform_kind, su=t(q.su) if rht else None, sv=t(q.sv) if rht else None,
                               phase_u=None if rht else t(q.phase_u), phase_v=None if rht else t(q.phase_v),
                               bias=t(q.bias))
        assert rel_l2(y.float().cpu().numpy(), ref) < 2e-3, name
