"""The oracle's restatement of codebook construction (nearest-point search and
the stage-scale sweep, quipsharp/rvq.py:28-66) against the reference's own
per-candidate errors, recorded by tests/golden/make_codebook_scales.py.  The
samples are regenerated from the recorded seeds with torch's CPU generator, as
the reference draws them.  To keep the CPU suite short, each sweep is checked
at the reference's chosen candidate, its neighbours and a few others."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import quipsharp_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_codebook_scales.json")


def _sweeps():
    with open(GOLDEN) as f:
        return json.load(f)["sweeps"]


def _candidates(kind):
    return (torch.linspace(0.5, 4.0, 71) if kind == "stage" else torch.linspace(0.05, 2.0, 79)).numpy()


@pytest.mark.parametrize("i", range(5))
def test_oracle_sweep_matches_reference_errors(i):
    sw = _sweeps()[i]
    g = torch.Generator().manual_seed(sw["seed"])
    x = torch.randn(sw["n_samples"], 8, generator=g).numpy()
    cands = _candidates(sw["kind"])
    ref = np.array(sw["mse"])
    best = int(np.argmin(ref))
    assert float(cands[best]) == sw["best"]
    pick = sorted({0, len(cands) - 1, best, max(best - 1, 0), min(best + 1, len(cands) - 1), len(cands) // 2})
    rvq = len(sw["stages"]) > 1
    got = O.sweep_scale_mse(x, [tuple(s) for s in sw["stages"]], cands[pick], rvq,
                            prev=[tuple(p) for p in sw["prev"]])
    # the reference's means are float32 sums; the oracle sums in float64
    np.testing.assert_allclose(got, ref[pick], rtol=2e-5)
    assert pick[int(np.argmin(got))] == best


def test_recorded_build_codebook_scales_are_candidates():
    with open(GOLDEN) as f:
        built = json.load(f)["build_codebook"]
    stage = set(torch.linspace(0.5, 4.0, 71).tolist())
    resid = set(torch.linspace(0.05, 2.0, 79).tolist())
    for key, rec in built.items():
        s1, s2 = rec["stage_scales"]
        assert s1 in stage and s2 in resid and rec["scale"] in stage, key
