"""Record the REFERENCE's codebook-construction results (numbersletter/quipsharp,
checkpoint.py:60-77 build_codebook; rvq.py:28-66 fit_stage_scale /
fit_residual_stage_scale) into reference_codebook_scales.json.

Usage (needs a checkout of the reference; it is not needed to run the tests):

    python tests/golden/make_codebook_scales.py /path/to/quipsharp-reference

Writes:
  * "build_codebook": for each (bits, seed) the two RVQ stage scales and the
    returned input scale, as the reference computes them on the CPU with its
    default sample counts (20,000 Gaussian 8-vectors per sweep);
  * "sweeps": small sweeps (2,000 samples) with the per-candidate mean squared
    error each candidate scale gives, computed with the reference's own
    quantize functions in the order of rvq.py:28-37, and the chosen scale.
"""
from __future__ import annotations

import json
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from quipsharp.checkpoint import build_codebook
    from quipsharp.codebooks.e8p import E8PCodebook
    from quipsharp.codebooks.e8_1bit import E8OneBitCodebook
    from quipsharp.quantize import RVQCodebookAdapter
    from quipsharp.rvq import RVQStage, rvq_quantize, fit_stage_scale, fit_residual_stage_scale

    cbs = {"e8p": E8PCodebook(), "e8_1bit": E8OneBitCodebook()}

    def mses(x, codebook, candidates):
        out = []
        for s in candidates:
            s = s.item()
            vals, _ = codebook.quantize(x / s)
            out.append((x - vals * s).pow(2).mean().item())
        return out

    sweeps = []
    n = 2000
    stage_c = torch.linspace(0.5, 4.0, 71)
    resid_c = torch.linspace(0.05, 2.0, 79)
    for name, seed in (("e8p", 5), ("e8_1bit", 9)):
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(n, 8, generator=g)
        best = fit_stage_scale(cbs[name], n_samples=n, seed=seed)
        sweeps.append({"kind": "stage", "prev": [], "stages": [[name, 1.0]], "seed": seed, "n_samples": n,
                       "mse": mses(x, cbs[name], stage_c), "best": best})
    for second, seed in (("e8_1bit", 6), ("e8p", 8)):
        prev = [RVQStage(cbs["e8p"], 0.949999988079071)]
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(n, 8, generator=g)
        vals, _ = rvq_quantize(x, prev)
        best = fit_residual_stage_scale(prev, cbs[second], n_samples=n, seed=seed)
        sweeps.append({"kind": "residual", "prev": [["e8p", 0.949999988079071]], "stages": [[second, 1.0]],
                       "seed": seed, "n_samples": n, "mse": mses(x - vals, cbs[second], resid_c), "best": best})
    rvq = RVQCodebookAdapter([RVQStage(cbs["e8p"], 0.949999988079071), RVQStage(cbs["e8_1bit"], 0.5)])
    g = torch.Generator().manual_seed(7)
    x = torch.randn(n, 8, generator=g)
    sweeps.append({"kind": "stage", "prev": [], "stages": [["e8p", 0.949999988079071], ["e8_1bit", 0.5]],
                   "seed": 7, "n_samples": n, "mse": mses(x, rvq, stage_c),
                   "best": fit_stage_scale(rvq, n_samples=n, seed=7)})

    built = {}
    for bits, seed in (("3bit", 0), ("4bit", 0), ("3bit", 1)):
        t0 = time.time()
        cb, scale = build_codebook(bits, "cpu", seed)
        built[f"{bits}/{seed}"] = {"stage_scales": [st.scale for st in cb.stages], "scale": scale}
        print(bits, seed, built[f"{bits}/{seed}"], f"{time.time() - t0:.0f} s", flush=True)

    out = os.path.join(HERE, "reference_codebook_scales.json")
    with open(out, "w") as f:
        json.dump({"build_codebook": built, "sweeps": sweeps}, f, indent=1)
    print("wrote", out)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QUIPSHARP_REF", ""))
