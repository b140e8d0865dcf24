"""GPU parity of a checkpoint written by the reference (tests/golden/ckpt_ref_*):
after load_quantized_checkpoint every quantized module's fused CUDA forward
matches the oracle on the loaded buffers (tolerances as in test_gpu_linear)."""
import json
import os
import sys

import pytest
import torch

from oracle import quipsharp_oracle as O
from quipsharp_b200 import checkpoint as C
from quipsharp_b200 import _native as N
from quipsharp_b200 import synthetic as syn
from conftest import rel_l2
from test_gpu_linear import TOL

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLDEN)
from make_ckpt_fixture import toy_decoder, LAYERS  # noqa: E402


@pytest.mark.parametrize("bits,dt", [("2bit", torch.float16), ("3bit", torch.bfloat16)])
def test_loaded_checkpoint_forward_vs_oracle(bits, dt):
    d = os.path.join(GOLDEN, f"ckpt_ref_{bits}")
    kinds = [syn.E8P] if bits == "2bit" else [syn.E8P, syn.E8_1BIT]
    scales = json.load(open(os.path.join(d, "stage_scales.json"))) if bits == "3bit" else None
    model = C.load_quantized_checkpoint(d, device="cuda", model=toy_decoder(),
                                        codebook=C.codebook_for(bits, scales))
    for i, (name, n, m, _) in enumerate(LAYERS):
        q = model.get_submodule(name)
        assert q._kernel is not None  # packed at load time
        x = syn.make_activations(3, n, dtype=dt, seed=20 + i)
        y = q(x.cuda())
        torch.cuda.synchronize()
        N.check(N.lib().qs_device_status(N.stream_of(y)))
        t = lambda v: None if v is None else v.detach().cpu().numpy()
        rht = q.transform_kind == "rht"
        ref = O.linear_forward(x.float().numpy(), q.codes.cpu().numpy(), kinds, scales, float(q.scale.item()),
                               q.transform_kind, su=t(q.su) if rht else None, sv=t(q.sv) if rht else None,
                               phase_u=None if rht else t(q.phase_u), phase_v=None if rht else t(q.phase_v),
                               bias=t(q.bias))
        assert y.shape == (3, m) and y.dtype == dt
        assert rel_l2(y.float().cpu().numpy(), ref) < TOL[dt], name
