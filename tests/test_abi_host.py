"""C-ABI library and host-side logic (no GPU needed): the library loads, exports
every entry point the header declares, reports the compiled-in tables, sizes
and argument errors; the Python layer raises the reference's exception types."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

from conftest import ROOT
from quipsharp_b200 import _native as N


def header_symbols():
    text = open(os.path.join(ROOT, "include", "quipsharp_b200.h")).read()
    return sorted(set(re.findall(r"\b(qs_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    lib = N.lib()
    syms = header_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(N.EXPORTS)


def test_version_and_tables(golden):
    assert b"sm_100a" in N.lib().qs_version()
    buf = (ctypes.c_float * 2048)()
    N.check(N.lib().qs_codebook_table(N.QS_CB_E8P, buf))
    assert np.array_equal(np.frombuffer(buf, np.float32).reshape(256, 8), golden["abs_table"])
    N.check(N.lib().qs_codebook_table(N.QS_CB_E8_1BIT, buf))
    assert np.array_equal(np.frombuffer(buf, np.float32).reshape(256, 8), golden["onebit_table"])
    assert N.lib().qs_codebook_table(7, buf) == N.QS_ERR_INVALID_ARG


def test_python_tables_match_reference(golden):
    from quipsharp_b200.codebooks.e8p import build_abs_table, _enumerate_d8hat_abs_le_norm10
    from quipsharp_b200.codebooks.e8_1bit import build_table, _norm2_shell
    assert np.array_equal(build_abs_table().numpy(), golden["abs_table"])
    assert np.array_equal(_enumerate_d8hat_abs_le_norm10().numpy(), golden["raw227"])
    assert np.array_equal(build_table().numpy(), golden["onebit_table"])
    assert _norm2_shell().shape == (240, 8)


def test_sizes():
    lib = N.lib()
    k = N.int_array([N.QS_CB_E8P, N.QS_CB_E8_1BIT])
    # 3-bit RVQ 4096 -> 11008: E8P 2 bits/weight + 1-bit stage 1 bit/weight
    assert lib.qs_packed_bytes(2, k, 11008, 4096) == 11008 * 4096 // 4 + 11008 * 4096 // 8
    assert lib.qs_packed_bytes(1, k, 4096, 4096) == 4096 * 4096 // 4
    assert lib.qs_packed_bytes(1, k, 10, 24) > 0          # padded to 16 rows x 256 features
    assert lib.qs_packed_bytes(1, k, 10, 20) == -1        # n not a multiple of 8
    assert lib.qs_packed_bytes(3, k, 16, 256) == -1
    assert lib.qs_linear_workspace_bytes(1, 4096, 4096) > 0
    assert lib.qs_linear_input_bytes(0, 4096) >= 0


def test_argument_errors_without_gpu():
    lib = N.lib()
    k = N.int_array([N.QS_CB_E8P])
    assert lib.qs_fwht(None, 3, None, 3, N.QS_F32, 1, 3, None, None, None) == N.QS_ERR_NOT_POW2
    assert lib.qs_fwht(None, 65536, None, 65536, N.QS_F32, 1, 65536, None, None, None) == N.QS_ERR_UNSUPPORTED
    assert lib.qs_rfft(0, None, 7, None, 7, N.QS_F32, 1, 7, None, None) == N.QS_ERR_ODD_DIM
    assert lib.qs_rfft(0, None, 2 * 47, None, 2 * 47, N.QS_F32, 1, 2 * 47, None, None) == N.QS_ERR_UNSUPPORTED
    assert lib.qs_decode(5, None, N.QS_I64, 1, None, None) == N.QS_ERR_INVALID_ARG
    assert lib.qs_decode(0, None, N.QS_I64, 0, None, None) == N.QS_OK  # empty input is a no-op
    assert lib.qs_pack_codes(None, 1, k, 16, 256, None, 0, None) == N.QS_ERR_INVALID_ARG
    assert lib.qs_linear_fwd(None, N.QS_F16, 1, 4096, 4096, None, 1, k, None, None, N.QS_RHT,
                             None, None, None, None, None, None, None, 0, None) == N.QS_ERR_INVALID_ARG
    assert lib.qs_linear_fwd(None, N.QS_F16, 1, 4096, 4000, None, 1, k, None, None, N.QS_RHT,
                             None, None, None, None, None, None, None, 0, None) == N.QS_ERR_NOT_POW2
    assert b"power-of-two" in lib.qs_last_error()


def test_python_layer_errors_match_reference():
    from quipsharp_b200.hadamard import fwht
    from quipsharp_b200.rfft import to_transformed_space
    from quipsharp_b200.codebooks import E8PCodebook
    with pytest.raises(ValueError):
        fwht(torch.randn(3))
    with pytest.raises(AssertionError):
        to_transformed_space(torch.randn(2, 7), torch.ones(3, dtype=torch.complex64))
    # no CPU path: CPU tensors are refused rather than computed some other way
    with pytest.raises(RuntimeError, match="CUDA"):
        fwht(torch.randn(4, 8))
    with pytest.raises(RuntimeError, match="CUDA"):
        E8PCodebook().dequantize(torch.tensor([1, 2]))
    with pytest.raises(NotImplementedError):
        E8PCodebook().quantize(torch.randn(2, 8))


def test_pack_unpack_round_trip():
    """tests/test_e8p.py:72-83 of the reference, on the package's helpers."""
    from quipsharp_b200.codebooks.e8p import pack_code, unpack_code
    torch.manual_seed(0)
    abs_idx = torch.randint(0, 256, (500,))
    sign_bits7 = torch.randint(0, 2, (500, 7))
    shift_bit = torch.randint(0, 2, (500,))
    code = pack_code(abs_idx, sign_bits7, shift_bit)
    assert code.min() >= 0 and code.max() < (1 << 16)
    a2, s2, sh2 = unpack_code(code)
    assert torch.equal(a2, abs_idx) and torch.equal(s2, sign_bits7) and torch.equal(sh2, shift_bit)


def test_quantized_linear_state_dict_keys_match_reference():
    from quipsharp_b200.checkpoint import QuantizedLinear
    m = QuantizedLinear(64, 32, 8, "rht", num_stages=2, has_bias=True)
    assert set(m.state_dict()) == {"bias", "codes", "scale", "su", "sv"}
    assert m.codes.shape == (2, 32, 8) and m.codes.dtype == torch.int16
    r = QuantizedLinear(48, 40, 8, "rfft")
    assert set(r.state_dict()) == {"codes", "scale", "phase_u", "phase_v"}
    assert r.phase_u.dtype == torch.complex64 and r.phase_u.shape == (20,)


def test_tp_peers_struct_matches_the_header(tmp_path):
    """The ctypes mirror of qs_tp_peers has the C layout of include/quipsharp_b200.h
    (compiled here with the host compiler), and the exchange allocation's layout
    helpers give 16-byte aligned control words after the padded flags."""
    import shutil
    import subprocess
    from quipsharp_b200.tensor_parallel import exchange_floats, ctl_offset, make_peers
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no host C compiler")
    src = tmp_path / "peers.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "quipsharp_b200.h"\n'
        "int main(void) {\n"
        '  printf("%zu %zu %zu %zu %zu %zu %d\\n", sizeof(qs_tp_peers), offsetof(qs_tp_peers, rank),\n'
        "         offsetof(qs_tp_peers, recv), offsetof(qs_tp_peers, flags), offsetof(qs_tp_peers, ctl),\n"
        "         offsetof(qs_tp_peers, recv_floats), QS_TP_MAX_RANKS);\n"
        "  return 0;\n}\n")
    exe = tmp_path / "peers"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    P = N.TPPeers
    assert got == [ctypes.sizeof(P), P.rank.offset, P.recv.offset, P.flags.offset, P.ctl.offset,
                   P.recv_floats.offset, N.QS_TP_MAX_RANKS]
    for world in range(1, 9):
        cap = 1 << 16
        assert (ctl_offset(cap, world) * 4) % 16 == 0 and ctl_offset(cap, world) >= 2 * cap + 2 * world
        assert exchange_floats(cap, world) == ctl_offset(cap, world) + 4
        bases = [0x10000 * (r + 1) * 4096 for r in range(world)]
        pe = make_peers(world, world - 1, bases, cap)
        assert pe.flags[0] == bases[0] + 2 * cap * 4 and pe.ctl == bases[-1] + ctl_offset(cap, world) * 4


def _group_layer(m, ws, y, k, fake=0x100000):
    """A qs_linear_layer with well-formed (never dereferenced) device pointers."""
    L = N.LinearLayer()
    L.m, L.packed, L.stages, L.kinds = m, fake, 1, ctypes.cast(k, ctypes.c_void_p)
    L.layer_scale, L.transform, L.su, L.sv = fake, N.QS_RHT, fake, fake
    L.y, L.workspace, L.workspace_bytes = y, ws, N.lib().qs_linear_workspace_bytes(1, m, 4096)
    return L


def test_linear_group_struct_and_checks(tmp_path):
    """qs_linear_layer's ctypes mirror has the header's C layout; qs_linear_fwd_group
    validates every layer (and that no two share memory) before launching."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no host C compiler")
    fields = [f for f, _ in N.LinearLayer._fields_]
    src = tmp_path / "layer.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "quipsharp_b200.h"\n'
        "int main(void) {\n"
        '  printf("%zu %d\\n", sizeof(qs_linear_layer), QS_GROUP_MAX_LAYERS);\n'
        + "".join(f'  printf("%zu\\n", offsetof(qs_linear_layer, {f}));\n' for f in fields)
        + "  return 0;\n}\n")
    exe = tmp_path / "layer"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    assert got == [ctypes.sizeof(N.LinearLayer), N.QS_GROUP_MAX_LAYERS] + \
        [getattr(N.LinearLayer, f).offset for f in fields]

    lib = N.lib()
    k = N.int_array([N.QS_CB_E8P])
    MB = 1 << 20
    a = _group_layer(4096, 0x10000000, 0x20000000, k)
    b = _group_layer(1024, 0x10000000 + 64 * MB, 0x20000000 + 64 * MB, k)
    arr = (N.LinearLayer * 2)(a, b)
    assert lib.qs_linear_fwd_group(0x30000000, N.QS_F16, 1, 4096, 0, arr, None) == N.QS_ERR_INVALID_ARG
    assert lib.qs_linear_fwd_group(0x30000000, N.QS_F16, 1, 4096, 9, arr, None) == N.QS_ERR_INVALID_ARG
    assert lib.qs_linear_fwd_group(0x30000000, N.QS_F16, 0, 4096, 2, arr, None) == N.QS_OK  # empty batch
    bad = (N.LinearLayer * 2)(a, _group_layer(1000, 0x10000000 + 64 * MB, 0x20000000 + 64 * MB, k))
    assert lib.qs_linear_fwd_group(0x30000000, N.QS_F16, 1, 4096, 2, bad, None) == N.QS_ERR_NOT_POW2
    small = _group_layer(1024, 0x10000000 + 64 * MB, 0x20000000 + 64 * MB, k)
    small.workspace_bytes = 16
    arr2 = (N.LinearLayer * 2)(a, small)
    assert lib.qs_linear_fwd_group(0x30000000, N.QS_F16, 1, 4096, 2, arr2, None) == N.QS_ERR_WORKSPACE
    for shared in (dict(workspace=a.workspace + 256), dict(y=a.y), dict(y=a.workspace)):
        c = _group_layer(1024, 0x10000000 + 64 * MB, 0x20000000 + 64 * MB, k)
        for f, v in shared.items():
            setattr(c, f, v)
        arr3 = (N.LinearLayer * 2)(a, c)
        assert lib.qs_linear_fwd_group(0x30000000, N.QS_F16, 1, 4096, 2, arr3, None) == N.QS_ERR_INVALID_ARG
        assert b"share" in lib.qs_last_error()
