"""CPU-side checks of the C ABI: the library loads, exports every symbol
include/gdn2.h declares, and rejects invalid arguments before any launch."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_header_symbols_are_exported(gdn2):
    lib = gdn2._lib.load()
    with open(os.path.join(ROOT, "include", "gdn2.h")) as f:
        hdr = f.read()
    declared = set(re.findall(r"\b(gdn2_\w+)\s*\(", hdr))
    assert declared, "no declarations found"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in gdn2.h but not exported"
    assert set(gdn2._lib.EXPORTS) <= declared


def test_status_strings_and_version(gdn2):
    lib = gdn2._lib.load()
    assert lib.gdn2_abi_version() >= 100
    assert b"aligned" in lib.gdn2_status_string(5)
    assert lib.gdn2_status_string(0) == b"ok"


def _args(gdn2, **kw):
    a = dict(B=4, T=4096, H=16, K=128, V=128, N=4, NT=256, flags=gdn2._lib.SAVE_FOR_BWD,
             dtype_qkv=gdn2._lib.BF16, dtype_bw=gdn2._lib.F32, scale=128 ** -0.5)
    a.update(kw)
    return gdn2._lib.ChunkArgs(**a)


def test_workspace_sizes(gdn2):
    lib = gdn2._lib.load()
    ws = lib.gdn2_chunk_workspace_size(_args(gdn2))
    tok = 4 * 4096 * 16
    # G fp32 K, Aqk/A 64 bf16 each, Y/U/kg/qg bf16, v_new bf16, chunk states bf16
    assert ws >= tok * (128 * 4 + 2 * 64 * 2 + 4 * 128 * 2 + 128 * 2) + 256 * 16 * 128 * 128 * 2
    assert lib.gdn2_chunk_workspace_size(_args(gdn2, K=96)) == 0
    assert lib.gdn2_chunk_bwd_workspace_size(_args(gdn2)) == 256 * 16 * 128 * 128 * 2 + tok * 128 * 2


def test_segmented_scan_workspace(gdn2):
    """Few (sequence, head) pairs over a long sequence: the plan cuts the scans
    into segments and the workspaces grow by the segment states and
    transitions (fp32 [N*H, nseg, 128, 128] each; the backward one more)."""
    lib = gdn2._lib.load()
    seg = _args(gdn2, B=1, N=1, H=2, NT=33, T=2100)
    tok, nh = 2100 * 2, 2
    plain = lib.gdn2_chunk_bwd_workspace_size(_args(gdn2, B=1, N=1, H=2, NT=16, T=1000))
    assert plain == 16 * 2 * 128 * 128 * 2 + 1000 * 2 * 128 * 2  # 16 chunks: one segment
    fwd, bwd = lib.gdn2_chunk_workspace_size(seg), lib.gdn2_chunk_bwd_workspace_size(seg)
    per = nh * 128 * 128 * 4
    # 11 segments of 3 chunks
    assert bwd == 33 * nh * 128 * 128 * 2 + tok * 128 * 2 + 11 * per
    assert fwd >= 2 * 11 * per
    # many pairs (config 2): one CTA per pair fills the GPU, no segments
    assert lib.gdn2_chunk_bwd_workspace_size(_args(gdn2)) == 256 * 16 * 128 * 128 * 2 + 4 * 4096 * 16 * 128 * 2
    # the chunk states buffer is found through the offset query
    off = lib.gdn2_chunk_workspace_offset(seg, gdn2._lib.WS_CHUNK_STATES)
    assert 0 < off < fwd and off % 256 == 0
    nosave = _args(gdn2, B=1, N=1, H=2, NT=33, T=2100, flags=0)
    assert lib.gdn2_chunk_workspace_offset(nosave, gdn2._lib.WS_CHUNK_STATES) == 2 ** 64 - 1


@pytest.mark.parametrize("kw,code", [
    (dict(K=96), 4), (dict(V=32), 4), (dict(dtype_qkv=1, dtype_bw=0), 3), (dict(dtype_qkv=2), 3),
    (dict(dtype_qkv=1, flags=1 << 9), 7), (dict(NT=255), 2),
    (dict(N=3), 2), (dict(flags=4), 7),
])
def test_invalid_chunk_args_rejected(gdn2, kw, code):
    lib = gdn2._lib.load()
    st = lib.gdn2_chunk_fwd(_args(gdn2, **kw), None, 0, None)
    assert st == code, gdn2._lib.load().gdn2_status_string(st)


def test_null_pointers_and_workspace_rejected(gdn2):
    lib = gdn2._lib.load()
    assert lib.gdn2_chunk_fwd(_args(gdn2), None, 0, None) == 1  # q..o are NULL
    buf = (ctypes.c_char * 64)()
    p = ctypes.addressof(buf)
    p16 = (p + 15) & ~15
    a = _args(gdn2, q=p16, k=p16, v=p16, g=p16, b=p16, w=p16, o=p16)
    assert lib.gdn2_chunk_fwd(a, None, 0, None) == 6  # workspace missing
    a = _args(gdn2, q=p16 + 2, k=p16, v=p16, g=p16, b=p16, w=p16, o=p16)
    assert lib.gdn2_chunk_fwd(a, None, 0, None) == 5  # misaligned


def test_recurrent_args_rejected(gdn2):
    lib = gdn2._lib.load()
    R = gdn2._lib.RecurrentArgs
    assert lib.gdn2_recurrent_fwd(R(B=2, T=1, H=3, HV=4, K=128, V=128, N=2), None) == 2  # HV % H
    assert lib.gdn2_recurrent_fwd(R(B=2, T=1, H=2, HV=2, K=100, V=128, N=2), None) == 4
    assert lib.gdn2_recurrent_fwd(R(B=2, T=1, H=2, HV=2, K=128, V=128, N=2), None) == 1


def test_ops_fail_loudly_without_a_gpu(gdn2):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    x = torch.zeros(1, 64, 1, 64)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        gdn2.chunk_gdn2(x, x, x, x, x, x)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        gdn2.fused_recurrent_gdn2(x, x, x, x, x, x)


def _prep(gdn2, **kw):
    a = dict(rows=0, T=1, N=0, Dk=64, Dv=64, Dfg=64, conv_size=4, proj_stride=3 * 64 + 2 * 64 + 2 * 64,
             b_scale=1.0, flags=0)
    a.update(kw)
    return gdn2._lib.PrepArgs(**a)


@pytest.mark.parametrize("kw,code", [
    (dict(Dk=60), 2), (dict(conv_size=5), 2), (dict(conv_size=1), 2), (dict(proj_stride=100), 2),
    (dict(proj_stride=3 * 64 + 2 * 64 + 2 * 64 + 4), 2), (dict(flags=1), 7),
    (dict(rows=10, T=3, N=3), 2), (dict(rows=8, T=4, N=2), 1),
])
def test_invalid_prep_args_rejected(gdn2, kw, code):
    lib = gdn2._lib.load()
    st = lib.gdn2_layer_prep_fwd(_prep(gdn2, **kw), None)
    assert st == code, lib.gdn2_status_string(st)


def test_prep_state_alias_needs_one_token_per_sequence(gdn2):
    lib = gdn2._lib.load()
    buf = ctypes.create_string_buffer(64)
    p = ctypes.addressof(buf)
    a = _prep(gdn2, rows=8, T=4, N=2, conv_state_in=p, conv_state_out=p, proj=p, q=p, k=p, v=p, b=p, w=p,
              conv_weight=p)
    assert lib.gdn2_layer_prep_fwd(a, None) == 7
    assert lib.gdn2_layer_prep_bwd_workspace_size(_prep(gdn2, rows=512, T=512, N=1)) == \
        4 * (2 * 64 + 64) * 5 * 4  # four row tiles of 128, C conv channels, W taps + bias, fp32
    assert lib.gdn2_layer_prep_bwd_workspace_size(_prep(gdn2, rows=512, T=512, N=1, conv_size=0)) == 0


def test_invalid_norm_gate_args_rejected(gdn2):
    lib = gdn2._lib.load()
    assert lib.gdn2_norm_gate_fwd(None, None, None, 1e-5, 10, 96, None, None, None) == 4
    assert lib.gdn2_norm_gate_fwd(None, None, None, 1e-5, 10, 128, None, None, None) == 1
    assert lib.gdn2_norm_gate_fwd(None, None, None, 1e-5, 0, 128, None, None, None) == 0
    assert lib.gdn2_norm_gate_bwd_workspace_size(10, 128) == 128 * 4
    assert lib.gdn2_norm_gate_bwd_workspace_size(10 ** 6, 128) == 1184 * 128 * 4
