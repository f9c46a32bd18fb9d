"""gdn2_chunk_fwd_static_scratch: the forward for callers that cannot allocate
device memory (engines that reserved the device up front, plugins inside a
framework that owns the allocator, loops that cannot afford an allocation's
implicit synchronisation).  It uses a 32 MiB scratch array built into the
library instead of a caller workspace.

The GPU test calls it through the C ABI twice in a row, on two different
problems, and checks each result against the ordinary entry point
(gdn2_chunk_fwd with a caller-allocated workspace) with the operator's
tolerance.  This file is collected last on purpose."""

import ctypes

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from tolerance import assert_close


def _bind(lib):
    fn = lib.gdn2_chunk_fwd_static_scratch
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _problem(gdn2, seed, B, T, H, K, V, *, bf16_gates, gate, h0):
    L = gdn2._lib
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)  # noqa: E731
    bw = torch.bfloat16 if bf16_gates else torch.float32
    t = dict(q=r(B, T, H, K).bfloat16(), k=r(B, T, H, K).bfloat16(), v=r(B, T, H, V).bfloat16(),
             g=(r(B, T, H, K) if gate else -F.softplus(r(B, T, H, K)) * 0.1).contiguous(),
             b=torch.sigmoid(r(B, T, H, K)).to(bw), w=torch.sigmoid(r(B, T, H, V)).to(bw))
    flags = L.L2NORM_QK | L.STORE_FINAL
    if gate:
        t["A_log"] = torch.rand(H, device="cuda", generator=g) * 2
        t["dt_bias"] = r(H * K) * 0.5
        flags |= L.GATE_IN_KERNEL
    if h0:
        t["h0"] = r(B, H, K, V) * 0.1
        flags |= L.HAS_H0
    return t, flags


def _args(gdn2, t, flags, o, ht):
    L = gdn2._lib
    B, T, H, K = t["q"].shape
    V = t["v"].shape[-1]
    p = lambda n: t[n].data_ptr() if n in t else None  # noqa: E731
    return L.ChunkArgs(B=B, T=T, H=H, K=K, V=V, N=B, NT=B * ((T + 63) // 64),
                       scale=K ** -0.5, flags=flags, dtype_qkv=L.BF16,
                       dtype_bw=L.BF16 if t["b"].dtype == torch.bfloat16 else L.F32,
                       q=p("q"), k=p("k"), v=p("v"), g=p("g"), b=p("b"), w=p("w"),
                       A_log=p("A_log"), dt_bias=p("dt_bias"), h0=p("h0"),
                       ht=ht.data_ptr(), o=o.data_ptr())


@pytest.mark.gpu
def test_static_scratch_forward_matches_workspace_forward(gdn2):
    lib = gdn2._lib.load()
    fwd_static = _bind(lib)
    stream = torch.cuda.current_stream().cuda_stream
    cases = [
        dict(seed=1, B=1, T=1000, H=16, K=128, V=128, bf16_gates=False, gate=False, h0=True),
        dict(seed=2, B=2, T=333, H=4, K=64, V=128, bf16_gates=True, gate=True, h0=False),
    ]
    for c in cases:  # two calls in a row through the shared scratch
        t, flags = _problem(gdn2, **c)
        B, T, H, K = t["q"].shape
        V = t["v"].shape[-1]
        o_ref = torch.empty(B, T, H, V, device="cuda", dtype=torch.bfloat16)
        ht_ref = torch.empty(B, H, K, V, device="cuda")
        a_ref = _args(gdn2, t, flags, o_ref, ht_ref)
        ws = torch.empty(lib.gdn2_chunk_workspace_size(a_ref), device="cuda", dtype=torch.uint8)
        gdn2._lib.check(lib.gdn2_chunk_fwd(a_ref, ws.data_ptr(), ws.numel(), stream), "gdn2_chunk_fwd")

        o = torch.full_like(o_ref, float("nan"))
        ht = torch.full_like(ht_ref, float("nan"))
        a = _args(gdn2, t, flags, o, ht)
        st = fwd_static(ctypes.addressof(a), stream)
        assert st == 0, lib.gdn2_status_string(st)
        torch.cuda.synchronize()
        assert_close(o, o_ref, f"o (case seed={c['seed']})")
        assert_close(ht, ht_ref, f"ht (case seed={c['seed']})")


def test_static_scratch_rejects_oversized_and_backward_contexts(gdn2):
    """Checked before any device work, so this runs without a GPU too."""
    lib = gdn2._lib.load()
    fwd_static = _bind(lib)
    L = gdn2._lib
    buf = (ctypes.c_char * 64)()
    p = (ctypes.addressof(buf) + 15) & ~15
    big = L.ChunkArgs(B=1, T=4096, H=16, K=128, V=128, N=1, NT=64, scale=0.088,
                      flags=0, dtype_qkv=L.BF16, dtype_bw=L.F32,
                      q=p, k=p, v=p, g=p, b=p, w=p, o=p)
    assert lib.gdn2_chunk_workspace_size(big) > 32 << 20
    assert fwd_static(ctypes.addressof(big), None) == 9
    assert b"32 MiB" in lib.gdn2_status_string(9)
    small = L.ChunkArgs(B=1, T=64, H=1, K=128, V=128, N=1, NT=1, scale=0.088,
                        flags=L.SAVE_FOR_BWD, dtype_qkv=L.BF16, dtype_bw=L.F32,
                        q=p, k=p, v=p, g=p, b=p, w=p, o=p)
    assert fwd_static(ctypes.addressof(small), None) == 7
    assert np.isfinite(lib.gdn2_chunk_workspace_size(small))
    # reusing intra-chunk factors is refused: the shared array may hold another problem's
    skip = L.ChunkArgs.from_buffer_copy(small)
    skip.flags = L.SKIP_INTRA
    assert fwd_static(ctypes.addressof(skip), None) == 7
