"""Chunkwise GDN2 with the reference's Python interface and autograd contract.

Mirrors ``lit_gpt/gdn2_ops/chunk_gdn2.py``: ``chunk_gdn2`` (:1363-1511,
same arguments, validation and return values) and ``ChunkGDN2Function``
(:2504-2665, same forward argument list and the same gradient list:
dq, dk, dv, dg, db, dw, dA_log, dt_bias, dh0).  Forward and backward are
single calls into ``gdn2_chunk_fwd`` / ``gdn2_chunk_bwd`` of
libgdn2_b200.so; the forward keeps what the backward needs in one
workspace tensor instead of recomputing it.
"""

from __future__ import annotations

import torch

from . import _lib

CHUNK = 64


def prepare_chunk_indices(cu_seqlens: torch.Tensor, cu_seqlens_cpu: torch.Tensor | None = None):
    """(chunk_index [NT, 2] int32 = (sequence, chunk in sequence),
    chunk_offset [N+1] int32, NT) for a packed batch, as the reference's
    ``prepare_chunk_indices`` / ``prepare_chunk_offsets`` (fla ops/utils/index.py)."""
    cpu = cu_seqlens_cpu if cu_seqlens_cpu is not None else cu_seqlens.detach().cpu()
    lens = (cpu[1:] - cpu[:-1]).to(torch.int64)
    nchunks = (lens + CHUNK - 1) // CHUNK
    offs = torch.zeros(len(lens) + 1, dtype=torch.int64)
    offs[1:] = torch.cumsum(nchunks, 0)
    NT = int(offs[-1])
    seq = torch.repeat_interleave(torch.arange(len(lens)), nchunks)
    within = torch.arange(NT) - offs[:-1][seq] if NT > 0 else torch.zeros(0, dtype=torch.int64)
    idx = torch.stack([seq, within], 1).to(torch.int32)
    dev = cu_seqlens.device
    return idx.to(dev, non_blocking=True), offs.to(torch.int32).to(dev, non_blocking=True), NT


def _bw_dtype(b: torch.Tensor, w: torch.Tensor) -> torch.dtype:
    if b.dtype == w.dtype and b.dtype in (torch.bfloat16, torch.float32):
        return b.dtype
    return torch.float32


def _make_args(q, k, v, g, b, w, A_log, dt_bias, scale, initial_state, ht, o, flags,
               lower_bound, geom):
    B, T, H, K = q.shape
    V = v.shape[-1]
    cu, cidx, coff, N, NT = geom
    return _lib.ChunkArgs(
        B=B, T=T, H=H, K=K, V=V, N=N, NT=NT,
        cu_seqlens=_lib.ptr(cu), chunk_index=_lib.ptr(cidx), chunk_offset=_lib.ptr(coff),
        scale=float(scale), lower_bound=float(lower_bound if lower_bound is not None else 0.0),
        flags=flags, dtype_qkv=_lib.F32 if q.dtype == torch.float32 else _lib.BF16,
        dtype_bw=_lib.BF16 if b.dtype == torch.bfloat16 else _lib.F32,
        q=_lib.ptr(q), k=_lib.ptr(k), v=_lib.ptr(v), g=_lib.ptr(g), b=_lib.ptr(b), w=_lib.ptr(w),
        A_log=_lib.ptr(A_log), dt_bias=_lib.ptr(dt_bias), h0=_lib.ptr(initial_state),
        ht=_lib.ptr(ht), o=_lib.ptr(o),
    )


def _chunk_forward(q, k, v, g, b, w, A_log, dt_bias, scale, initial_state, output_final_state,
                   use_qk_l2norm_in_kernel, use_gate_in_kernel, cu_seqlens, cu_seqlens_cpu,
                   lower_bound, transpose_state_layout, save):
    """One ``gdn2_chunk_fwd`` call.  Returns (o, ht, saved, meta, ws, args):
    ``saved`` and ``meta`` are what ``_chunk_backward`` needs (``save`` keeps
    the backward's operands in the workspace)."""
    _lib.require_device(q)
    dtypes = (q.dtype, k.dtype, v.dtype, g.dtype, b.dtype, w.dtype)
    # fp32 q: the fp32 path (every input in fp32, the recurrence in fp32);
    # otherwise the bf16 tensor-core path with fp32 accumulation
    fp32 = q.dtype == torch.float32
    cdt = torch.float32 if fp32 else torch.bfloat16
    bw = torch.float32 if fp32 else _bw_dtype(b, w)
    qb, kb, vb = (x.to(cdt).contiguous() for x in (q, k, v))
    # bf16 g (the layer's gate pre-activation) is read as is on the bf16 path; anything else as fp32
    gf = g.contiguous() if (g.dtype == torch.bfloat16 and not fp32) else g.to(torch.float32).contiguous()
    bb, wb = b.to(bw).contiguous(), w.to(bw).contiguous()
    A_log_f = A_log.float().contiguous() if (use_gate_in_kernel and A_log is not None) else None
    dt_f = dt_bias.float().contiguous() if (use_gate_in_kernel and dt_bias is not None) else None
    B, T, H, K = q.shape
    V = v.shape[-1]
    if cu_seqlens is not None:
        cu = cu_seqlens.to(torch.int64).contiguous()
        cidx, coff, NT = prepare_chunk_indices(cu, cu_seqlens_cpu)
        N = len(cu_seqlens) - 1
    else:
        cu = cidx = coff = None
        N = B
        NT = B * ((T + CHUNK - 1) // CHUNK)
    geom = (cu, cidx, coff, N, NT)
    flags = _lib.G_BF16 if gf.dtype == torch.bfloat16 else 0
    if use_qk_l2norm_in_kernel:
        flags |= _lib.L2NORM_QK
    if use_gate_in_kernel:
        flags |= _lib.GATE_IN_KERNEL
        if lower_bound is not None:
            flags |= _lib.LOWER_BOUND
    if transpose_state_layout:
        flags |= _lib.TRANSPOSE_STATE
    h0 = None
    if initial_state is not None:
        h0 = initial_state.contiguous()
        flags |= _lib.HAS_H0
    if save:
        flags |= _lib.SAVE_FOR_BWD
    o = torch.empty(B, T, H, V, device=q.device, dtype=cdt)
    ht = None
    if output_final_state:
        shp = (N, H, V, K) if transpose_state_layout else (N, H, K, V)
        ht = torch.empty(shp, device=q.device, dtype=torch.float32)
        flags |= _lib.STORE_FINAL
    lb = lower_bound if (flags & _lib.LOWER_BOUND) else None
    args = _make_args(qb, kb, vb, gf, bb, wb, A_log_f, dt_f, scale, h0, ht, o, flags, lb, geom)
    lib = _lib.load()
    ws_bytes = lib.gdn2_chunk_workspace_size(args)
    ws = torch.empty(max(ws_bytes, 1), device=q.device, dtype=torch.uint8)
    with torch.cuda.device(q.device):
        _lib.check(lib.gdn2_chunk_fwd(args, ws.data_ptr(), ws_bytes, _lib.stream_ptr(q.device)),
                   "gdn2_chunk_fwd")
    o_out = o if dtypes[0] == cdt else o.to(dtypes[0])
    saved = (qb, kb, vb, gf, bb, wb, A_log_f, dt_f, h0, ws, cu, cidx, coff)
    meta = (flags, float(scale), lb, N, NT, ws_bytes, dtypes,
            A_log.dtype if A_log is not None else None,
            dt_bias.dtype if dt_bias is not None else None,
            initial_state is not None)
    return o_out, ht, saved, meta, ws, args


def _chunk_backward(saved, meta, do, dht, state_only=False):
    """One ``gdn2_chunk_bwd`` call on a forward's saved state.  Returns the
    gradient tuple of ``ChunkGDN2Function.backward`` or, with ``state_only``,
    only d(loss)/d(initial state) for the given do and dht (the state-cotangent
    scan alone; the initial state's layout follows the forward's)."""
    (qb, kb, vb, gf, bb, wb, A_log_f, dt_f, h0, ws, cu, cidx, coff) = saved
    (flags, scale, lb, N, NT, ws_bytes, dtypes, A_dtype, dt_dtype, has_h0) = meta
    B, T, H, K = qb.shape
    V = vb.shape[-1]
    dev = qb.device
    geom = (cu, cidx, coff, N, NT)
    bflags = flags & ~_lib.STORE_FINAL
    if state_only:
        bflags |= _lib.BWD_STATE_ONLY
    args = _make_args(qb, kb, vb, gf, bb, wb, A_log_f, dt_f, scale, h0, None, None, bflags, lb, geom)
    dob = do.to(qb.dtype).contiguous()
    dht_f = dht.to(torch.float32).contiguous() if dht is not None else None
    tr = bool(flags & _lib.TRANSPOSE_STATE)
    if state_only:
        dh0 = torch.empty((N, H, V, K) if tr else (N, H, K, V), device=dev, dtype=torch.float32)
        grads = _lib.ChunkGrads(dout=_lib.ptr(dob), dht=_lib.ptr(dht_f), dh0=_lib.ptr(dh0))
    else:
        dq = torch.empty_like(qb)
        dk = torch.empty_like(kb)
        dv = torch.empty_like(vb)
        dg = torch.empty_like(gf)
        db = torch.empty_like(bb)
        dw = torch.empty_like(wb)
        dh0 = torch.empty_like(h0) if has_h0 else None
        gated = bool(flags & _lib.GATE_IN_KERNEL)
        dA = torch.zeros(H, device=dev, dtype=torch.float32) if gated else None
        ddt = torch.zeros(H * K, device=dev, dtype=torch.float32) if (gated and dt_f is not None) else None
        grads = _lib.ChunkGrads(
            dout=_lib.ptr(dob), dht=_lib.ptr(dht_f), dq=_lib.ptr(dq), dk=_lib.ptr(dk),
            dv=_lib.ptr(dv), dg=_lib.ptr(dg), db=_lib.ptr(db), dw=_lib.ptr(dw),
            dh0=_lib.ptr(dh0), dA_log=_lib.ptr(dA), ddt_bias=_lib.ptr(ddt))
    lib = _lib.load()
    bws_bytes = lib.gdn2_chunk_bwd_workspace_size(args)
    bws = torch.empty(max(bws_bytes, 1), device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        _lib.check(lib.gdn2_chunk_bwd(args, grads, ws.data_ptr(), ws_bytes, bws.data_ptr(),
                                      bws_bytes, _lib.stream_ptr(dev)), "gdn2_chunk_bwd")
    if state_only:
        return dh0
    qd, kd, vd, gd, bd, wd = dtypes
    return (dq.to(qd), dk.to(kd), dv.to(vd), dg.to(gd), db.to(bd), dw.to(wd),
            dA.to(A_dtype) if dA is not None else None,
            ddt.to(dt_dtype) if ddt is not None else None,
            dh0)


class ChunkGDN2Function(torch.autograd.Function):
    """Autograd wrapper; forward signature as the reference's
    ``ChunkGDN2Function.forward`` (``chunk_gdn2.py:2515-2536``)."""

    @staticmethod
    def forward(ctx, q, k, v, g, b, w, A_log, dt_bias, scale, initial_state,
                output_final_state, use_qk_l2norm_in_kernel, use_gate_in_kernel,
                cu_seqlens, cu_seqlens_cpu, safe_gate, lower_bound, disable_recompute,
                return_intermediate_states, transpose_state_layout):
        need_grad = any(ctx.needs_input_grad[i] for i in (0, 1, 2, 3, 4, 5, 6, 7, 9))
        o_out, ht, saved, meta, ws, args = _chunk_forward(
            q, k, v, g, b, w, A_log, dt_bias, scale, initial_state, output_final_state,
            use_qk_l2norm_in_kernel, use_gate_in_kernel, cu_seqlens, cu_seqlens_cpu, lower_bound,
            transpose_state_layout, need_grad or return_intermediate_states)
        if return_intermediate_states:
            assert torch.is_inference_mode_enabled(), (
                "return_intermediate_states is only allowed in inference mode")
            B, T, H, K = q.shape
            h = _intermediate_states(ws, args, B, T, H, K, v.shape[-1], meta[4], transpose_state_layout)
            return o_out, ht, h
        ctx.save_for_backward(*saved)
        ctx.meta = meta
        return o_out, ht

    @staticmethod
    def backward(ctx, do, dht):
        g = _chunk_backward(ctx.saved_tensors, ctx.meta, do, dht)
        return g[:8] + (None, g[8], None, None, None, None, None, None, None, None, None, None)


def _intermediate_states(ws, args, B, T, H, K, V, NT, transpose):
    """The per-chunk entering states h [B, NT_per_seq, H, K, V] (bf16), as the
    reference returns them with ``return_intermediate_states``."""
    off = _lib.load().gdn2_chunk_workspace_offset(args, _lib.WS_CHUNK_STATES)
    if off == 2 ** 64 - 1:
        raise RuntimeError("the forward workspace keeps no chunk states for these arguments")
    if args.dtype_qkv == _lib.F32:
        # the fp32 path keeps them in fp32, [NT, H, K, V]
        hs = ws[off:off + NT * H * K * V * 4].view(torch.float32).view(NT, H, K, V)
        h = (hs.transpose(-1, -2) if transpose else hs).contiguous()
    else:
        # the bf16 path keeps each chunk state transposed, [NT, H, V, K]
        hT = ws[off:off + NT * H * K * V * 2].view(torch.bfloat16).view(NT, H, V, K)
        h = (hT if transpose else hT.transpose(-1, -2)).contiguous()
    if args.cu_seqlens is None:
        return h.view(B, NT // max(B, 1), H, *h.shape[-2:])
    return h.unsqueeze(0)


@torch.compiler.disable
def chunk_gdn2(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    b: torch.Tensor,
    w: torch.Tensor,
    scale: float | None = None,
    initial_state: torch.Tensor | None = None,
    output_final_state: bool = False,
    use_qk_l2norm_in_kernel: bool = False,
    use_gate_in_kernel: bool = False,
    cu_seqlens: torch.LongTensor | None = None,
    cu_seqlens_cpu: torch.LongTensor | None = None,
    safe_gate: bool = False,
    lower_bound: float | None = None,
    disable_recompute: bool = False,
    return_intermediate_states: bool = False,
    transpose_state_layout: bool = False,
    **kwargs,
):
    r"""Chunkwise forward for GDN2 (drop-in for the reference's ``chunk_gdn2``).

    q, k, g, b: ``[B, T, H, K]``; v, w: ``[B, T, H, V]``; ``initial_state``
    ``[N, H, K, V]`` fp32; ``g`` is the natural-log decay, or the raw
    pre-activation with ``use_gate_in_kernel`` (then ``A_log`` and optional
    ``dt_bias`` come through ``kwargs``).  Returns ``(o, final_state)`` or,
    with ``return_intermediate_states``, ``(o, final_state, h)``.
    ``disable_recompute`` is accepted for compatibility: the forward always
    keeps what the backward needs.
    """
    if cu_seqlens is not None:
        if q.shape[0] != 1:
            raise ValueError(
                f"The batch size is expected to be 1 rather than {q.shape[0]} "
                f"when using `cu_seqlens`. Please flatten variable-length "
                f"inputs before processing.",
            )
        if initial_state is not None and initial_state.shape[0] != len(cu_seqlens) - 1:
            raise ValueError(
                f"The number of initial states is expected to be equal to the "
                f"number of input sequences, i.e., {len(cu_seqlens) - 1} rather "
                f"than {initial_state.shape[0]}.",
            )
    if initial_state is not None:
        assert initial_state.dtype == torch.float32, "initial_state must be in float32."

    A_log, dt_bias = None, None
    if use_gate_in_kernel:
        assert "A_log" in kwargs, "A_log must be provided when use_gate_in_kernel=True."
        A_log, dt_bias = kwargs["A_log"], kwargs.get("dt_bias")

    if safe_gate and use_gate_in_kernel:
        if lower_bound is None:
            raise ValueError(
                "`lower_bound` must be specified when `safe_gate=True` and "
                "`use_gate_in_kernel=True`.")
        if not (-5 <= lower_bound < 0):
            raise ValueError(f"`lower_bound` must be in the safe range [-5, 0), got {lower_bound}.")

    assert q.shape == k.shape == g.shape, "q, k, g must have the same shape."
    assert k.shape[-1] <= 256, "Currently we only support key headdim <=256 for GDN-2 :-("
    assert b.shape == q.shape, (
        "b (channel-wise erase gate) must have shape [B, T, H, K] matching q; "
        f"got {tuple(b.shape)} vs q {tuple(q.shape)}."
    )
    assert w.shape == v.shape, (
        "w (channel-wise write gate) must have shape [B, T, H, V] matching v; "
        f"got {tuple(w.shape)} vs v {tuple(v.shape)}."
    )
    assert v.shape == (*q.shape[:3], v.shape[-1]), (
        "v must be of shape (batch size, seq len, num of head, head dim)."
    )
    if scale is None:
        scale = k.shape[-1] ** -0.5

    return ChunkGDN2Function.apply(
        q, k, v, g, b, w, A_log, dt_bias, scale, initial_state, output_final_state,
        use_qk_l2norm_in_kernel, use_gate_in_kernel, cu_seqlens, cu_seqlens_cpu,
        safe_gate, lower_bound, disable_recompute, return_intermediate_states,
        transpose_state_layout,
    )


def gdn2_telemetry_snapshot(reset: bool = True) -> dict:
    """Interface twin of the reference's ``gdn2_telemetry_snapshot``
    (``chunk_gdn2.py:134-153``), which trainers import next to ``chunk_gdn2``.
    The reference collects gate-range maxima to drive its anchored-clamp guard;
    this operator is exact for any gate range and keeps no such statistics, so
    the snapshot is always empty."""
    return {}
