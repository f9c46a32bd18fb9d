"""Token-serial GDN2 (decode) with the reference's Python interface.

Mirrors ``lit_gpt/gdn2_ops/fused_recurrent_gdn2.py``:
``fused_recurrent_gdn2_fwd`` (:284-395, the serving launcher with paged
state pool / speculative decoding / in-place state) and
``fused_recurrent_gdn2`` (:399-492, the validated public entry point).
Both run the CUDA kernel behind ``gdn2_recurrent_fwd``.
"""

from __future__ import annotations

import torch

from . import _lib


def _dt(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.BF16
    if t.dtype == torch.float32:
        return _lib.F32
    raise TypeError(f"unsupported dtype {t.dtype} (bf16 or fp32)")


@torch.compiler.disable
def fused_recurrent_gdn2_fwd(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    b: torch.Tensor,
    w: torch.Tensor,
    A_log: torch.Tensor | None = None,
    dt_bias: torch.Tensor | None = None,
    initial_state: torch.Tensor | None = None,
    scale: float | None = None,
    output_final_state: bool = False,
    inplace_final_state: bool = True,
    cu_seqlens: torch.LongTensor | None = None,
    ssm_state_indices: torch.Tensor | None = None,
    num_accepted_tokens: torch.Tensor | None = None,
    use_qk_l2norm_in_kernel: bool = False,
    use_gate_in_kernel: bool = False,
    lower_bound: float | None = None,
    out: torch.Tensor | None = None,
    transpose_state_layout: bool = False,
    **kwargs,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Launch the recurrent kernel (reference launcher semantics).

    ``inplace_final_state`` writes the final state back into
    ``initial_state``; with ``ssm_state_indices`` every token's state goes to
    its pool slot (``fused_recurrent_gdn2.py:245-262``).
    """
    _lib.require_device(q)
    if scale is None:
        scale = k.shape[-1] ** -0.5
    B, T, H, K = k.shape
    V = v.shape[-1]
    HV = v.shape[2]
    N = B if cu_seqlens is None else len(cu_seqlens) - 1

    # q, k share a dtype; g, b, w share one (bf16 or fp32)
    qkv_dtype = q.dtype if q.dtype in (torch.bfloat16, torch.float32) else torch.float32
    q, k, v = (x.to(qkv_dtype).contiguous() for x in (q, k, v))
    gbw_dtype = g.dtype if g.dtype in (torch.bfloat16, torch.float32) else torch.float32
    g, b, w = (x.to(gbw_dtype).contiguous() for x in (g, b, w))

    if out is None:
        out = torch.zeros_like(v)
    else:
        assert out.shape == v.shape
    if inplace_final_state:
        assert initial_state is not None, "inplace_final_state=True requires an initial_state"
        final_state = initial_state
    elif output_final_state:
        shp = (N, HV, V, K) if transpose_state_layout else (N, HV, K, V)
        final_state = q.new_empty(*shp, dtype=torch.float32)
    else:
        final_state = None
    if initial_state is not None:
        assert initial_state.dtype == torch.float32 and initial_state.is_contiguous()
    if ssm_state_indices is not None and final_state is None:
        raise ValueError("ssm_state_indices requires a state output (in place or final)")

    flags = 0
    if use_qk_l2norm_in_kernel:
        flags |= _lib.L2NORM_QK
    if use_gate_in_kernel:
        flags |= _lib.GATE_IN_KERNEL
        assert A_log is not None, "A_log must be provided when use_gate_in_kernel=True."
        if lower_bound is not None:
            flags |= _lib.LOWER_BOUND
    if transpose_state_layout:
        flags |= _lib.TRANSPOSE_STATE
    if initial_state is not None:
        flags |= _lib.HAS_H0
    if final_state is not None:
        flags |= _lib.STORE_FINAL

    slot = HV * K * V
    idx32 = None
    stride_seq = 1
    if ssm_state_indices is not None:
        idx32 = ssm_state_indices.to(torch.int32).contiguous()
        stride_seq = idx32.stride(0) if idx32.ndim > 1 else 1
    acc32 = None
    if num_accepted_tokens is not None:
        acc32 = num_accepted_tokens.to(torch.int32).contiguous()
    cu = None if cu_seqlens is None else cu_seqlens.to(torch.int64).contiguous()
    A_log_f = None if A_log is None else A_log.float().contiguous()
    dt_f = None if dt_bias is None else dt_bias.float().contiguous()

    args = _lib.RecurrentArgs(
        B=B, T=T, H=H, HV=HV, K=K, V=V, N=N,
        cu_seqlens=_lib.ptr(cu), ssm_state_indices=_lib.ptr(idx32),
        num_accepted_tokens=_lib.ptr(acc32), stride_indices_seq=stride_seq,
        state_slot_stride_in=initial_state.stride(0) if initial_state is not None else slot,
        state_slot_stride_out=final_state.stride(0) if final_state is not None else slot,
        scale=float(scale), lower_bound=float(lower_bound or 0.0),
        flags=flags, inplace=int(bool(inplace_final_state)),
        dtype_qkv=_dt(q), dtype_gbw=_dt(g),
        q=_lib.ptr(q), k=_lib.ptr(k), v=_lib.ptr(v), g=_lib.ptr(g), b=_lib.ptr(b), w=_lib.ptr(w),
        A_log=_lib.ptr(A_log_f), dt_bias=_lib.ptr(dt_f),
        h0=_lib.ptr(initial_state), ht=_lib.ptr(final_state), o=_lib.ptr(out),
    )
    with torch.cuda.device(q.device):
        _lib.check(_lib.load().gdn2_recurrent_fwd(args, _lib.stream_ptr(q.device)),
                   "gdn2_recurrent_fwd")
    return out, final_state


def fused_recurrent_gdn2(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    b: torch.Tensor,
    w: torch.Tensor,
    A_log: torch.Tensor | None = None,
    dt_bias: torch.Tensor | None = None,
    scale: float | None = None,
    initial_state: torch.Tensor = None,
    output_final_state: bool = False,
    use_qk_l2norm_in_kernel: bool = False,
    use_gate_in_kernel: bool = False,
    lower_bound: float | None = None,
    cu_seqlens: torch.LongTensor | None = None,
    transpose_state_layout: bool = False,
    **kwargs,
) -> tuple[torch.Tensor, torch.Tensor]:
    r"""Token-by-token forward for GDN2 (inference only, no gradients).

    Same arguments, shapes and checks as the reference
    (``fused_recurrent_gdn2.py:399-492``): q, k ``[B, T, H, K]``; v, w
    ``[B, T, HV, V]``; g, b ``[B, T, HV, K]``; ``initial_state``
    ``[N, HV, K, V]`` fp32.  Returns ``(o, final_state)``.
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
    assert b.shape == (*q.shape[:3], k.shape[-1]), (
        f"b must have shape [B, T, HV, K]; got {tuple(b.shape)} "
        f"vs expected {(*q.shape[:3], k.shape[-1])}."
    )
    assert w.shape == v.shape, (
        f"w must have shape [B, T, HV, V] matching v; got {tuple(w.shape)} "
        f"vs v {tuple(v.shape)}."
    )
    if scale is None:
        scale = k.shape[-1] ** -0.5
    if initial_state is not None:
        initial_state = initial_state.contiguous()
    return fused_recurrent_gdn2_fwd(
        q=q, k=k, v=v, g=g, b=b, w=w, A_log=A_log, dt_bias=dt_bias, scale=scale,
        initial_state=initial_state, inplace_final_state=False,
        output_final_state=output_final_state,
        use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel,
        use_gate_in_kernel=use_gate_in_kernel, lower_bound=lower_bound,
        cu_seqlens=cu_seqlens, transpose_state_layout=transpose_state_layout,
    )
