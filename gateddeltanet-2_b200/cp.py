"""Context-parallel prefill: one sequence's T axis sharded over the ranks of a
process group (contiguous, equal shards in rank order).

Protocol (forward, inference/prefill):

1. every rank reduces its shard to the affine map of the state it receives,
   ``S_out = M S_in + h_e`` (``gdn2_cp_transition``);
2. one ``all_gather_into_tensor`` of the ``[N, H, K, K+V]`` fp32 maps
   (2 MiB per rank at H=16, K=V=128) -- the only collective;
3. each rank folds the maps of the ranks before it into its entering state
   (``gdn2_cp_compose``, fp32);
4. each rank runs the ordinary chunked forward on its shard from that state
   (the "correction pass"), which yields its outputs and exit state.

The reference implements this scheme for KDA only
(``lit_gpt/gdn2_ops/chunk_kda.py:774-945``); ``chunk_gdn2`` never passes a
context-parallel context.  The steps are pluggable (``backend``) so the
distributed control flow can be exercised without a GPU.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .chunk import chunk_gdn2


class CudaBackend:
    """The B200 kernels behind the C ABI."""

    def transition(self, q, k, v, g, b, w, *, scale, use_qk_l2norm_in_kernel,
                   use_gate_in_kernel, A_log, dt_bias, lower_bound):
        _lib.require_device(q)
        B, T, H, K = q.shape
        V = v.shape[-1]
        bw = b.dtype if (b.dtype == w.dtype and b.dtype in (torch.bfloat16, torch.float32)) else torch.float32
        qb, kb, vb = (x.to(torch.bfloat16).contiguous() for x in (q, k, v))
        gf = g.float().contiguous()
        bb, wb = b.to(bw).contiguous(), w.to(bw).contiguous()
        flags = 0
        if use_qk_l2norm_in_kernel:
            flags |= _lib.L2NORM_QK
        A_f = dt_f = None
        if use_gate_in_kernel:
            flags |= _lib.GATE_IN_KERNEL
            A_f = A_log.float().contiguous()
            dt_f = dt_bias.float().contiguous() if dt_bias is not None else None
            if lower_bound is not None:
                flags |= _lib.LOWER_BOUND
        args = _lib.ChunkArgs(
            B=B, T=T, H=H, K=K, V=V, N=B, NT=B * ((T + 63) // 64), scale=float(scale),
            lower_bound=float(lower_bound or 0.0), flags=flags, dtype_qkv=_lib.BF16,
            dtype_bw=_lib.BF16 if bw == torch.bfloat16 else _lib.F32,
            q=qb.data_ptr(), k=kb.data_ptr(), v=vb.data_ptr(), g=gf.data_ptr(), b=bb.data_ptr(),
            w=wb.data_ptr(), A_log=_lib.ptr(A_f), dt_bias=_lib.ptr(dt_f))
        lib = _lib.load()
        nbytes = lib.gdn2_chunk_workspace_size(args)
        ws = torch.empty(max(nbytes, 1), device=q.device, dtype=torch.uint8)
        maps = torch.empty(B, H, K, K + V, device=q.device, dtype=torch.float32)
        with torch.cuda.device(q.device):
            _lib.check(lib.gdn2_cp_transition(args, maps.data_ptr(), ws.data_ptr(), nbytes,
                                              _lib.stream_ptr(q.device)), "gdn2_cp_transition")
        return maps

    def compose(self, gathered, rank, state):
        W, N, H, K, KV = gathered.shape
        V = KV - K
        state = state.contiguous().clone()
        with torch.cuda.device(state.device):
            _lib.check(_lib.load().gdn2_cp_compose(gathered.contiguous().data_ptr(), rank, N, H, K, V,
                                                   state.data_ptr(), _lib.stream_ptr(state.device)),
                       "gdn2_cp_compose")
        return state

    def forward(self, q, k, v, g, b, w, *, initial_state, **kw):
        with torch.no_grad():
            return chunk_gdn2(q, k, v, g, b, w, initial_state=initial_state,
                              output_final_state=True, **kw)


def chunk_gdn2_cp(q, k, v, g, b, w, *, group=None, scale=None, initial_state=None,
                  use_qk_l2norm_in_kernel=False, use_gate_in_kernel=False, A_log=None,
                  dt_bias=None, lower_bound=None, backend=None):
    """Forward of ``chunk_gdn2`` for a sequence whose T axis is sharded over
    ``group`` (this rank holds shard ``rank``; all shards have equal length).

    q, k, g, b: ``[B, T_shard, H, K]``; v, w: ``[B, T_shard, H, V]``;
    ``initial_state``: the sequence's initial state ``[B, H, K, V]`` fp32 (read
    on every rank), or None.  Returns ``(o_shard, exit_state)``; the last
    rank's exit state is the sequence's final state.
    """
    backend = backend or CudaBackend()
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    B, T, H, K = q.shape
    V = v.shape[-1]
    if scale is None:
        scale = K ** -0.5
    gate_kw = dict(use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel,
                   use_gate_in_kernel=use_gate_in_kernel, lower_bound=lower_bound)
    maps = backend.transition(q, k, v, g, b, w, scale=scale, A_log=A_log, dt_bias=dt_bias, **gate_kw)
    if world > 1:
        flat = torch.empty((world * maps.shape[0],) + tuple(maps.shape[1:]), dtype=maps.dtype,
                           device=maps.device)
        dist.all_gather_into_tensor(flat, maps.contiguous(), group=group)
        gathered = flat.view((world,) + tuple(maps.shape))
    else:
        gathered = maps.unsqueeze(0)
    if initial_state is None:
        state = torch.zeros(B, H, K, V, dtype=torch.float32, device=maps.device)
    else:
        state = initial_state.to(device=maps.device, dtype=torch.float32)
    state = backend.compose(gathered, rank, state)
    fwd_kw = dict(gate_kw)
    if use_gate_in_kernel:
        fwd_kw.update(A_log=A_log, dt_bias=dt_bias)
    return backend.forward(q, k, v, g, b, w, initial_state=state, scale=scale, **fwd_kw)
