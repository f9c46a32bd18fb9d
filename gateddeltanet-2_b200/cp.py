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

Backward (training): the cotangent of a shard's exit state maps to that of
its entering state affinely, ``dS_in = M^T dS_out + g`` with ``g`` this
shard's own contribution (the state-cotangent scan alone, ``dS_out`` = the
shard's own ``dht``).  One ``all_gather`` of the ``g`` (``[N, H, K, V]`` fp32
per rank); each rank folds the ranks after it into the cotangent of its exit
state (``gdn2_cp_compose_bwd``) and runs the ordinary backward of its shard
with it.  The gradient of the sequence's initial state is rank 0's.  The maps
only parallelise the forward: the gradients are those of the sequential
computation.

The reference implements this scheme for KDA only
(``lit_gpt/gdn2_ops/chunk_kda.py:774-945``); ``chunk_gdn2`` never passes a
context-parallel context.  The steps are pluggable (``backend``) so the
distributed control flow can be exercised without a GPU.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .chunk import _chunk_backward, _chunk_forward, chunk_gdn2


class CudaBackend:
    """The B200 kernels behind the C ABI.  ``transition`` keeps its workspace,
    which holds the shard's intra-chunk factors; ``forward`` on the same inputs
    then runs only the state scan from the composed state (``GDN2_SKIP_INTRA``)."""

    def __init__(self):
        self._kept = None

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
        # the original input tensors are held (not their addresses), so the reuse
        # below can only ever match these very tensors, unmodified since
        gated = (A_log, dt_bias) if use_gate_in_kernel else (None, None)
        self._kept = (_reuse_key((q, k, v, g, b, w) + gated, flags, scale, lower_bound),
                      (q, k, v, g, b, w) + gated, args, ws, nbytes,
                      (qb, kb, vb, gf, bb, wb, A_f, dt_f), q.dtype)
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
        kept, self._kept = self._kept, None
        gate = bool(kw.get("use_gate_in_kernel"))
        flags = (_lib.L2NORM_QK if kw.get("use_qk_l2norm_in_kernel") else 0) | \
            (_lib.GATE_IN_KERNEL if gate else 0) | \
            (_lib.LOWER_BOUND if (gate and kw.get("lower_bound") is not None) else 0)
        A_log, dt_bias = (kw.get("A_log"), kw.get("dt_bias")) if gate else (None, None)
        same = kept is not None and \
            kept[0] == _reuse_key((q, k, v, g, b, w, A_log, dt_bias), flags, kw.get("scale"),
                                  kw.get("lower_bound"))
        if same:
            # the transition's workspace holds this shard's intra-chunk factors: scan only
            _, _, targs, ws, nbytes, held, qdtype = kept
            B, T, H, K = q.shape
            V = v.shape[-1]
            o = torch.empty(B, T, H, V, device=q.device, dtype=torch.bfloat16)
            ht = torch.empty(B, H, K, V, device=q.device, dtype=torch.float32)
            h0 = initial_state.to(torch.float32).contiguous()
            args = _lib.ChunkArgs.from_buffer_copy(targs)
            args.flags = targs.flags | _lib.HAS_H0 | _lib.STORE_FINAL | _lib.SKIP_INTRA
            args.h0, args.ht, args.o = h0.data_ptr(), ht.data_ptr(), o.data_ptr()
            with torch.cuda.device(q.device):
                _lib.check(_lib.load().gdn2_chunk_fwd(args, ws.data_ptr(), nbytes, _lib.stream_ptr(q.device)),
                           "gdn2_chunk_fwd")
            del held  # the inputs the factors were computed from stay alive until here
            return (o if qdtype == torch.bfloat16 else o.to(qdtype)), ht
        with torch.no_grad():
            return chunk_gdn2(q, k, v, g, b, w, initial_state=initial_state,
                              output_final_state=True, **kw)

    # ---- training pieces -------------------------------------------------
    def forward_train(self, q, k, v, g, b, w, *, initial_state, scale, use_qk_l2norm_in_kernel,
                      use_gate_in_kernel, A_log, dt_bias, lower_bound):
        """The shard's forward from ``initial_state``, keeping its backward operands."""
        self._kept = None  # the backward needs the saving forward's own workspace layout
        o, ht, saved, meta, _, _ = _chunk_forward(
            q, k, v, g, b, w, A_log, dt_bias, scale, initial_state, True, use_qk_l2norm_in_kernel,
            use_gate_in_kernel, None, None, lower_bound, False, True)
        return o, ht, (saved, meta)

    def state_cotangent(self, data, do, dht):
        """d(loss)/d(entering state) of the shard alone, for its do and dht."""
        return _chunk_backward(data[0], data[1], do, dht, state_only=True)

    def compose_bwd(self, gathered_maps, gathered_g, rank, dht):
        W, N, H, K, _ = gathered_maps.shape
        V = gathered_g.shape[-1]
        out = dht.to(torch.float32).contiguous().clone()
        with torch.cuda.device(out.device):
            _lib.check(_lib.load().gdn2_cp_compose_bwd(
                gathered_maps.contiguous().data_ptr(), gathered_g.contiguous().data_ptr(), rank, W,
                N, H, K, V, out.data_ptr(), _lib.stream_ptr(out.device)), "gdn2_cp_compose_bwd")
        return out

    def backward(self, data, do, dS_out):
        """(dq, dk, dv, dg, db, dw, dA_log, ddt_bias, d entering state) of the shard."""
        return _chunk_backward(data[0], data[1], do, dS_out)


def _reuse_key(tensors, flags, scale, lower_bound):
    """What decides whether a shard's forward may reuse its transition's
    intra-chunk factors: the identity and in-place version of every tensor the
    factors depend on (q, k, v, g, b, w and, with the gate in the kernel,
    A_log and dt_bias), the flags, the scale and the lower bound."""
    ident = tuple((id(t), t._version) if t is not None else None for t in tensors)
    lb = float(lower_bound) if (flags & _lib.LOWER_BOUND) and lower_bound is not None else None
    return ident, flags, float(scale) if scale is not None else None, lb


def _gather(x, group, world):
    if world == 1:
        return x.unsqueeze(0)
    flat = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(flat, x.contiguous(), group=group)
    return flat.view((world,) + tuple(x.shape))


class ChunkGDN2CPFunction(torch.autograd.Function):
    """Autograd of the context-parallel op (see the module docstring)."""

    @staticmethod
    def forward(ctx, q, k, v, g, b, w, A_log, dt_bias, initial_state, scale, use_qk_l2norm_in_kernel,
                use_gate_in_kernel, lower_bound, group, backend):
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        B, T, H, K = q.shape
        V = v.shape[-1]
        kw = dict(use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel, use_gate_in_kernel=use_gate_in_kernel,
                  A_log=A_log, dt_bias=dt_bias, lower_bound=lower_bound)
        maps = backend.transition(q, k, v, g, b, w, scale=scale, **kw)
        gathered = _gather(maps, group, world)
        if initial_state is None:
            state = torch.zeros(B, H, K, V, dtype=maps.dtype, device=maps.device)
        else:
            state = initial_state.to(device=maps.device, dtype=maps.dtype)
        S_in = backend.compose(gathered, rank, state)
        o, ht, data = backend.forward_train(q, k, v, g, b, w, initial_state=S_in, scale=scale, **kw)
        ctx.data, ctx.gathered = data, gathered
        ctx.cp = (rank, world, group, backend, initial_state is not None, ht.shape, ht.dtype)
        return o, ht

    @staticmethod
    def backward(ctx, do, dht):
        rank, world, group, backend, has_h0, ht_shape, ht_dtype = ctx.cp
        if dht is None:
            dht = torch.zeros(ht_shape, dtype=ht_dtype, device=do.device)
        gp = backend.state_cotangent(ctx.data, do, dht)
        gathered_g = _gather(gp, group, world)
        dS_out = backend.compose_bwd(ctx.gathered, gathered_g, rank, dht)
        dq, dk, dv, dg, db, dw, dA, ddt, dS_in = backend.backward(ctx.data, do, dS_out)
        dh0 = None
        if has_h0:
            dh0 = dS_in if rank == 0 else torch.zeros_like(dS_in)
        return dq, dk, dv, dg, db, dw, dA, ddt, dh0, None, None, None, None, None, None


def chunk_gdn2_cp(q, k, v, g, b, w, *, group=None, scale=None, initial_state=None,
                  use_qk_l2norm_in_kernel=False, use_gate_in_kernel=False, A_log=None,
                  dt_bias=None, lower_bound=None, backend=None):
    """``chunk_gdn2`` for a sequence whose T axis is sharded over ``group``
    (this rank holds shard ``rank``; all shards have equal length).  With
    inputs that require grad the result is differentiable (every rank must
    run the backward: it holds one all_gather).

    q, k, g, b: ``[B, T_shard, H, K]``; v, w: ``[B, T_shard, H, V]``;
    ``initial_state``: the sequence's initial state ``[B, H, K, V]`` fp32 (read
    on every rank), or None.  Returns ``(o_shard, exit_state)``; the last
    rank's exit state is the sequence's final state.
    """
    backend = backend or CudaBackend()
    if scale is None:
        scale = q.shape[-1] ** -0.5
    inputs = (q, k, v, g, b, w, A_log, dt_bias, initial_state)
    if torch.is_grad_enabled() and any(x is not None and x.requires_grad for x in inputs):
        return ChunkGDN2CPFunction.apply(q, k, v, g, b, w, A_log, dt_bias, initial_state, scale,
                                         use_qk_l2norm_in_kernel, use_gate_in_kernel, lower_bound,
                                         group, backend)
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
