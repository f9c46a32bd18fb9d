"""Run the CPU oracle (``oracle.gdn2_oracle``) over heads in parallel processes.

TEST / BASELINE INFRASTRUCTURE ONLY: used by ``bench.py`` for its
``cpu_baseline`` leg and its ``--impl reference`` arm (the reference's
algorithm restated on the host cores).  Heads are independent, so the work
splits over a ``spawn`` process pool with no communication.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import time

import numpy as np


def _fwd_bwd_heads(args):
    from oracle import gdn2_oracle as orc
    q, k, v, g, b, w, do = args
    r = orc.chunk_gdn2(q, k, v, g, b, w, output_final_state=True, do=do)
    return r.o.shape


def _decode_heads(args):
    from oracle import gdn2_oracle as orc
    q, k, v, g, b, w, S = args
    o, S2, _ = orc.recurrent_fwd(q, k, v, g, b, w, q.shape[-1] ** -0.5, S)
    return o.shape


class OraclePool:
    """A spawn-context pool of ``nproc`` workers (default: all host cores)."""

    def __init__(self, nproc: int | None = None):
        self.nproc = nproc or os.cpu_count() or 1
        self._pool = mp.get_context("spawn").Pool(self.nproc)

    def close(self):
        self._pool.close()
        self._pool.join()

    def fwd_bwd(self, q, k, v, g, b, w, do) -> float:
        """Forward + backward of the op on [B, T, H, *] numpy inputs; the heads
        are dealt round-robin to the workers.  Returns wall seconds."""
        H = q.shape[2]
        parts = []
        for i in range(self.nproc):
            hs = list(range(i, H, self.nproc))
            if hs:
                parts.append(tuple(np.ascontiguousarray(x[:, :, hs]) for x in (q, k, v, g, b, w, do)))
        t0 = time.perf_counter()
        self._pool.map(_fwd_bwd_heads, parts)
        return time.perf_counter() - t0

    def decode(self, q, k, v, g, b, w, S) -> float:
        """One token-serial step over [N, 1, H, *] inputs and state [N, H, K, V]."""
        H = q.shape[2]
        parts = []
        for i in range(self.nproc):
            hs = list(range(i, H, self.nproc))
            if hs:
                parts.append(tuple(np.ascontiguousarray(x[:, :, hs]) for x in (q, k, v, g, b, w))
                             + (np.ascontiguousarray(S[:, hs]),))
        t0 = time.perf_counter()
        self._pool.map(_decode_heads, parts)
        return time.perf_counter() - t0


def synthetic(B, T, H, K, V, seed=0):
    """Config-2 style inputs as float64 numpy: q, k L2-normalised, v ~ N(0,1),
    b, w = sigmoid(N(0,1)), g = -softplus(N(0,1)) * 0.1, cotangent ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, T, H, K))
    k = rng.standard_normal((B, T, H, K))
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((B, T, H, V))
    b = 1 / (1 + np.exp(-rng.standard_normal((B, T, H, K))))
    w = 1 / (1 + np.exp(-rng.standard_normal((B, T, H, V))))
    g = -np.log1p(np.exp(rng.standard_normal((B, T, H, K)))) * 0.1
    do = rng.standard_normal((B, T, H, V))
    return q, k, v, g, b, w, do
