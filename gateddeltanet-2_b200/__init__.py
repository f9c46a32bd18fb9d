"""B200-native (sm_100a) Gated Delta Rule-2 operator.

Drop-in for the reference's ``lit_gpt.gdn2_ops``:

* ``chunk_gdn2`` / ``ChunkGDN2Function`` — chunkwise forward + backward
  (training / prefill), ``lit_gpt/gdn2_ops/chunk_gdn2.py``;
* ``fused_recurrent_gdn2`` / ``fused_recurrent_gdn2_fwd`` — token-serial
  decode, ``lit_gpt/gdn2_ops/fused_recurrent_gdn2.py``;
* ``cp`` — context-parallel prefill over ranks (T sharded);
* ``GatedDeltaNet2`` — the token-mixer layer around the operator
  (``lit_gpt/gdn2.py``), with its fused prep and gated-norm kernels.

Every op runs hand-written CUDA in ``libgdn2_b200.so`` through the C ABI
declared in ``include/gdn2.h``; there is no CPU or Triton fallback.

The directory name is not a Python identifier, so load it with
``importlib.import_module("gateddeltanet-2_b200")``; the import also
registers the alias ``gdn2_b200`` so later ``import gdn2_b200`` works.
"""

import sys as _sys

from . import _lib, cp
from .chunk import ChunkGDN2Function, chunk_gdn2, gdn2_telemetry_snapshot, prepare_chunk_indices
from .layer import FusedRMSNormSwishGate, GatedDeltaNet2, LayerCache, ShortConvolution
from .recurrent import fused_recurrent_gdn2, fused_recurrent_gdn2_fwd

_sys.modules.setdefault("gdn2_b200", _sys.modules[__name__])

__all__ = [
    "chunk_gdn2",
    "ChunkGDN2Function",
    "fused_recurrent_gdn2",
    "fused_recurrent_gdn2_fwd",
    "prepare_chunk_indices",
    "gdn2_telemetry_snapshot",
    "cp",
    "GatedDeltaNet2",
    "LayerCache",
    "ShortConvolution",
    "FusedRMSNormSwishGate",
]
