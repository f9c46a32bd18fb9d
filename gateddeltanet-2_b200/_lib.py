"""ctypes binding of the C ABI in include/gdn2.h (libgdn2_b200.so).

This is the only route from Python to the CUDA kernels.  There is no CPU
fallback: if the library is missing or no sm_100 device is present the
operators raise.
"""

from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgdn2_b200.so")

# enum gdn2_dtype
BF16, F32 = 0, 1
# enum gdn2_flags
L2NORM_QK = 1 << 0
GATE_IN_KERNEL = 1 << 1
LOWER_BOUND = 1 << 2
TRANSPOSE_STATE = 1 << 3
HAS_H0 = 1 << 4
STORE_FINAL = 1 << 5
SAVE_FOR_BWD = 1 << 6
BWD_STATE_ONLY = 1 << 7
G_BF16 = 1 << 8
SKIP_INTRA = 1 << 9
# enum gdn2_ws_buffer
WS_CHUNK_STATES = 0

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_f32 = ctypes.c_float


class ChunkArgs(ctypes.Structure):
    _fields_ = [
        ("B", _i64), ("T", _i64), ("H", _i64), ("K", _i64), ("V", _i64),
        ("N", _i64), ("NT", _i64),
        ("cu_seqlens", _p), ("chunk_index", _p), ("chunk_offset", _p),
        ("scale", _f32), ("lower_bound", _f32),
        ("flags", _i32), ("dtype_qkv", _i32), ("dtype_bw", _i32),
        ("q", _p), ("k", _p), ("v", _p), ("g", _p), ("b", _p), ("w", _p),
        ("A_log", _p), ("dt_bias", _p), ("h0", _p), ("ht", _p), ("o", _p),
    ]


class ChunkGrads(ctypes.Structure):
    _fields_ = [
        ("dout", _p), ("dht", _p), ("dq", _p), ("dk", _p), ("dv", _p), ("dg", _p),
        ("db", _p), ("dw", _p), ("dh0", _p), ("dA_log", _p), ("ddt_bias", _p),
    ]


class RecurrentArgs(ctypes.Structure):
    _fields_ = [
        ("B", _i64), ("T", _i64), ("H", _i64), ("HV", _i64), ("K", _i64), ("V", _i64),
        ("N", _i64),
        ("cu_seqlens", _p), ("ssm_state_indices", _p), ("num_accepted_tokens", _p),
        ("stride_indices_seq", _i64), ("state_slot_stride_in", _i64),
        ("state_slot_stride_out", _i64),
        ("scale", _f32), ("lower_bound", _f32),
        ("flags", _i32), ("inplace", _i32), ("dtype_qkv", _i32), ("dtype_gbw", _i32),
        ("q", _p), ("k", _p), ("v", _p), ("g", _p), ("b", _p), ("w", _p),
        ("A_log", _p), ("dt_bias", _p), ("h0", _p), ("ht", _p), ("o", _p),
    ]


class PrepArgs(ctypes.Structure):
    _fields_ = [
        ("rows", _i64), ("T", _i64), ("N", _i64), ("cu_seqlens", _p),
        ("Dk", _i64), ("Dv", _i64), ("Dfg", _i64), ("conv_size", _i64), ("proj_stride", _i64),
        ("b_scale", _f32), ("flags", _i32),
        ("proj", _p), ("conv_weight", _p), ("conv_bias", _p),
        ("conv_state_in", _p), ("conv_state_out", _p),
        ("q", _p), ("k", _p), ("v", _p), ("b", _p), ("w", _p), ("f0", _p), ("g0", _p),
    ]


class PrepGrads(ctypes.Structure):
    _fields_ = [
        ("dq", _p), ("dk", _p), ("dv", _p), ("db", _p), ("dw", _p), ("df0", _p), ("dg0", _p),
        ("dproj", _p), ("dconv_weight", _p), ("dconv_bias", _p),
    ]


class KernelStat(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("launches", _i64), ("total_ms", ctypes.c_double)]


class Gdn2Error(RuntimeError):
    """A non-zero status from the C ABI."""


_lib = None

# every symbol include/gdn2.h declares
EXPORTS = (
    "gdn2_chunk_workspace_size", "gdn2_chunk_bwd_workspace_size", "gdn2_chunk_workspace_offset",
    "gdn2_chunk_fwd", "gdn2_chunk_fwd_static_scratch",
    "gdn2_chunk_bwd", "gdn2_recurrent_fwd", "gdn2_cp_transition", "gdn2_cp_compose",
    "gdn2_cp_compose_bwd",
    "gdn2_status_string", "gdn2_device_supported", "gdn2_abi_version",
    "gdn2_profile_enable", "gdn2_profile_read", "gdn2_device_fault_read",
    "gdn2_layer_prep_fwd", "gdn2_layer_prep_bwd_workspace_size", "gdn2_layer_prep_bwd",
    "gdn2_norm_gate_fwd", "gdn2_norm_gate_bwd_workspace_size", "gdn2_norm_gate_bwd",
)


def load() -> ctypes.CDLL:
    """Load libgdn2_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python gateddeltanet-2_b200/build.py` "
            "(the operator has no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    lib.gdn2_chunk_workspace_size.argtypes = [ctypes.POINTER(ChunkArgs)]
    lib.gdn2_chunk_workspace_size.restype = ctypes.c_size_t
    lib.gdn2_chunk_bwd_workspace_size.argtypes = [ctypes.POINTER(ChunkArgs)]
    lib.gdn2_chunk_bwd_workspace_size.restype = ctypes.c_size_t
    lib.gdn2_chunk_workspace_offset.argtypes = [ctypes.POINTER(ChunkArgs), ctypes.c_int]
    lib.gdn2_chunk_workspace_offset.restype = ctypes.c_size_t
    lib.gdn2_chunk_fwd.argtypes = [ctypes.POINTER(ChunkArgs), _p, ctypes.c_size_t, _p]
    lib.gdn2_chunk_fwd.restype = ctypes.c_int
    lib.gdn2_chunk_bwd.argtypes = [ctypes.POINTER(ChunkArgs), ctypes.POINTER(ChunkGrads), _p,
                                   ctypes.c_size_t, _p, ctypes.c_size_t, _p]
    lib.gdn2_chunk_bwd.restype = ctypes.c_int
    lib.gdn2_recurrent_fwd.argtypes = [ctypes.POINTER(RecurrentArgs), _p]
    lib.gdn2_recurrent_fwd.restype = ctypes.c_int
    lib.gdn2_cp_transition.argtypes = [ctypes.POINTER(ChunkArgs), _p, _p, ctypes.c_size_t, _p]
    lib.gdn2_cp_transition.restype = ctypes.c_int
    lib.gdn2_cp_compose.argtypes = [_p, _i32, _i64, _i64, _i64, _i64, _p, _p]
    lib.gdn2_cp_compose.restype = ctypes.c_int
    lib.gdn2_cp_compose_bwd.argtypes = [_p, _p, _i32, _i32, _i64, _i64, _i64, _i64, _p, _p]
    lib.gdn2_cp_compose_bwd.restype = ctypes.c_int
    lib.gdn2_status_string.argtypes = [ctypes.c_int]
    lib.gdn2_status_string.restype = ctypes.c_char_p
    lib.gdn2_device_supported.argtypes = [ctypes.c_int]
    lib.gdn2_device_supported.restype = ctypes.c_int
    lib.gdn2_profile_enable.argtypes = [ctypes.c_int]
    lib.gdn2_profile_enable.restype = ctypes.c_int
    lib.gdn2_profile_read.argtypes = [ctypes.POINTER(KernelStat), ctypes.c_int]
    lib.gdn2_profile_read.restype = ctypes.c_int
    lib.gdn2_abi_version.argtypes = []
    lib.gdn2_abi_version.restype = ctypes.c_int
    lib.gdn2_device_fault_read.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_uint)]
    lib.gdn2_device_fault_read.restype = ctypes.c_int
    lib.gdn2_layer_prep_fwd.argtypes = [ctypes.POINTER(PrepArgs), _p]
    lib.gdn2_layer_prep_fwd.restype = ctypes.c_int
    lib.gdn2_layer_prep_bwd_workspace_size.argtypes = [ctypes.POINTER(PrepArgs)]
    lib.gdn2_layer_prep_bwd_workspace_size.restype = ctypes.c_size_t
    lib.gdn2_layer_prep_bwd.argtypes = [ctypes.POINTER(PrepArgs), ctypes.POINTER(PrepGrads), _p,
                                        ctypes.c_size_t, _p]
    lib.gdn2_layer_prep_bwd.restype = ctypes.c_int
    lib.gdn2_norm_gate_fwd.argtypes = [_p, _p, _p, _f32, _i64, _i64, _p, _p, _p]
    lib.gdn2_norm_gate_fwd.restype = ctypes.c_int
    lib.gdn2_norm_gate_bwd_workspace_size.argtypes = [_i64, _i64]
    lib.gdn2_norm_gate_bwd_workspace_size.restype = ctypes.c_size_t
    lib.gdn2_norm_gate_bwd.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _p, _p, _p, _p, ctypes.c_size_t, _p]
    lib.gdn2_norm_gate_bwd.restype = ctypes.c_int
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = load().gdn2_status_string(status).decode()
        raise Gdn2Error(f"{what} failed with status {status}: {msg}")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_checked_devices: set[int] = set()


def require_device(t: torch.Tensor) -> None:
    """Raise unless ``t`` lives on an sm_100 device the library can run on."""
    if not t.is_cuda:
        raise RuntimeError(
            "gdn2 B200 operators run only on CUDA tensors (no CPU fallback); "
            f"got a tensor on {t.device}")
    idx = t.device.index if t.device.index is not None else torch.cuda.current_device()
    if idx in _checked_devices:
        return
    if not load().gdn2_device_supported(idx):
        cap = torch.cuda.get_device_capability(idx)
        raise RuntimeError(f"libgdn2_b200 is built for sm_100a; device {idx} has capability {cap}")
    _checked_devices.add(idx)


def profile_enable(on: bool) -> None:
    """Start/stop recording per-launch CUDA-event timings inside the library."""
    load().gdn2_profile_enable(1 if on else 0)


def profile_read() -> dict:
    """{kernel name: (launches, total device ms)} since the last read."""
    buf = (KernelStat * 16)()
    n = load().gdn2_profile_read(buf, 16)
    if n < 0:
        check(n, "gdn2_profile_read")
    return {buf[i].name.decode(): (int(buf[i].launches), float(buf[i].total_ms)) for i in range(n)}


def device_fault_read(clear: bool = True) -> int:
    """Fault word of the current device: bit 0 = a bounded wait inside a
    tensor-core kernel gave up (its results are invalid).  Synchronises."""
    import torch
    torch.cuda.synchronize()
    out = ctypes.c_uint(0)
    check(load().gdn2_device_fault_read(1 if clear else 0, ctypes.byref(out)), "gdn2_device_fault_read")
    return int(out.value)
