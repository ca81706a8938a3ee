"""ctypes binding of libcc1d_sm100.so (the C ABI declared in include/cc1d.h).

The structs below mirror the header field for field.  The library is loaded
on first use; if it is missing the call fails loudly -- there is no CPU or
pure-PyTorch fallback on the product path.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_NAME = "libcc1d_sm100.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_ptr = ctypes.c_void_p

# Status codes (enum cc1d_status).
CC1D_OK = 0
CC1D_ERR_INVALID_ARGUMENT = 1
CC1D_ERR_UNSUPPORTED = 2
CC1D_ERR_CUDA = 3
CC1D_ERR_WORKSPACE = 4


def _fields(*groups):
    out = []
    for g in groups:
        out.extend(g)
    return out


def _tensor3(prefix, ptr_name):
    return [(ptr_name, c_ptr), (f"{prefix}_batch_stride", c_i64), (f"{prefix}_dim_stride", c_i64),
            (f"{prefix}_seq_stride", c_i64)]


class FwdParams(ctypes.Structure):
    _fields_ = _fields(
        [("dtype", c_i32), ("width", c_i32), ("batch", c_i64), ("dim", c_i64), ("seqlen", c_i64),
         ("silu", c_i32), ("_pad0", c_i32)],
        _tensor3("x", "x"),
        [("weight", c_ptr), ("weight_dim_stride", c_i64), ("weight_width_stride", c_i64)],
        [("bias", c_ptr), ("bias_stride", c_i64)],
        [("seq_idx", c_ptr), ("seq_idx_batch_stride", c_i64), ("seq_idx_seq_stride", c_i64)],
        _tensor3("init", "initial_states"),
        _tensor3("out", "out"),
        _tensor3("final", "final_states"),
    )


class BwdParams(ctypes.Structure):
    _fields_ = _fields(
        [("dtype", c_i32), ("width", c_i32), ("batch", c_i64), ("dim", c_i64), ("seqlen", c_i64),
         ("silu", c_i32), ("_pad0", c_i32)],
        _tensor3("x", "x"),
        [("weight", c_ptr), ("weight_dim_stride", c_i64), ("weight_width_stride", c_i64)],
        [("bias", c_ptr), ("bias_stride", c_i64)],
        _tensor3("dout", "dout"),
        [("seq_idx", c_ptr), ("seq_idx_batch_stride", c_i64), ("seq_idx_seq_stride", c_i64)],
        _tensor3("init", "initial_states"),
        _tensor3("dfinal", "dfinal_states"),
        _tensor3("dx", "dx"),
        _tensor3("dinit", "dinitial_states"),
        [("dwdb_acc", c_ptr)],
        [("dweight_out", c_ptr), ("dweight_dim_stride", c_i64), ("dweight_width_stride", c_i64)],
        [("dbias_out", c_ptr), ("dbias_stride", c_i64)],
        [("workspace", c_ptr), ("workspace_bytes", ctypes.c_size_t)],
    )


class UpdateParams(ctypes.Structure):
    _fields_ = _fields(
        [("dtype", c_i32), ("width", c_i32), ("batch", c_i64), ("dim", c_i64), ("seqlen", c_i64),
         ("state_len", c_i64), ("state_rows", c_i64), ("silu", c_i32), ("_pad0", c_i32)],
        _tensor3("x", "x"),
        [("weight", c_ptr), ("weight_dim_stride", c_i64), ("weight_width_stride", c_i64)],
        [("bias", c_ptr), ("bias_stride", c_i64)],
        _tensor3("state", "conv_state"),
        [("conv_state_indices", c_ptr), ("cache_seqlens", c_ptr)],
        _tensor3("out", "out"),
    )


class VarlenParams(ctypes.Structure):
    _fields_ = [
        ("dtype", c_i32), ("_pad0", c_i32), ("batch", c_i64), ("dim", c_i64), ("state_len", c_i64),
        ("total_tokens", c_i64),
        ("x", c_ptr), ("x_token_stride", c_i64), ("x_dim_stride", c_i64),
        ("cu_seqlens", c_ptr),
        ("states", c_ptr), ("states_batch_stride", c_i64), ("states_dim_stride", c_i64),
        ("states_seq_stride", c_i64),
    ]


class InprojConvParams(ctypes.Structure):
    _fields_ = [
        ("dtype", c_i32), ("width", c_i32), ("batch", c_i64), ("seqlen", c_i64), ("dim", c_i64),
        ("hidden_dim", c_i64), ("silu", c_i32), ("_pad0", c_i32),
        ("hidden", c_ptr), ("hidden_row_stride", c_i64),
        ("in_weight", c_ptr), ("in_weight_row_stride", c_i64),
        ("conv_weight", c_ptr), ("conv_weight_dim_stride", c_i64), ("conv_weight_width_stride", c_i64),
        ("conv_bias", c_ptr), ("conv_bias_stride", c_i64),
        ("initial_states", c_ptr), ("init_batch_stride", c_i64), ("init_dim_stride", c_i64),
        ("init_seq_stride", c_i64),
        ("out", c_ptr), ("out_row_stride", c_i64),
        ("final_states", c_ptr), ("final_batch_stride", c_i64), ("final_dim_stride", c_i64),
        ("final_seq_stride", c_i64),
    ]


class PeerReduceParams(ctypes.Structure):
    _fields_ = [("rank", c_i32), ("world", c_i32), ("exchange", c_ptr), ("epochs", c_ptr),
                ("max_polls", ctypes.c_uint32), ("flags", ctypes.c_uint32), ("status", c_ptr)]


# cc1d_peer_reduce.flags
PEER_FUSED = 0
PEER_PUSH = 1
PEER_FINISH = 2


# Every symbol include/cc1d.h declares, with its ctypes signature.
SIGNATURES = {
    "cc1d_fwd": (c_i32, [ctypes.POINTER(FwdParams), c_ptr]),
    "cc1d_bwd_workspace_size": (c_i32, [ctypes.POINTER(BwdParams), ctypes.POINTER(ctypes.c_size_t)]),
    "cc1d_bwd": (c_i32, [ctypes.POINTER(BwdParams), c_ptr]),
    "cc1d_bwd_noalloc": (c_i32, [ctypes.POINTER(BwdParams), c_ptr]),
    "cc1d_bwd_peer_reduce": (c_i32, [ctypes.POINTER(BwdParams), ctypes.POINTER(PeerReduceParams), c_ptr]),
    "cc1d_peer_blocks": (c_i64, [c_i64, c_i32]),
    "cc1d_peer_exchange_bytes": (c_i64, [c_i64, c_i32, c_i32]),
    "cc1d_update": (c_i32, [ctypes.POINTER(UpdateParams), c_ptr]),
    "cc1d_varlen_states": (c_i32, [ctypes.POINTER(VarlenParams), c_ptr]),
    "cc1d_inproj_conv_fwd": (c_i32, [ctypes.POINTER(InprojConvParams), c_ptr]),
    "cc1d_device_status": (c_i32, [ctypes.POINTER(ctypes.c_uint)]),
    "cc1d_last_error": (ctypes.c_char_p, []),
    "cc1d_version": (ctypes.c_char_p, []),
    "cc1d_abi_version": (c_i32, []),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.is_file():
                raise RuntimeError(
                    f"{LIB_NAME} not found at {LIB_PATH}. Build it with "
                    "`python -m causal_conv1d_b200._build` (nvcc, sm_100a); there is no "
                    "CPU fallback."
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


class Cc1dError(RuntimeError):
    """A C ABI call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def check(status: int, what: str) -> None:
    if status != CC1D_OK:
        msg = load().cc1d_last_error().decode(errors="replace")
        raise Cc1dError(status, f"{what} failed (status {status}): {msg}")


def device_wait_timeouts(device=None) -> int:
    """Bounded in-kernel waits that gave up on `device` (default: the current
    CUDA device) since the last call for that device, and reset its count;
    synchronises that device.  The counts are per device: a process driving
    several GPUs asks each one (``device_wait_timeouts(d)`` for every d)."""
    import torch

    lib = load()
    n = ctypes.c_uint(0)
    prev = torch.cuda.current_device()
    if device is None:
        dev = prev
    elif isinstance(device, int):
        dev = device
    else:
        dev = torch.device(device).index
        dev = prev if dev is None else dev
    try:
        if dev != prev:
            torch.cuda.set_device(dev)
        check(lib.cc1d_device_status(ctypes.byref(n)), "cc1d_device_status")
    finally:
        if dev != prev:
            torch.cuda.set_device(prev)
    return int(n.value)
