"""TEST INFRASTRUCTURE ONLY -- Python wrapper of the CPU oracle.

Loads ``libcc1d_oracle.so`` (built from ``cc1d_oracle.c`` by ``make -C
oracle``), a plain-C restatement of the reference's CPU kernels for the
causal conv1d hot path.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference arm use it, as the checker or as the
timed CPU path; the product (``causal_conv1d_b200``) never imports it.

All functions take and return CPU torch tensors.  ``acc64=True`` accumulates
in double (the checker); ``acc64=False`` accumulates in float like the
reference's CPU kernels (the timed port).
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
LIB_PATH = HERE / "libcc1d_oracle.so"

_DTYPE_CODE = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}
_lib = None


def build(force: bool = False) -> Path:
    """Compile the oracle with the committed Makefile (gcc + OpenMP)."""
    src = HERE / "cc1d_oracle.c"
    hdr = REPO / "include" / "cc1d.h"
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < max(src.stat().st_mtime, hdr.stat().st_mtime):
        subprocess.run(["make", "-s", "-C", str(HERE)] + (["-B"] if force else []), check=True)
    return LIB_PATH


def _structs():
    # The oracle reads the product's C ABI structs (include/cc1d.h); the
    # ctypes mirror lives with the product binding.
    from causal_conv1d_b200 import _lib as abi

    return abi


def load():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        abi = _structs()
        lib = ctypes.CDLL(str(LIB_PATH))
        lib.oracle_fwd.argtypes = [ctypes.POINTER(abi.FwdParams), ctypes.c_int, ctypes.c_int]
        lib.oracle_bwd.argtypes = [ctypes.POINTER(abi.BwdParams), ctypes.c_int, ctypes.c_int]
        lib.oracle_update.argtypes = [ctypes.POINTER(abi.UpdateParams), ctypes.c_int, ctypes.c_int]
        lib.oracle_varlen_states.argtypes = [ctypes.POINTER(abi.VarlenParams)]
        for f in (lib.oracle_fwd, lib.oracle_bwd, lib.oracle_update, lib.oracle_varlen_states):
            f.restype = ctypes.c_int
        lib.oracle_max_threads.restype = ctypes.c_int
        _lib = lib
    return _lib


def max_threads() -> int:
    return int(load().oracle_max_threads())


def _cpu(t):
    if t is None:
        return None
    if t.device.type != "cpu":
        raise ValueError("the oracle takes CPU tensors")
    return t


def fwd(x, weight, bias=None, seq_idx=None, initial_states=None, silu=False, return_final_states=False,
        acc64=True, nthreads=0, out=None, final_states=None):
    """Returns (out, final_states or None)."""
    abi = _structs()
    lib = load()
    x, weight, bias, seq_idx, initial_states = map(_cpu, (x, weight, bias, seq_idx, initial_states))
    B, D, L = x.shape
    W = weight.shape[1]
    if out is None:
        out = torch.empty(B, D, L, dtype=x.dtype)
    if return_final_states and final_states is None:
        final_states = torch.empty(B, D, W - 1, dtype=x.dtype)
    p = abi.FwdParams()
    p.dtype = _DTYPE_CODE[x.dtype]
    p.width = W
    p.batch, p.dim, p.seqlen = B, D, L
    p.silu = 1 if silu else 0
    p.x = x.data_ptr()
    p.x_batch_stride, p.x_dim_stride, p.x_seq_stride = x.stride()
    p.weight = weight.data_ptr()
    p.weight_dim_stride, p.weight_width_stride = weight.stride()
    if bias is not None:
        p.bias, p.bias_stride = bias.data_ptr(), bias.stride(0)
    if seq_idx is not None:
        p.seq_idx = seq_idx.data_ptr()
        p.seq_idx_batch_stride, p.seq_idx_seq_stride = seq_idx.stride()
    if initial_states is not None:
        p.initial_states = initial_states.data_ptr()
        p.init_batch_stride, p.init_dim_stride, p.init_seq_stride = initial_states.stride()
    p.out = out.data_ptr()
    p.out_batch_stride, p.out_dim_stride, p.out_seq_stride = out.stride()
    if return_final_states:
        p.final_states = final_states.data_ptr()
        p.final_batch_stride, p.final_dim_stride, p.final_seq_stride = final_states.stride()
    rc = lib.oracle_fwd(ctypes.byref(p), 1 if acc64 else 0, int(nthreads))
    if rc:
        raise RuntimeError(f"oracle_fwd failed ({rc})")
    return out, (final_states if return_final_states else None)


def bwd(x, weight, dout, bias=None, seq_idx=None, initial_states=None, dfinal_states=None, silu=False,
        acc64=True, nthreads=0):
    """Returns dict(dx, dweight (fp32), dbias (fp32 or None), dinit, dweight_cast, dbias_cast)."""
    abi = _structs()
    lib = load()
    x, weight, dout, bias, seq_idx, initial_states, dfinal_states = map(
        _cpu, (x, weight, dout, bias, seq_idx, initial_states, dfinal_states))
    B, D, L = x.shape
    W = weight.shape[1]
    dx = torch.empty(B, D, L, dtype=x.dtype)
    dwdb = torch.zeros(D * (W + 1), dtype=torch.float32)
    dw_cast = torch.empty(D, W, dtype=x.dtype)
    db_cast = torch.empty(D, dtype=x.dtype) if bias is not None else None
    dinit = torch.empty(B, D, W - 1, dtype=x.dtype) if initial_states is not None else None
    p = abi.BwdParams()
    p.dtype = _DTYPE_CODE[x.dtype]
    p.width = W
    p.batch, p.dim, p.seqlen = B, D, L
    p.silu = 1 if silu else 0
    p.x = x.data_ptr()
    p.x_batch_stride, p.x_dim_stride, p.x_seq_stride = x.stride()
    p.weight = weight.data_ptr()
    p.weight_dim_stride, p.weight_width_stride = weight.stride()
    if bias is not None:
        p.bias, p.bias_stride = bias.data_ptr(), bias.stride(0)
    p.dout = dout.data_ptr()
    p.dout_batch_stride, p.dout_dim_stride, p.dout_seq_stride = dout.stride()
    if seq_idx is not None:
        p.seq_idx = seq_idx.data_ptr()
        p.seq_idx_batch_stride, p.seq_idx_seq_stride = seq_idx.stride()
    if initial_states is not None:
        p.initial_states = initial_states.data_ptr()
        p.init_batch_stride, p.init_dim_stride, p.init_seq_stride = initial_states.stride()
        p.dinitial_states = dinit.data_ptr()
        p.dinit_batch_stride, p.dinit_dim_stride, p.dinit_seq_stride = dinit.stride()
    if dfinal_states is not None:
        p.dfinal_states = dfinal_states.data_ptr()
        p.dfinal_batch_stride, p.dfinal_dim_stride, p.dfinal_seq_stride = dfinal_states.stride()
    p.dx = dx.data_ptr()
    p.dx_batch_stride, p.dx_dim_stride, p.dx_seq_stride = dx.stride()
    p.dwdb_acc = dwdb.data_ptr()
    p.dweight_out = dw_cast.data_ptr()
    p.dweight_dim_stride, p.dweight_width_stride = dw_cast.stride()
    if db_cast is not None:
        p.dbias_out, p.dbias_stride = db_cast.data_ptr(), db_cast.stride(0)
    rc = lib.oracle_bwd(ctypes.byref(p), 1 if acc64 else 0, int(nthreads))
    if rc:
        raise RuntimeError(f"oracle_bwd failed ({rc})")
    return {
        "dx": dx,
        "dweight": dwdb[: D * W].view(D, W),
        "dbias": dwdb[D * W:] if bias is not None else None,
        "dwdb": dwdb,
        "dinit": dinit,
        "dweight_cast": dw_cast,
        "dbias_cast": db_cast,
    }


def update(x, conv_state, weight, bias=None, silu=False, cache_seqlens=None, conv_state_indices=None, acc64=True,
           nthreads=0):
    """conv_state is updated in place; returns out (same shape as a 3-D x)."""
    abi = _structs()
    lib = load()
    x, conv_state, weight, bias, cache_seqlens, conv_state_indices = map(
        _cpu, (x, conv_state, weight, bias, cache_seqlens, conv_state_indices))
    squeeze = x.dim() == 2
    if squeeze:
        x = x.unsqueeze(-1)
    B, D, L = x.shape
    out = torch.empty(B, D, L, dtype=x.dtype)
    p = abi.UpdateParams()
    p.dtype = _DTYPE_CODE[x.dtype]
    p.width = weight.shape[1]
    p.batch, p.dim, p.seqlen = B, D, L
    p.state_len = conv_state.shape[2]
    p.state_rows = conv_state.shape[0]
    p.silu = 1 if silu else 0
    p.x = x.data_ptr()
    p.x_batch_stride, p.x_dim_stride, p.x_seq_stride = x.stride()
    p.weight = weight.data_ptr()
    p.weight_dim_stride, p.weight_width_stride = weight.stride()
    if bias is not None:
        p.bias, p.bias_stride = bias.data_ptr(), bias.stride(0)
    p.conv_state = conv_state.data_ptr()
    p.state_batch_stride, p.state_dim_stride, p.state_seq_stride = conv_state.stride()
    p.conv_state_indices = 0 if conv_state_indices is None else conv_state_indices.data_ptr()
    p.cache_seqlens = 0 if cache_seqlens is None else cache_seqlens.data_ptr()
    p.out = out.data_ptr()
    p.out_batch_stride, p.out_dim_stride, p.out_seq_stride = out.stride()
    rc = lib.oracle_update(ctypes.byref(p), 1 if acc64 else 0, int(nthreads))
    if rc:
        raise RuntimeError(f"oracle_update failed ({rc})")
    return out.squeeze(-1) if squeeze else out


def varlen_states(x, cu_seqlens, state_len):
    abi = _structs()
    lib = load()
    x = _cpu(x)
    cu = _cpu(cu_seqlens).to(torch.int32).contiguous()
    T, D = x.shape
    B = cu.shape[0] - 1
    states = torch.empty(B, state_len, D, dtype=x.dtype).transpose(1, 2)
    p = abi.VarlenParams()
    p.dtype = _DTYPE_CODE[x.dtype]
    p.batch, p.dim, p.state_len, p.total_tokens = B, D, state_len, T
    p.x = x.data_ptr()
    p.x_token_stride, p.x_dim_stride = x.stride()
    p.cu_seqlens = cu.data_ptr()
    p.states = states.data_ptr()
    p.states_batch_stride, p.states_dim_stride, p.states_seq_stride = states.stride()
    rc = lib.oracle_varlen_states(ctypes.byref(p))
    if rc:
        raise RuntimeError(f"oracle_varlen_states failed ({rc})")
    return states

