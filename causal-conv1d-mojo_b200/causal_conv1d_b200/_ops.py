"""torch.library custom ops over the C ABI.

Each op mutates pre-allocated outputs in place and returns nothing, like the
reference's ``causal_conv1d_mojo::_fwd_inplace`` / ``_bwd_full_inplace``
(src/causal_conv1d_mojo/_fn.py:82-201), so ``torch.compile(fullgraph=True)``
sees one opaque node per kernel call and CUDA-graph capture records the
launches on the current stream.  Unlike the reference, the decode update and
the varlen state gather are custom ops too.

Every op launches on ``torch.cuda.current_stream()`` of the tensors' device
and never synchronises.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_DTYPE_CODE = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


def _ptr(t: torch.Tensor | None) -> int:
    return 0 if t is None else t.data_ptr()


def _s3(t: torch.Tensor | None) -> tuple[int, int, int]:
    return (0, 0, 0) if t is None else (t.stride(0), t.stride(1), t.stride(2))


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


class _on_device:
    """Make `dev` the current CUDA device for the duration of a call."""

    __slots__ = ("dev", "prev")

    def __init__(self, dev: torch.device):
        self.dev = dev.index if dev.index is not None else torch.cuda.current_device()
        self.prev = -1

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.dev:
            self.prev = cur
            torch.cuda.set_device(self.dev)
        return self

    def __exit__(self, *exc):
        if self.prev >= 0:
            torch.cuda.set_device(self.prev)
        return False


def _require_cuda(x: torch.Tensor, op: str) -> None:
    if not x.is_cuda:
        raise RuntimeError(
            f"{op}: causal_conv1d_b200 runs only on CUDA (sm_100a) devices; got a tensor on "
            f"{x.device}. There is no CPU fallback; use causal_conv1d_ref for a pure-PyTorch path."
        )


def _fwd_params(x, weight, bias, seq_idx, initial_states, out, apply_silu, final_states_out):
    p = _lib.FwdParams()
    p.dtype = _DTYPE_CODE[x.dtype]
    p.width = weight.shape[1]
    p.batch, p.dim, p.seqlen = x.shape
    p.silu = 1 if apply_silu else 0
    p.x = x.data_ptr()
    p.x_batch_stride, p.x_dim_stride, p.x_seq_stride = x.stride()
    p.weight = weight.data_ptr()
    p.weight_dim_stride, p.weight_width_stride = weight.stride()
    if bias is not None:
        p.bias = bias.data_ptr()
        p.bias_stride = bias.stride(0)
    if seq_idx is not None:
        p.seq_idx = seq_idx.data_ptr()
        p.seq_idx_batch_stride, p.seq_idx_seq_stride = seq_idx.stride()
    if initial_states is not None:
        p.initial_states = initial_states.data_ptr()
        p.init_batch_stride, p.init_dim_stride, p.init_seq_stride = initial_states.stride()
    p.out = out.data_ptr()
    p.out_batch_stride, p.out_dim_stride, p.out_seq_stride = out.stride()
    if final_states_out is not None:
        p.final_states = final_states_out.data_ptr()
        p.final_batch_stride, p.final_dim_stride, p.final_seq_stride = final_states_out.stride()
    return p


def _fwd_impl(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    seq_idx: torch.Tensor | None,
    initial_states: torch.Tensor | None,
    out: torch.Tensor,
    apply_silu: bool,
    final_states_out: torch.Tensor | None,
) -> None:
    _require_cuda(x, "causal_conv1d_fn")
    lib = _lib.load()
    p = _fwd_params(x, weight, bias, seq_idx, initial_states, out, apply_silu, final_states_out)
    with _on_device(x.device):
        _lib.check(lib.cc1d_fwd(ctypes.byref(p), _stream(x.device)), "cc1d_fwd")


def _fwd_fake(x, weight, bias, seq_idx, initial_states, out, apply_silu, final_states_out) -> None:
    return None


fwd = torch.library.custom_op("causal_conv1d_b200::fwd", mutates_args=("out", "final_states_out"))(_fwd_impl)
fwd.register_fake(_fwd_fake)


def _bwd_params(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx, dwdb_acc, dinitial_states,
                dweight_out, dbias_out, apply_silu):
    p = _lib.BwdParams()
    p.dtype = _DTYPE_CODE[x.dtype]
    p.width = weight.shape[1]
    p.batch, p.dim, p.seqlen = x.shape
    p.silu = 1 if apply_silu else 0
    p.x = x.data_ptr()
    p.x_batch_stride, p.x_dim_stride, p.x_seq_stride = x.stride()
    p.weight = weight.data_ptr()
    p.weight_dim_stride, p.weight_width_stride = weight.stride()
    if bias is not None:
        p.bias = bias.data_ptr()
        p.bias_stride = bias.stride(0)
    p.dout = dout.data_ptr()
    p.dout_batch_stride, p.dout_dim_stride, p.dout_seq_stride = dout.stride()
    if seq_idx is not None:
        p.seq_idx = seq_idx.data_ptr()
        p.seq_idx_batch_stride, p.seq_idx_seq_stride = seq_idx.stride()
    if initial_states is not None:
        p.initial_states = initial_states.data_ptr()
        p.init_batch_stride, p.init_dim_stride, p.init_seq_stride = initial_states.stride()
    if dfinal_states is not None:
        p.dfinal_states = dfinal_states.data_ptr()
        p.dfinal_batch_stride, p.dfinal_dim_stride, p.dfinal_seq_stride = dfinal_states.stride()
    p.dx = dx.data_ptr()
    p.dx_batch_stride, p.dx_dim_stride, p.dx_seq_stride = dx.stride()
    if dinitial_states is not None:
        p.dinitial_states = dinitial_states.data_ptr()
        p.dinit_batch_stride, p.dinit_dim_stride, p.dinit_seq_stride = dinitial_states.stride()
    p.dwdb_acc = dwdb_acc.data_ptr()
    if dweight_out is not None:
        p.dweight_out = dweight_out.data_ptr()
        p.dweight_dim_stride, p.dweight_width_stride = dweight_out.stride()
    if dbias_out is not None:
        p.dbias_out = dbias_out.data_ptr()
        p.dbias_stride = dbias_out.stride(0)
    return p


def bwd_workspace_bytes(p: _lib.BwdParams) -> int:
    lib = _lib.load()
    n = ctypes.c_size_t(0)
    _lib.check(lib.cc1d_bwd_workspace_size(ctypes.byref(p), ctypes.byref(n)), "cc1d_bwd_workspace_size")
    return int(n.value)


def _bwd_impl(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    dout: torch.Tensor,
    seq_idx: torch.Tensor | None,
    initial_states: torch.Tensor | None,
    dfinal_states: torch.Tensor | None,
    dx: torch.Tensor,
    dwdb_acc: torch.Tensor,
    dinitial_states: torch.Tensor | None,
    dweight_out: torch.Tensor | None,
    dbias_out: torch.Tensor | None,
    apply_silu: bool,
) -> None:
    _require_cuda(x, "causal_conv1d_fn backward")
    lib = _lib.load()
    p = _bwd_params(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx, dwdb_acc, dinitial_states,
                    dweight_out, dbias_out, apply_silu)
    with _on_device(x.device):
        nbytes = bwd_workspace_bytes(p)
        ws = None
        if nbytes > 0:
            ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
            p.workspace = ws.data_ptr()
            p.workspace_bytes = nbytes
        _lib.check(lib.cc1d_bwd(ctypes.byref(p), _stream(x.device)), "cc1d_bwd")
        del ws  # the caching allocator keeps the block stream-ordered


def _bwd_fake(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx, dwdb_acc, dinitial_states,
              dweight_out, dbias_out, apply_silu) -> None:
    return None


bwd = torch.library.custom_op(
    "causal_conv1d_b200::bwd",
    mutates_args=("dx", "dwdb_acc", "dinitial_states", "dweight_out", "dbias_out"),
)(_bwd_impl)
bwd.register_fake(_bwd_fake)


def _bwd_peer_impl(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    dout: torch.Tensor,
    initial_states: torch.Tensor | None,
    dfinal_states: torch.Tensor | None,
    dx: torch.Tensor,
    dwdb_acc: torch.Tensor,
    dinitial_states: torch.Tensor | None,
    dweight_out: torch.Tensor | None,
    dbias_out: torch.Tensor | None,
    apply_silu: bool,
    exchange_ptrs: torch.Tensor,
    epochs: torch.Tensor,
    rank: int,
    world: int,
    max_polls: int,
    status: torch.Tensor | None,
    flags: int,
) -> None:
    """Backward of a batch shard with dweight/dbias summed over `world` ranks
    in the same kernel (cc1d_bwd_peer_reduce).  exchange_ptrs: int64 device
    tensor of the ranks' peer-mapped exchange buffer addresses.  status:
    optional int32 device word, incremented by every wait for a peer that
    gave up (the outputs it could not reduce are written as NaN).
    max_polls (0 = the library default) and status are passed explicitly:
    a mutated argument of a custom op must be present in every call.
    flags: _lib.PEER_FUSED, or PEER_PUSH (backward + push, outputs not
    written) followed later by PEER_FINISH with the same arguments (only the
    wait and the outputs; x, dout and dx are not touched)."""
    _require_cuda(x, "causal_conv1d_fn backward (peer reduce)")
    lib = _lib.load()
    p = _bwd_params(x, weight, bias, dout, None, initial_states, dfinal_states, dx, dwdb_acc, dinitial_states,
                    dweight_out, dbias_out, apply_silu)
    q = _lib.PeerReduceParams()
    q.rank, q.world = rank, world
    q.exchange, q.epochs = exchange_ptrs.data_ptr(), epochs.data_ptr()
    q.max_polls = max_polls
    q.flags = flags
    q.status = _ptr(status)
    with _on_device(x.device):
        nbytes = bwd_workspace_bytes(p) if flags != _lib.PEER_FINISH else 0
        ws = None
        if nbytes > 0:
            ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
            p.workspace = ws.data_ptr()
            p.workspace_bytes = nbytes
        _lib.check(lib.cc1d_bwd_peer_reduce(ctypes.byref(p), ctypes.byref(q), _stream(x.device)),
                   "cc1d_bwd_peer_reduce")
        del ws


def _bwd_peer_fake(x, weight, bias, dout, initial_states, dfinal_states, dx, dwdb_acc, dinitial_states,
                   dweight_out, dbias_out, apply_silu, exchange_ptrs, epochs, rank, world, max_polls,
                   status, flags) -> None:
    return None


bwd_peer = torch.library.custom_op(
    "causal_conv1d_b200::bwd_peer",
    mutates_args=("dx", "dwdb_acc", "dinitial_states", "dweight_out", "dbias_out", "epochs", "status"),
)(_bwd_peer_impl)
bwd_peer.register_fake(_bwd_peer_fake)


def _update_impl(
    x: torch.Tensor,
    conv_state: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    cache_seqlens: torch.Tensor | None,
    conv_state_indices: torch.Tensor | None,
    out: torch.Tensor,
    apply_silu: bool,
) -> None:
    _require_cuda(x, "causal_conv1d_update")
    lib = _lib.load()
    p = _lib.UpdateParams()
    p.dtype = _DTYPE_CODE[x.dtype]
    p.width = weight.shape[1]
    p.batch, p.dim, p.seqlen = x.shape
    p.state_len = conv_state.shape[2]
    p.state_rows = conv_state.shape[0]
    p.silu = 1 if apply_silu else 0
    p.x = x.data_ptr()
    p.x_batch_stride, p.x_dim_stride, p.x_seq_stride = x.stride()
    p.weight = weight.data_ptr()
    p.weight_dim_stride, p.weight_width_stride = weight.stride()
    if bias is not None:
        p.bias = bias.data_ptr()
        p.bias_stride = bias.stride(0)
    p.conv_state = conv_state.data_ptr()
    p.state_batch_stride, p.state_dim_stride, p.state_seq_stride = conv_state.stride()
    p.conv_state_indices = _ptr(conv_state_indices)
    p.cache_seqlens = _ptr(cache_seqlens)
    p.out = out.data_ptr()
    p.out_batch_stride, p.out_dim_stride, p.out_seq_stride = out.stride()
    with _on_device(x.device):
        _lib.check(lib.cc1d_update(ctypes.byref(p), _stream(x.device)), "cc1d_update")


def _update_fake(x, conv_state, weight, bias, cache_seqlens, conv_state_indices, out, apply_silu) -> None:
    return None


update = torch.library.custom_op("causal_conv1d_b200::update", mutates_args=("conv_state", "out"))(_update_impl)
update.register_fake(_update_fake)


def _varlen_impl(x: torch.Tensor, cu_seqlens: torch.Tensor, states: torch.Tensor) -> None:
    _require_cuda(x, "causal_conv1d_varlen_states")
    lib = _lib.load()
    p = _lib.VarlenParams()
    p.dtype = _DTYPE_CODE[x.dtype]
    p.batch, p.dim, p.state_len = states.shape
    p.total_tokens = x.shape[0]
    p.x = x.data_ptr()
    p.x_token_stride, p.x_dim_stride = x.stride()
    p.cu_seqlens = cu_seqlens.data_ptr()
    p.states = states.data_ptr()
    p.states_batch_stride, p.states_dim_stride, p.states_seq_stride = states.stride()
    with _on_device(x.device):
        _lib.check(lib.cc1d_varlen_states(ctypes.byref(p), _stream(x.device)), "cc1d_varlen_states")


def _varlen_fake(x, cu_seqlens, states) -> None:
    return None


varlen_states = torch.library.custom_op("causal_conv1d_b200::varlen_states", mutates_args=("states",))(_varlen_impl)
varlen_states.register_fake(_varlen_fake)


def _inproj_conv_impl(
    hidden: torch.Tensor,
    in_weight: torch.Tensor,
    conv_weight: torch.Tensor,
    conv_bias: torch.Tensor | None,
    initial_states: torch.Tensor | None,
    out: torch.Tensor,
    apply_silu: bool,
    final_states_out: torch.Tensor | None,
) -> None:
    """out (B, L, N) = conv(hidden (B, L, K) @ in_weight (N, K)^T) in one kernel
    (cc1d_inproj_conv_fwd); final_states_out (B, N, W-1) optional."""
    _require_cuda(hidden, "in_proj_causal_conv1d")
    lib = _lib.load()
    B, L, K = hidden.shape
    N, W = conv_weight.shape
    p = _lib.InprojConvParams()
    p.dtype = _DTYPE_CODE[hidden.dtype]
    p.width = W
    p.batch, p.seqlen, p.dim, p.hidden_dim = B, L, N, K
    p.silu = 1 if apply_silu else 0
    p.hidden = hidden.data_ptr()
    p.hidden_row_stride = hidden.stride(1)
    p.in_weight = in_weight.data_ptr()
    p.in_weight_row_stride = in_weight.stride(0)
    p.conv_weight = conv_weight.data_ptr()
    p.conv_weight_dim_stride, p.conv_weight_width_stride = conv_weight.stride()
    if conv_bias is not None:
        p.conv_bias, p.conv_bias_stride = conv_bias.data_ptr(), conv_bias.stride(0)
    if initial_states is not None:
        p.initial_states = initial_states.data_ptr()
        p.init_batch_stride, p.init_dim_stride, p.init_seq_stride = initial_states.stride()
    p.out = out.data_ptr()
    p.out_row_stride = out.stride(1)
    if final_states_out is not None:
        p.final_states = final_states_out.data_ptr()
        p.final_batch_stride, p.final_dim_stride, p.final_seq_stride = final_states_out.stride()
    with _on_device(hidden.device):
        _lib.check(lib.cc1d_inproj_conv_fwd(ctypes.byref(p), _stream(hidden.device)), "cc1d_inproj_conv_fwd")


def _inproj_conv_fake(hidden, in_weight, conv_weight, conv_bias, initial_states, out, apply_silu,
                      final_states_out) -> None:
    return None


inproj_conv = torch.library.custom_op(
    "causal_conv1d_b200::inproj_conv", mutates_args=("out", "final_states_out"))(_inproj_conv_impl)
inproj_conv.register_fake(_inproj_conv_fake)
