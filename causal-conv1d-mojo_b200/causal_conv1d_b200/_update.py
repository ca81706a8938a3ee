"""``causal_conv1d_update``: the decode-step API.

Same signature, validation, error types and messages as the reference
(src/causal_conv1d_mojo/_update.py:24-231); the work is one launch of the
sm_100a update kernel through the ``causal_conv1d_b200::update`` custom op.
conv_state is mutated in place; cache_seqlens is read, never advanced.
"""

from __future__ import annotations

import torch

from . import _ops

_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def causal_conv1d_update(
    x: torch.Tensor,
    conv_state: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    activation: str | None = None,
    cache_seqlens: torch.Tensor | None = None,
    conv_state_indices: torch.Tensor | None = None,
) -> torch.Tensor:
    """Single-step (or short-burst) causal conv1d update for decoding.

    x: (batch, dim) or (batch, dim, seqlen) -- the new tokens
    conv_state: (batch_or_pool_size, dim, state_len), state_len >= width - 1,
        mutated in place.  Linear mode drops the oldest `seqlen` values and
        appends x; circular mode (cache_seqlens given) writes x at
        cache_seqlens[b] modulo state_len.
    weight: (dim, width); bias: (dim,) or None
    activation: None | "silu" | "swish"
    cache_seqlens: (batch,) int32 or None -- per-batch write head.
    conv_state_indices: (batch,) int32 or None -- row of conv_state serving
        batch element b; a negative index zeroes out[b] and leaves the state
        untouched.  cache_seqlens stays indexed by b.

    Returns: out with the same shape as x.
    """
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("only activation in {None, 'silu', 'swish'} is supported")
    if x.dtype not in _DTYPES:
        raise NotImplementedError(f"unsupported dtype {x.dtype}; only fp16/bf16/fp32 are supported")
    if weight.dtype != x.dtype:
        raise NotImplementedError(f"weight.dtype ({weight.dtype}) must match x.dtype ({x.dtype})")
    if bias is not None and bias.dtype != x.dtype:
        raise NotImplementedError(f"bias.dtype ({bias.dtype}) must match x.dtype ({x.dtype})")
    if conv_state.dtype != x.dtype:
        raise NotImplementedError(f"conv_state.dtype ({conv_state.dtype}) must match x.dtype ({x.dtype})")
    width = weight.shape[1]
    if width < 2 or width > 9:
        raise NotImplementedError(f"width must be in 2..9 (got {width}).")

    unsqueeze = x.dim() == 2
    if unsqueeze:
        x = x.unsqueeze(-1)

    batch, dim, seqlen = x.shape
    state_len = conv_state.shape[-1]
    if conv_state_indices is None:
        if conv_state.shape != (batch, dim, state_len):
            raise ValueError(
                f"conv_state shape {tuple(conv_state.shape)} != expected {(batch, dim, state_len)}"
            )
    else:
        if conv_state.shape[1] != dim or conv_state.shape[2] != state_len:
            raise ValueError(f"conv_state shape {tuple(conv_state.shape)}: expected (*, {dim}, {state_len})")
    if state_len < width - 1:
        raise ValueError(f"conv_state.shape[-1]={state_len} must be >= width-1={width - 1}")
    if (
        x.device != weight.device
        or x.device != conv_state.device
        or (bias is not None and x.device != bias.device)
    ):
        raise NotImplementedError("x, weight, bias, conv_state must all be on the same device")

    if cache_seqlens is not None:
        if cache_seqlens.shape != (batch,):
            raise ValueError(f"cache_seqlens shape {tuple(cache_seqlens.shape)} != expected {(batch,)}")
        if cache_seqlens.dtype != torch.int32:
            raise ValueError(f"cache_seqlens.dtype must be int32 (got {cache_seqlens.dtype})")
        if cache_seqlens.device != x.device:
            raise ValueError(
                f"cache_seqlens.device ({cache_seqlens.device}) must match x.device ({x.device})"
            )
        if not cache_seqlens.is_contiguous():
            cache_seqlens = cache_seqlens.contiguous()

    if conv_state_indices is not None:
        if conv_state_indices.shape != (batch,):
            raise ValueError(
                f"conv_state_indices shape {tuple(conv_state_indices.shape)} != expected {(batch,)}"
            )
        if conv_state_indices.dtype != torch.int32:
            raise ValueError(f"conv_state_indices.dtype must be int32 (got {conv_state_indices.dtype})")
        if conv_state_indices.device != x.device:
            raise ValueError(
                f"conv_state_indices.device ({conv_state_indices.device}) must match x.device ({x.device})"
            )
        if not conv_state_indices.is_contiguous():
            conv_state_indices = conv_state_indices.contiguous()

    out = torch.empty_like(x)
    apply_silu = activation in ("silu", "swish")
    _ops.update(x, conv_state, weight, bias, cache_seqlens, conv_state_indices, out, apply_silu)
    if unsqueeze:
        out = out.squeeze(-1)
    return out
