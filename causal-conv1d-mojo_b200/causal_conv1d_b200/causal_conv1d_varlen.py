"""Packed variable-length helpers: ``causal_conv1d_varlen_states``.

Given packed tokens x (total_tokens, dim) and cumulative lengths
cu_seqlens (batch + 1,), produce the conv states (batch, dim, state_len)
holding the last state_len tokens of every sequence, left zero-padded --
the hand-off from a packed prefill to decoding.

The reference (src/causal_conv1d_mojo/causal_conv1d_varlen.py:29-61) loops
over sequences in Python with one torch copy each; here one CUDA launch
gathers every sequence.  ``causal_conv1d_varlen_states_ref`` is the
pure-PyTorch reference with the same output (bit-exact, pure data movement).
"""

from __future__ import annotations

import torch

from . import _ops


def causal_conv1d_varlen_states(x: torch.Tensor, cu_seqlens: torch.Tensor, state_len: int) -> torch.Tensor:
    """Extract the trailing `state_len` tokens of each packed sequence.

    Args:
        x: (total_tokens, dim) packed batch of token activations.
        cu_seqlens: (batch + 1,) cumulative sequence lengths starting at 0,
            non-decreasing.
        state_len: tokens kept per sequence; shorter sequences are left
            zero-padded.

    Returns:
        states: (batch, dim, state_len) with x's dtype and device, stored as
        (batch, state_len, dim) in memory like upstream.
    """
    _, dim = x.shape
    batch = cu_seqlens.shape[0] - 1
    states = torch.empty(batch, state_len, dim, dtype=x.dtype, device=x.device).transpose(1, 2)
    if cu_seqlens.device != x.device:
        raise ValueError(f"cu_seqlens.device ({cu_seqlens.device}) must match x.device ({x.device})")
    cu = cu_seqlens
    if cu.dtype != torch.int32:
        cu = cu.to(torch.int32)
    cu = cu.contiguous()
    _ops.varlen_states(x, cu, states)
    return states


def causal_conv1d_varlen_states_ref(x: torch.Tensor, cu_seqlens: torch.Tensor, state_len: int) -> torch.Tensor:
    """Pure-PyTorch reference of :func:`causal_conv1d_varlen_states`."""
    _, dim = x.shape
    batch = cu_seqlens.shape[0] - 1
    states = torch.zeros(batch, state_len, dim, dtype=x.dtype, device=x.device).transpose(1, 2)
    bounds = cu_seqlens.tolist()
    for i in range(batch):
        end = int(bounds[i + 1])
        start = max(int(bounds[i]), end - state_len)
        n = end - start
        if n > 0:
            states[i, :, state_len - n:] = x[start:end].transpose(0, 1)
    return states
