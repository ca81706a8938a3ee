"""The in_proj GEMM of a Mamba block fused with causal_conv1d_fn's forward.

In a Mamba block the conv's input xBC is the output of the in_proj linear
layer; run separately, xBC is written to HBM by the GEMM and read back by the
conv.  ``in_proj_causal_conv1d`` computes

    xBC = hidden @ in_weight.T                      # (B, L, N), never stored
    out = causal_conv1d_fn(xBC as (B, N, L), conv_weight, conv_bias,
                           initial_states, activation)

in one sm_100a kernel (tcgen05 tensor-core GEMM whose epilogue applies the
conv), with xBC rounded to bf16 before the conv exactly as a stored bf16 GEMM
output would be.  Forward only (prefill / inference); bf16; widths 2..4.
The reference package has no such fused op: this is the neighbouring step of
the conv, the call pair it replaces is ``F.linear`` then ``causal_conv1d_fn``.
"""

from __future__ import annotations

import torch

from . import _ops


def in_proj_causal_conv1d(
    hidden: torch.Tensor,
    in_weight: torch.Tensor,
    conv_weight: torch.Tensor,
    conv_bias: torch.Tensor | None = None,
    initial_states: torch.Tensor | None = None,
    return_final_states: bool = False,
    activation: str | None = None,
):
    """
    hidden: (batch, seqlen, hidden_dim) bf16, unit stride over hidden_dim
    in_weight: (dim, hidden_dim) bf16 (an nn.Linear weight)
    conv_weight: (dim, width), conv_bias: (dim,), width in 2..4
    initial_states: (batch, dim, width - 1) or None

    Returns out (batch, dim, seqlen) in channel-last strides -- the layout
    causal_conv1d_fn returns for a channel-last input -- or
    (out, final_states) with final_states (batch, dim, width - 1) holding the
    last width-1 columns of xBC.
    """
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("activation must be None, silu, or swish")
    if hidden.dim() != 3 or in_weight.dim() != 2 or conv_weight.dim() != 2:
        raise ValueError("hidden must be (batch, seqlen, hidden_dim), in_weight (dim, hidden_dim), "
                         "conv_weight (dim, width)")
    B, L, K = hidden.shape
    N, W = conv_weight.shape
    if in_weight.shape != (N, K):
        raise ValueError(f"in_weight must be ({N}, {K}), got {tuple(in_weight.shape)}")
    for name, t in (("hidden", hidden), ("in_weight", in_weight), ("conv_weight", conv_weight),
                    ("conv_bias", conv_bias), ("initial_states", initial_states)):
        if t is not None and t.dtype != torch.bfloat16:
            raise NotImplementedError(f"{name} must be bfloat16 (the fused kernel is bf16 only)")
    if conv_bias is not None and conv_bias.shape != (N,):
        raise ValueError(f"conv_bias must be ({N},)")
    if initial_states is not None and initial_states.shape != (B, N, W - 1):
        raise ValueError(f"initial_states must be ({B}, {N}, {W - 1})")
    if hidden.stride(2) != 1:
        hidden = hidden.contiguous()
    if in_weight.stride(1) != 1:
        in_weight = in_weight.contiguous()
    out = torch.empty(B, L, N, dtype=hidden.dtype, device=hidden.device)
    fs = torch.empty(B, N, W - 1, dtype=hidden.dtype, device=hidden.device) if return_final_states else None
    _ops.inproj_conv(hidden, in_weight, conv_weight, conv_bias, initial_states, out,
                     activation in ("silu", "swish"), fs)
    out = out.transpose(1, 2)
    return (out, fs) if return_final_states else out
