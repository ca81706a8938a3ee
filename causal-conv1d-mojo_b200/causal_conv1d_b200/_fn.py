"""``causal_conv1d_fn``: the forward + autograd backward API.

Same signature, defaults, validation order, error types and messages as the
reference (src/causal_conv1d_mojo/_fn.py:335-520), so code written for
causal-conv1d-mojo (or Tri Dao's causal-conv1d) runs unchanged.  After
validation every call goes to the sm_100a kernels through the
``causal_conv1d_b200::fwd`` / ``::bwd`` custom ops; CPU tensors are rejected.

Differences from the reference, all on the GPU side of the boundary:
  * final_states is written by the forward kernel itself (no separate copy)
    and, with initial_states and seqlen < W-1, holds the last W-1 columns of
    cat([initial_states, x]) as the pure-PyTorch reference does
    (src/causal_conv1d_mojo/reference.py:50-56);
  * the backward consumes dout in the layout of x (copying only when the two
    differ), folds dfinal_states into dx / dinitial_states inside the kernel,
    and reduces dweight/dbias deterministically (no atomics), writing the
    parameter-dtype gradients directly.
"""

from __future__ import annotations

import torch

from . import _ops

_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def _same_layout(t: torch.Tensor, ref: torch.Tensor) -> bool:
    """True when `t` walks memory along the same unit-stride axis as `ref`."""
    if ref.stride(-1) == 1 or ref.shape[-1] <= 1:
        return t.stride(-1) == 1 or t.shape[-1] <= 1
    if ref.stride(1) == 1:
        return t.stride(1) == 1 or t.shape[1] <= 1
    return True


def _like_layout(t: torch.Tensor, ref: torch.Tensor) -> torch.Tensor:
    """`t` with the memory layout of `ref` (a copy only when needed)."""
    if _same_layout(t, ref):
        return t
    out = torch.empty_like(ref)
    out.copy_(t)
    return out


class _CausalConv1dFn(torch.autograd.Function):
    """Autograd op; forward and backward are single custom-op calls.

    Mirrors the reference's `_CausalConv1dFn`
    (src/causal_conv1d_mojo/_fn.py:204-332): same inputs, same returned
    tuple shape, the same set of saved tensors.
    """

    @staticmethod
    def forward(ctx, x, weight, bias, seq_idx, initial_states, apply_silu, final_states_out):
        out = torch.empty_like(x)
        _ops.fwd(x, weight, bias, seq_idx, initial_states, out, apply_silu, final_states_out)
        ctx.save_for_backward(x, weight, bias, seq_idx, initial_states)
        ctx.apply_silu = apply_silu
        ctx.return_final_states = final_states_out is not None
        if final_states_out is not None:
            return out, final_states_out
        return out

    @staticmethod
    def backward(ctx, *grad_outputs):
        dout = grad_outputs[0]
        dfinal = grad_outputs[1] if ctx.return_final_states else None
        x, weight, bias, seq_idx, initial_states = ctx.saved_tensors
        D, W = weight.shape
        dout = _like_layout(dout, x)
        if dfinal is not None and dfinal.dtype != x.dtype:
            dfinal = dfinal.to(x.dtype)
        dx = torch.empty_like(x)
        dwdb = torch.empty(D * (W + 1), dtype=torch.float32, device=x.device)
        dweight = torch.empty(D, W, dtype=weight.dtype, device=x.device)
        dbias = torch.empty(D, dtype=bias.dtype, device=x.device) if bias is not None else None
        dinit = torch.empty_like(initial_states) if initial_states is not None else None
        _ops.bwd(x, weight, bias, dout, seq_idx, initial_states, dfinal, dx, dwdb, dinit, dweight, dbias,
                 ctx.apply_silu)
        return dx, dweight, dbias, None, dinit, None, None


def causal_conv1d_fn(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    seq_idx: torch.Tensor | None = None,
    initial_states: torch.Tensor | None = None,
    return_final_states: bool = False,
    final_states_out: torch.Tensor | None = None,
    activation: str | None = None,
) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
    """
    x: (batch, dim, seqlen)
    weight: (dim, width)
    bias: (dim,)
    seq_idx: (batch, seqlen)
    initial_states: (batch, dim, width - 1)
    final_states_out: (batch, dim, width - 1), to be written to
    activation: either None or "silu" or "swish"

    out: (batch, dim, seqlen)
    """
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("only activation in {None, 'silu', 'swish'} is supported")
    if x.dtype not in _DTYPES:
        raise NotImplementedError(f"unsupported dtype {x.dtype}; only fp16/bf16/fp32 are supported")
    if weight.dtype != x.dtype:
        raise NotImplementedError(f"weight.dtype ({weight.dtype}) must match x.dtype ({x.dtype})")
    if bias is not None and bias.dtype != x.dtype:
        raise NotImplementedError(f"bias.dtype ({bias.dtype}) must match x.dtype ({x.dtype})")
    width = weight.shape[1]
    max_width = 5 if x.dtype == torch.float32 else 9
    if width < 2 or width > max_width:
        dtype_clause = "" if x.dtype == torch.float32 else " for fp32"
        raise NotImplementedError(
            f"width must be in 2..{max_width}{dtype_clause} (got {width}). "
            f"Widths outside this range are not supported."
        )
    if width > 5 and x.requires_grad and x.shape[-1] % 1024 != 0:
        raise NotImplementedError(
            f"width > 5 with autograd requires seqlen aligned to 1024 "
            f"(got seqlen={x.shape[-1]}, width={width})."
        )
    if x.device != weight.device or (bias is not None and x.device != bias.device):
        raise NotImplementedError(
            f"x, weight, bias must all be on the same device "
            f"(got x={x.device}, weight={weight.device}, "
            f"bias={'None' if bias is None else bias.device})"
        )
    if final_states_out is not None and not return_final_states:
        raise ValueError("final_states_out is only meaningful when return_final_states=True")

    batch, dim, seqlen = x.shape
    if seq_idx is not None:
        if return_final_states:
            raise ValueError(
                "seq_idx and return_final_states are mutually exclusive "
                "(packed sequences have no single 'last W-1 cols')"
            )
        if initial_states is not None:
            raise ValueError("seq_idx and initial_states are mutually exclusive")
        if seq_idx.shape != (batch, seqlen):
            raise ValueError(f"seq_idx shape {tuple(seq_idx.shape)} != expected {(batch, seqlen)}")
        if seq_idx.dtype != torch.int32:
            raise ValueError(f"seq_idx.dtype must be int32 (got {seq_idx.dtype})")
        if seq_idx.device != x.device:
            raise ValueError(f"seq_idx.device ({seq_idx.device}) must match x.device ({x.device})")
        if not seq_idx.is_contiguous():
            seq_idx = seq_idx.contiguous()

    if initial_states is not None:
        if initial_states.shape != (batch, dim, width - 1):
            raise ValueError(
                f"initial_states shape {tuple(initial_states.shape)} != expected {(batch, dim, width - 1)}"
            )
        if initial_states.dtype != x.dtype:
            raise ValueError(f"initial_states.dtype ({initial_states.dtype}) must match x.dtype ({x.dtype})")
        if initial_states.device != x.device:
            raise ValueError(
                f"initial_states.device ({initial_states.device}) must match x.device ({x.device})"
            )

    if return_final_states:
        if final_states_out is None:
            final_states_out = torch.empty(batch, dim, width - 1, dtype=x.dtype, device=x.device)
        else:
            if final_states_out.shape != (batch, dim, width - 1):
                raise ValueError(
                    f"final_states_out shape {tuple(final_states_out.shape)} != expected {(batch, dim, width - 1)}"
                )
            if final_states_out.dtype != x.dtype:
                raise ValueError(
                    f"final_states_out.dtype ({final_states_out.dtype}) must match x.dtype ({x.dtype})"
                )
            if final_states_out.device != x.device:
                raise ValueError(
                    f"final_states_out.device ({final_states_out.device}) must match x.device ({x.device})"
                )

    apply_silu = activation in ("silu", "swish")
    return _CausalConv1dFn.apply(x, weight, bias, seq_idx, initial_states, apply_silu, final_states_out)
