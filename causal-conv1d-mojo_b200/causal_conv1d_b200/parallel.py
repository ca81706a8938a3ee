"""Sharding of causal_conv1d_fn across GPUs (one process per GPU).

Every (batch, channel) row of the conv is independent, so the work shards
with no data exchange:

* dim sharding  -- rank r owns channels [d0, d1): x, weight, bias and the
  states are sliced along dim.  Forward and backward need no collective.
* batch sharding -- rank r owns batch rows [b0, b1) and the full weights.
  The forward needs nothing; the backward produces partial weight/bias
  gradients, summed with ONE all-reduce of the fp32 buffer
  [dweight (dim, W) | dbias (dim)] that the backward kernel writes.  At the
  Mamba shapes that buffer is ~100-170 KB, so the collective is
  latency-bound.

The all-reduce goes through ``torch.distributed`` (NCCL on GPUs; the host
logic is exercised with gloo on CPU).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _ops
from ._fn import _like_layout


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) of `n` items owned by `rank` of `world`
    (the first n % world ranks get one extra item)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def dim_shard(weight: torch.Tensor, bias: torch.Tensor | None, rank: int, world: int):
    """Channel slice of the parameters owned by `rank` (views, no copy)."""
    d0, d1 = shard_range(weight.shape[0], rank, world)
    return weight[d0:d1], (bias[d0:d1] if bias is not None else None), (d0, d1)


def split_dwdb(dwdb: torch.Tensor, dim: int, width: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Views (dweight (dim, width), dbias (dim,)) of the packed fp32 buffer."""
    if dwdb.numel() != dim * (width + 1) or dwdb.dtype != torch.float32:
        raise ValueError("dwdb must be a float32 buffer of dim*(width+1) elements")
    return dwdb[: dim * width].view(dim, width), dwdb[dim * width:]


def allreduce_weight_grads(dwdb: torch.Tensor, group=None) -> torch.Tensor:
    """Sum the packed fp32 [dweight | dbias] buffer over the ranks of `group`
    (in place, one collective).  No-op when torch.distributed is not
    initialised or the group has a single rank."""
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(dwdb, op=dist.ReduceOp.SUM, group=group)
    return dwdb


class _BatchShardedFn(torch.autograd.Function):
    """causal_conv1d_fn over a batch shard; backward all-reduces dW/db."""

    @staticmethod
    def forward(ctx, x, weight, bias, initial_states, apply_silu, final_states_out, group):
        out = torch.empty_like(x)
        _ops.fwd(x, weight, bias, None, initial_states, out, apply_silu, final_states_out)
        ctx.save_for_backward(x, weight, bias, initial_states)
        ctx.apply_silu = apply_silu
        ctx.group = group
        ctx.return_final_states = final_states_out is not None
        if final_states_out is not None:
            return out, final_states_out
        return out

    @staticmethod
    def backward(ctx, *grads):
        dout = grads[0]
        dfinal = grads[1] if ctx.return_final_states else None
        x, weight, bias, initial_states = ctx.saved_tensors
        D, W = weight.shape
        dout = _like_layout(dout, x)
        dx = torch.empty_like(x)
        dwdb = torch.empty(D * (W + 1), dtype=torch.float32, device=x.device)
        dinit = torch.empty_like(initial_states) if initial_states is not None else None
        _ops.bwd(x, weight, bias, dout, None, initial_states, dfinal, dx, dwdb, dinit, None, None, ctx.apply_silu)
        allreduce_weight_grads(dwdb, ctx.group)
        dw, db = split_dwdb(dwdb, D, W)
        return (dx, dw.to(weight.dtype), db.to(bias.dtype) if bias is not None else None, dinit, None, None, None)


def causal_conv1d_fn_batch_sharded(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    initial_states: torch.Tensor | None = None,
    return_final_states: bool = False,
    activation: str | None = None,
    group=None,
):
    """causal_conv1d_fn on this rank's batch shard `x` with replicated
    weight/bias: weight.grad / bias.grad come out summed over all ranks of
    `group` (the data-parallel gradient), x.grad stays local."""
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("only activation in {None, 'silu', 'swish'} is supported")
    batch, dim, _ = x.shape
    width = weight.shape[1]
    fs = torch.empty(batch, dim, width - 1, dtype=x.dtype, device=x.device) if return_final_states else None
    return _BatchShardedFn.apply(x, weight, bias, initial_states, activation in ("silu", "swish"), fs, group)
