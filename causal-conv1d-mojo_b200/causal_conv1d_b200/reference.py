"""Pure-PyTorch reference implementations exported by the public API.

``causal_conv1d_ref`` and ``causal_conv1d_update_ref`` have the semantics of
the reference package's functions of the same names
(src/causal_conv1d_mojo/reference.py:21-121, themselves upstream
causal-conv1d's references): the conv runs in the weight dtype through
``torch.nn.functional`` and the result is cast back to the input dtype.
They run on any device and are meant for validating kernels and for
hardware without the sm_100a kernels; the product path never calls them.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def causal_conv1d_ref(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    initial_states: torch.Tensor | None = None,
    return_final_states: bool = False,
    final_states_out: torch.Tensor | None = None,
    activation: str | None = None,
) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
    """
    x: (batch, dim, seqlen); weight: (dim, width); bias: (dim,)
    initial_states / final_states_out: (batch, dim, width - 1)

    out: (batch, dim, seqlen)
    """
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("activation must be None, silu, or swish")
    in_dtype = x.dtype
    dim, width = weight.shape
    seqlen = x.shape[-1]
    kernel = weight.unsqueeze(1)  # (dim, 1, width): one filter per channel
    xs = x.to(weight.dtype)
    if initial_states is not None:
        # Prepend the carried context; no implicit zero padding needed.
        xs = torch.cat([initial_states.to(weight.dtype), xs], dim=-1)
        pre = F.conv1d(xs, kernel, bias, padding=0, groups=dim)
    else:
        pre = F.conv1d(xs, kernel, bias, padding=width - 1, groups=dim)
    pre = pre[..., :seqlen]
    y = pre if activation is None else F.silu(pre)
    y = y.to(in_dtype)
    if not return_final_states:
        return y
    # The last width-1 columns of the (possibly prefixed) input, left
    # zero-padded when there are fewer than width-1 columns.
    have = xs.shape[-1]
    if have >= width - 1:
        tail = xs[..., have - (width - 1):]
    else:
        tail = F.pad(xs, (width - 1 - have, 0))
    tail = tail.to(in_dtype)
    if final_states_out is not None:
        final_states_out.copy_(tail)
    else:
        final_states_out = tail
    return y, final_states_out


def causal_conv1d_update_ref(
    x: torch.Tensor,
    conv_state: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    activation: str | None = None,
    cache_seqlens: torch.Tensor | None = None,
) -> torch.Tensor:
    """
    x: (batch, dim) or (batch, dim, seqlen)
    conv_state: (batch, dim, state_len), state_len >= width - 1; updated in place
    cache_seqlens: (batch,) int32 or None; if given conv_state is a circular
        buffer written from cache_seqlens % state_len.

    out: same shape as x
    """
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("activation must be None, silu, or swish")
    in_dtype = x.dtype
    squeeze = x.dim() == 2
    if squeeze:
        x = x.unsqueeze(-1)
    batch, dim, seqlen = x.shape
    width = weight.shape[1]
    state_len = conv_state.shape[-1]
    assert conv_state.shape == (batch, dim, state_len)
    assert weight.shape == (dim, width)
    if cache_seqlens is None:
        window = torch.cat([conv_state, x], dim=-1).to(weight.dtype)
        conv_state.copy_(window[..., window.shape[-1] - state_len:])
    else:
        offs = torch.arange(-(width - 1), 0, device=x.device, dtype=torch.long)
        hist_pos = torch.remainder(cache_seqlens.long().unsqueeze(1) + offs, state_len)
        hist = conv_state.gather(2, hist_pos.unsqueeze(1).expand(batch, dim, width - 1))
        window = torch.cat([hist, x], dim=-1).to(weight.dtype)
        write_pos = torch.remainder(
            cache_seqlens.long().unsqueeze(1) + torch.arange(seqlen, device=x.device), state_len
        )
        conv_state.scatter_(2, write_pos.unsqueeze(1).expand(batch, dim, seqlen), x)
    # Sliding windows of `width` columns; keep the last `seqlen` outputs.
    taps = window.unfold(-1, width, 1)  # (batch, dim, n_windows, width)
    out = (taps * weight.view(1, dim, 1, width)).sum(-1)[..., -seqlen:]
    if bias is not None:
        out = out + bias.view(1, dim, 1)
    if activation is not None:
        out = F.silu(out)
    if squeeze:
        out = out.squeeze(-1)
    return out.to(in_dtype)
