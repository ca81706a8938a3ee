"""Helpers for the GPU parity tests: memory layouts and seeded inputs."""

from __future__ import annotations

import torch

LAYOUTS = ["contig", "chanlast", "sliced", "strided"]


def with_layout(t: torch.Tensor, layout: str) -> torch.Tensor:
    """Same values as the (B, D, L) tensor `t`, stored in another layout.

    contig   -- (D*L, L, 1)
    chanlast -- (L*D, 1, D): the Mamba layout, dim is the unit-stride axis
    sliced   -- unit seqlen stride, but a channel stride of 2*(L+5) and an
                odd element offset (vector loads must fall back)
    strided  -- no unit-stride axis at all (channel stride 2)
    """
    B, D, L = t.shape
    if layout == "contig":
        return t.contiguous()
    if layout == "chanlast":
        return t.transpose(1, 2).contiguous().transpose(1, 2)
    if layout == "sliced":
        big = torch.zeros(B, 2 * D, L + 5, dtype=t.dtype, device=t.device)
        v = big[:, ::2, 3:3 + L]
        v.copy_(t)
        return v
    if layout == "strided":
        big = torch.zeros(B, L, D, 2, dtype=t.dtype, device=t.device)
        v = big[..., 0].transpose(1, 2)
        v.copy_(t)
        return v
    raise ValueError(layout)


def seeded(shape, dtype, seed, kind="normal", device="cpu"):
    g = torch.Generator("cpu").manual_seed(seed)
    if kind == "normal":
        t = torch.randn(*shape, generator=g)
    else:  # uniform(-0.5, 0.5)
        t = torch.rand(*shape, generator=g) - 0.5
    return t.to(dtype).to(device)


def random_seq_idx(B, L, seed, pad=True):
    """Random runs of sequence ids (lengths 1..40), some runs padding (-1)."""
    g = torch.Generator("cpu").manual_seed(seed)
    out = torch.empty(B, L, dtype=torch.int32)
    for b in range(B):
        t, sid = 0, 0
        while t < L:
            n = int(torch.randint(1, 41, (1,), generator=g))
            val = -1 if (pad and torch.rand(1, generator=g).item() < 0.2) else sid
            out[b, t:t + n] = val
            sid += 1
            t += n
    return out
