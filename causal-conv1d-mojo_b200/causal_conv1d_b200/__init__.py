"""causal_conv1d_b200: causal depthwise conv1d for NVIDIA B200 (sm_100a).

A drop-in for the public API of causal-conv1d-mojo (and of Tri Dao's
causal-conv1d): ``causal_conv1d_fn`` (forward + autograd backward),
``causal_conv1d_update`` (decode step), ``causal_conv1d_varlen_states``,
and the pure-PyTorch references ``causal_conv1d_ref`` /
``causal_conv1d_update_ref`` / ``causal_conv1d_varlen_states_ref``.

The compute runs in hand-written CUDA kernels compiled ahead of time for
sm_100a into ``libcc1d_sm100.so`` (C ABI: include/cc1d.h) and called through
``torch.library`` custom ops.  There is no JIT and no CPU fallback.
"""

from __future__ import annotations

from ._fn import causal_conv1d_fn
from ._update import causal_conv1d_update
from .causal_conv1d_varlen import causal_conv1d_varlen_states, causal_conv1d_varlen_states_ref
from .reference import causal_conv1d_ref, causal_conv1d_update_ref

__version__ = "1.6.1"

__all__ = [
    "causal_conv1d_fn",
    "causal_conv1d_ref",
    "causal_conv1d_update",
    "causal_conv1d_update_ref",
    "causal_conv1d_varlen_states",
    "causal_conv1d_varlen_states_ref",
]
