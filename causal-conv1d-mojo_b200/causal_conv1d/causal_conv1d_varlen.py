"""Upstream module path ``causal_conv1d.causal_conv1d_varlen``."""

from causal_conv1d_b200.causal_conv1d_varlen import (  # noqa: F401
    causal_conv1d_varlen_states,
    causal_conv1d_varlen_states_ref,
)
