"""``import causal_conv1d`` shim over causal_conv1d_b200.

Lets code written against Tri Dao's causal-conv1d (or the
causal-conv1d-mojo compatibility package,
compat/src/causal_conv1d/__init__.py:1-48 in that project) run on the
sm_100a kernels unchanged.  Both distributions would own the same import
name, so loading is refused when upstream's files sit next to this one.
"""

from __future__ import annotations

from pathlib import Path as _Path

if (_Path(__file__).resolve().parent / "causal_conv1d_interface.py").is_file():
    raise ImportError(
        "Both upstream `causal-conv1d` and this `causal_conv1d` shim over causal_conv1d_b200 are "
        "installed in the same directory; they conflict on the `causal_conv1d` import name. "
        "Uninstall one of them."
    )

from causal_conv1d_b200 import (  # noqa: E402
    __version__,
    causal_conv1d_fn,
    causal_conv1d_ref,
    causal_conv1d_update,
    causal_conv1d_update_ref,
)

__all__ = [
    "__version__",
    "causal_conv1d_fn",
    "causal_conv1d_ref",
    "causal_conv1d_update",
    "causal_conv1d_update_ref",
]
