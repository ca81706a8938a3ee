"""The in_proj GEMM with the causal conv as its epilogue (cc1d_inproj_conv_fwd,
``causal_conv1d_b200.fused.in_proj_causal_conv1d``) against the exact
computation it stands for, and against the unfused pipeline it replaces
(torch GEMM, xBC stored in bf16, then causal_conv1d_fn).

Reference and tolerance.  The reference evaluates xBC = hidden @ in_weight.T
and the conv in float64 from the same bf16 inputs.  The kernel sums the K
products in fp32 (in its own order: error at most K * 2^-24 * sum_k |a_k b_k|,
the standard bound for recursive summation) and rounds xBC to bf16 (at most
2^-8 relative), so each xBC element is within
    dy = K * 2^-24 * (|hidden| @ |in_weight|.T) + 2^-8 * |xBC|
of the exact value -- the bound final_states are checked against.  Through
the conv (and SiLU, 1.1-Lipschitz) an output moves by at most
1.1 * sum_j |w_j| * dy_j, plus its own bf16 rounding (2^-8 relative) and
1e-5 for the fp32 conv arithmetic.  Every output element is checked against
that bound, and against the library's bf16 tolerance (rtol = atol = 1e-2).
Inputs: hidden ~ N(0, 1), in_weight ~ N(0, 1/K) (xBC ~ N(0, 1)), conv
weight and bias ~ U(-0.5, 0.5), states ~ N(0, 1).
"""

from __future__ import annotations

import pytest
import torch

from causal_conv1d_b200 import causal_conv1d_fn, causal_conv1d_ref
from causal_conv1d_b200.fused import in_proj_causal_conv1d

pytestmark = pytest.mark.gpu
DEV = "cuda"
DT = torch.bfloat16


def _inputs(B, L, K, N, W, seed, bias=True, init=True):
    g = torch.Generator(device=DEV).manual_seed(seed)
    hidden = torch.randn(B, L, K, generator=g, device=DEV).to(DT)
    win = (torch.randn(N, K, generator=g, device=DEV) / K ** 0.5).to(DT)
    cw = (torch.rand(N, W, generator=g, device=DEV) - 0.5).to(DT)
    cb = (torch.rand(N, generator=g, device=DEV) - 0.5).to(DT) if bias else None
    st = torch.randn(B, N, W - 1, generator=g, device=DEV).to(DT) if init else None
    return hidden, win, cw, cb, st


def _reference(hidden, win, cw, cb, st, silu):
    """Exact xBC and out (float64), the per-element bound dy of the kernel's
    bf16 xBC, and the per-element bound of its outputs."""
    K = hidden.shape[-1]
    W = cw.shape[1]
    y = hidden.double() @ win.double().t()  # (B, L, N)
    dy = K * 2.0 ** -24 * (hidden.float().abs() @ win.float().abs().t()).double() + 2.0 ** -8 * y.abs()
    x = y.transpose(1, 2)
    act = "silu" if silu else None
    out = causal_conv1d_ref(x, cw.double(), cb.double() if cb is not None else None,
                            initial_states=st.double() if st is not None else None, activation=act)
    d = dy.transpose(1, 2)
    d = torch.nn.functional.pad(d, (W - 1, 0))  # states are exact inputs: no error before position 0
    taps = sum(cw.double().abs()[None, :, j, None] * d[..., j:j + x.shape[-1]] for j in range(W))
    bound = 1.1 * taps + 2.0 ** -8 * out.abs() + 1e-5
    return y, dy, out, bound


def _check(got_out, got_fs, y, dy, ref_out, bound, W):
    got = got_out.double()
    assert torch.isfinite(got).all()
    diff = (got - ref_out).abs()
    over = diff > bound
    assert int(over.sum()) == 0, (f"{int(over.sum())} outputs beyond the error bound; worst excess "
                                 f"{(diff - bound).max().item():.3e}")
    torch.testing.assert_close(got_out.float(), ref_out.float(), rtol=1e-2, atol=1e-2)
    if got_fs is not None:
        want = y[:, -(W - 1):, :].transpose(1, 2)
        tol = dy[:, -(W - 1):, :].transpose(1, 2)
        bad = (got_fs.double() - want).abs() > tol
        assert int(bad.sum()) == 0, f"final_states: {int(bad.sum())} elements beyond the xBC error bound"


@pytest.mark.parametrize("B,L,K,N,W,bias,init,silu", [
    (2, 300, 512, 288, 3, False, False, True),   # N not a multiple of the 256-channel tile
    (3, 133, 200, 64, 2, True, True, False),     # K not a multiple of 64; one partial channel tile
    (1, 3, 64, 32, 4, True, True, True),         # seqlen = width - 1: every output reads initial states
    (4, 250, 256, 512, 4, True, True, True),     # sequence starts inside tiles (125 output rows per tile)
])
def test_fused_matches_gemm_then_conv(B, L, K, N, W, bias, init, silu):
    hidden, win, cw, cb, st = _inputs(B, L, K, N, W, seed=B * 1000 + L, bias=bias, init=init)
    out, fs = in_proj_causal_conv1d(hidden, win, cw, cb, initial_states=st, return_final_states=True,
                                    activation="silu" if silu else None)
    torch.cuda.synchronize()
    assert out.shape == (B, N, L) and out.stride(1) == 1  # channel-last, like causal_conv1d_fn's output
    y, dy, ref, bound = _reference(hidden, win, cw, cb, st, silu)
    _check(out, fs, y, dy, ref, bound, W)


def test_fused_c2_mamba2_shape_and_repeat():
    """The Mamba-2 2.7B prefill shape: in_proj's xBC part
    (16384 x 2560) @ (2560 x 5376), then the W = 4 conv with bias, SiLU and
    initial / final states; every element checked.  A second call on the same
    inputs gives bitwise the same result."""
    B, L, K, N, W = 8, 2048, 2560, 5376, 4
    hidden, win, cw, cb, st = _inputs(B, L, K, N, W, seed=2)
    out, fs = in_proj_causal_conv1d(hidden, win, cw, cb, initial_states=st, return_final_states=True,
                                    activation="silu")
    torch.cuda.synchronize()
    y, dy, ref, bound = _reference(hidden, win, cw, cb, st, True)
    _check(out, fs, y, dy, ref, bound, W)
    out2, fs2 = in_proj_causal_conv1d(hidden, win, cw, cb, initial_states=st, return_final_states=True,
                                      activation="silu")
    assert torch.equal(out, out2) and torch.equal(fs, fs2)
    # The unfused pipeline of this library (torch GEMM, then causal_conv1d_fn)
    # agrees within the same bound.
    y2 = torch.nn.functional.linear(hidden, win)
    out3 = causal_conv1d_fn(y2.transpose(1, 2), cw, cb, initial_states=st, activation="silu")
    _check(out3, None, y, dy, ref, bound, W)


def test_fused_rejects_unsupported_inputs():
    hidden, win, cw, cb, st = _inputs(1, 2, 64, 32, 4, seed=1)
    with pytest.raises(RuntimeError, match="seqlen must be >= width-1"):
        in_proj_causal_conv1d(hidden, win, cw, cb)
    h16 = torch.randn(1, 8, 64, device=DEV, dtype=torch.float16)
    with pytest.raises(NotImplementedError, match="bfloat16"):
        in_proj_causal_conv1d(h16, win, cw)
    hidden, win, cw, cb, st = _inputs(1, 8, 64, 40, 4, seed=1)
    with pytest.raises(RuntimeError, match="multiple of 32"):
        in_proj_causal_conv1d(hidden, win, cw)
