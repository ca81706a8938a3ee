"""Pins the CPU oracle to the reference: every golden fixture (computed by
the reference's own reference.py in float64, tests/golden/make_golden.py)
must be reproduced by the oracle's double-accumulating mode, and within the
parity tolerance by its float-accumulating port mode.  CPU only."""

from __future__ import annotations

import pytest
import torch

import oracle
from conftest import DTYPES, assert_bitwise, assert_close, golden_cases

# Oracle (float64 accumulate, rounded once to the dtype) vs the reference's
# float64 result rounded to float32: equal up to one rounding of the dtype.
PIN = {
    torch.float32: dict(rtol=2e-6, atol=1e-6),
    torch.bfloat16: dict(rtol=2 ** -7, atol=1e-6),
    torch.float16: dict(rtol=2 ** -10, atol=1e-6),
}


def _pin(actual, expected, dt, what, scale_atol=1.0):
    tol = PIN[dt]
    assert_close(actual, expected.to(dt), dt, what, rtol=tol["rtol"], atol=tol["atol"] * scale_atol)


@pytest.fixture(scope="module", autouse=True)
def _built():
    oracle.build()


@pytest.mark.parametrize("case", golden_cases("conv"), ids=lambda c: c["name"])
@pytest.mark.parametrize("acc64", [True, False], ids=["acc64", "acc32"])
def test_conv_fwd_bwd(golden, case, acc64):
    dt = DTYPES[case["dtype"]]
    inp = golden.inputs("conv", case)
    exp = golden.expected("conv", case)
    out, fs = oracle.fwd(inp["x"], inp["weight"], inp.get("bias"), inp.get("seq_idx"), inp.get("initial_states"),
                         silu=case["silu"], return_final_states=case["final"], acc64=acc64)
    if acc64:
        _pin(out, exp["out"], dt, "out")
    else:
        assert_close(out, exp["out"], dt, "out (acc32)")
    if case["final"]:
        assert_bitwise(fs, exp["final_states"].to(dt), "final_states")
    if not case["bwd"]:
        return
    g = oracle.bwd(inp["x"], inp["weight"], inp["dout"], inp.get("bias"), inp.get("seq_idx"),
                   inp.get("initial_states"), inp.get("dfinal"), silu=case["silu"], acc64=acc64)
    # dweight/dbias are sums over B*L terms: compare relative to their norm.
    wnorm = exp["dweight"].abs().max().item() + 1.0
    if acc64:
        _pin(g["dx"], exp["dx"], dt, "dx")
        assert_close(g["dweight"], exp["dweight"], torch.float32, "dweight", rtol=1e-6, atol=1e-6 * wnorm)
        if case["bias"]:
            bnorm = exp["dbias"].abs().max().item() + 1.0
            assert_close(g["dbias"], exp["dbias"], torch.float32, "dbias", rtol=1e-6, atol=1e-6 * bnorm)
        if case["init"]:
            _pin(g["dinit"], exp["dinit"], dt, "dinit")
    else:
        assert_close(g["dx"], exp["dx"], dt, "dx (acc32)")
        assert_close(g["dweight"], exp["dweight"], torch.float32, "dweight (acc32)", rtol=1e-4, atol=1e-5 * wnorm)
        if case["init"]:
            assert_close(g["dinit"], exp["dinit"], dt, "dinit (acc32)")


@pytest.mark.parametrize("case", golden_cases("update"), ids=lambda c: c["name"])
def test_update(golden, case):
    dt = DTYPES[case["dtype"]]
    inp = golden.inputs("update", case)
    exp = golden.expected("update", case)
    state = inp["conv_state"].clone()
    out = oracle.update(inp["x"], state, inp["weight"], inp.get("bias"), silu=case["silu"],
                        cache_seqlens=inp.get("cache_seqlens"), conv_state_indices=inp.get("conv_state_indices"))
    _pin(out, exp["out"], dt, "out")
    # The state update is pure data movement: bit-exact.
    assert_bitwise(state, exp["conv_state"].to(dt), "conv_state")


@pytest.mark.parametrize("case", golden_cases("varlen"), ids=lambda c: c["name"])
def test_varlen(golden, case):
    dt = DTYPES[case["dtype"]]
    inp = golden.inputs("varlen", case)
    exp = golden.expected("varlen", case)
    st = oracle.varlen_states(inp["x"], inp["cu_seqlens"], case["S"])
    assert_bitwise(st, exp["states"].to(dt), "states")
