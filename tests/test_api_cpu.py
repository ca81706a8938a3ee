"""Host-side behaviour of the public API, on CPU tensors (no GPU needed):
argument validation with the reference's error types and messages (the
cases of the reference's tests/test_fwd.py:146-156,209-219,294-316,386-405,
461-474 and tests/test_update.py:246-251), the loud refusal of CPU tensors
(no CPU fallback), the compat shim, and the exported pure-PyTorch
references against the golden fixtures."""

from __future__ import annotations

import pytest
import torch

import causal_conv1d_b200 as cc
from conftest import DTYPES, assert_bitwise, assert_close, golden_cases


def test_public_names():
    for name in ["causal_conv1d_fn", "causal_conv1d_ref", "causal_conv1d_update", "causal_conv1d_update_ref",
                 "causal_conv1d_varlen_states", "causal_conv1d_varlen_states_ref"]:
        assert callable(getattr(cc, name))
    assert cc.__version__ == "1.6.1"


def test_signatures_match_reference():
    import inspect

    assert list(inspect.signature(cc.causal_conv1d_fn).parameters) == [
        "x", "weight", "bias", "seq_idx", "initial_states", "return_final_states", "final_states_out", "activation"]
    assert list(inspect.signature(cc.causal_conv1d_update).parameters) == [
        "x", "conv_state", "weight", "bias", "activation", "cache_seqlens", "conv_state_indices"]
    assert list(inspect.signature(cc.causal_conv1d_varlen_states).parameters) == ["x", "cu_seqlens", "state_len"]


def test_compat_shim():
    import causal_conv1d

    assert causal_conv1d.causal_conv1d_fn is cc.causal_conv1d_fn
    assert causal_conv1d.causal_conv1d_update is cc.causal_conv1d_update
    assert causal_conv1d.__version__ == cc.__version__
    from causal_conv1d.causal_conv1d_varlen import causal_conv1d_varlen_states

    assert causal_conv1d_varlen_states is cc.causal_conv1d_varlen_states


def test_width_invalid_raises():
    x = torch.randn(1, 8, 16, dtype=torch.float16)
    with pytest.raises(NotImplementedError, match="width must be in"):
        cc.causal_conv1d_fn(x, torch.randn(8, 10, dtype=torch.float16))


def test_fwd_width6_fp32_rejected():
    x = torch.randn(2, 64, 128)
    with pytest.raises(NotImplementedError, match="width must be in 2..5"):
        cc.causal_conv1d_fn(x, torch.randn(64, 6))


def test_fwd_width10_fp16_rejected():
    x = torch.randn(2, 64, 128, dtype=torch.float16)
    with pytest.raises(NotImplementedError, match="width must be in 2..9"):
        cc.causal_conv1d_fn(x, torch.randn(64, 10, dtype=torch.float16))


def test_activation_and_dtype_validation():
    x = torch.randn(1, 8, 16)
    w = torch.randn(8, 4)
    with pytest.raises(NotImplementedError, match="activation"):
        cc.causal_conv1d_fn(x, w, activation="relu")
    with pytest.raises(NotImplementedError, match="unsupported dtype"):
        cc.causal_conv1d_fn(x.double(), w.double())
    with pytest.raises(NotImplementedError, match="weight.dtype"):
        cc.causal_conv1d_fn(x, w.half())
    with pytest.raises(NotImplementedError, match="bias.dtype"):
        cc.causal_conv1d_fn(x, w, torch.randn(8, dtype=torch.float16))


def test_final_states_out_validation():
    x = torch.randn(1, 8, 16, dtype=torch.float16)
    w = torch.randn(8, 4, dtype=torch.float16)
    with pytest.raises(ValueError, match="return_final_states=True"):
        cc.causal_conv1d_fn(x, w, return_final_states=False, final_states_out=torch.empty(1, 8, 3, dtype=torch.float16))


def test_initial_states_mutual_exclusion_with_seq_idx():
    x = torch.randn(1, 8, 16, dtype=torch.float16)
    w = torch.randn(8, 4, dtype=torch.float16)
    with pytest.raises(ValueError, match="mutually exclusive"):
        cc.causal_conv1d_fn(x, w, seq_idx=torch.zeros(1, 16, dtype=torch.int32),
                            initial_states=torch.randn(1, 8, 3, dtype=torch.float16))


def test_seq_idx_mutual_exclusion_with_final_states():
    x = torch.randn(1, 8, 16, dtype=torch.float16)
    w = torch.randn(8, 4, dtype=torch.float16)
    with pytest.raises(ValueError, match="mutually exclusive"):
        cc.causal_conv1d_fn(x, w, seq_idx=torch.zeros(1, 16, dtype=torch.int32), return_final_states=True)


def test_seq_idx_dtype_and_shape_validation():
    x = torch.randn(1, 8, 16, dtype=torch.float16)
    w = torch.randn(8, 4, dtype=torch.float16)
    with pytest.raises(ValueError, match="seq_idx.dtype must be int32"):
        cc.causal_conv1d_fn(x, w, seq_idx=torch.zeros(1, 16, dtype=torch.int64))
    with pytest.raises(ValueError, match="seq_idx shape"):
        cc.causal_conv1d_fn(x, w, seq_idx=torch.zeros(1, 15, dtype=torch.int32))


def test_initial_states_shape_validation():
    x = torch.randn(2, 8, 16, dtype=torch.float16)
    w = torch.randn(8, 4, dtype=torch.float16)
    with pytest.raises(ValueError, match="initial_states shape"):
        cc.causal_conv1d_fn(x, w, initial_states=torch.randn(2, 8, 4, dtype=torch.float16))


def test_wide_width_autograd_requires_aligned_seqlen():
    x = torch.randn(1, 8, 100, dtype=torch.float16, requires_grad=True)
    w = torch.randn(8, 7, dtype=torch.float16)
    with pytest.raises(NotImplementedError, match="aligned to 1024"):
        cc.causal_conv1d_fn(x, w)


def test_update_state_too_small_raises():
    x = torch.randn(1, 8, 1, dtype=torch.float16)
    with pytest.raises(ValueError, match="must be >="):
        cc.causal_conv1d_update(x, torch.zeros(1, 8, 2, dtype=torch.float16), torch.randn(8, 4, dtype=torch.float16))


def test_update_validation():
    x = torch.randn(2, 8, dtype=torch.float16)
    w = torch.randn(8, 4, dtype=torch.float16)
    st = torch.zeros(2, 8, 3, dtype=torch.float16)
    with pytest.raises(NotImplementedError, match="width must be in 2..9"):
        cc.causal_conv1d_update(x, st, torch.randn(8, 10, dtype=torch.float16))
    with pytest.raises(ValueError, match="conv_state shape"):
        cc.causal_conv1d_update(x, torch.zeros(3, 8, 3, dtype=torch.float16), w)
    with pytest.raises(ValueError, match="cache_seqlens.dtype must be int32"):
        cc.causal_conv1d_update(x, st, w, cache_seqlens=torch.zeros(2, dtype=torch.int64))
    with pytest.raises(ValueError, match="conv_state_indices.dtype must be int32"):
        cc.causal_conv1d_update(x, st, w, conv_state_indices=torch.zeros(2, dtype=torch.int64))
    with pytest.raises(NotImplementedError, match="conv_state.dtype"):
        cc.causal_conv1d_update(x, st.float(), w)


def test_cpu_tensors_are_refused_loudly():
    """No CPU fallback: a valid call on CPU tensors raises instead of
    silently computing somewhere else."""
    x = torch.randn(1, 8, 16)
    w = torch.randn(8, 4)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        cc.causal_conv1d_fn(x, w)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        cc.causal_conv1d_update(torch.randn(1, 8), torch.zeros(1, 8, 3), w)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        cc.causal_conv1d_varlen_states(torch.randn(5, 8), torch.tensor([0, 5], dtype=torch.int32), 3)


# ---- the exported pure-PyTorch references match the reference's results ----

@pytest.mark.parametrize("case", [c for c in golden_cases("conv") if c["seq"] is None], ids=lambda c: c["name"])
def test_causal_conv1d_ref_matches_golden(golden, case):
    dt = DTYPES[case["dtype"]]
    inp = golden.inputs("conv", case)
    exp = golden.expected("conv", case)
    f64 = {k: (v.double() if v is not None and v.dtype != torch.int32 else v) for k, v in inp.items()}
    res = cc.causal_conv1d_ref(f64["x"], f64["weight"], f64.get("bias"), initial_states=f64.get("initial_states"),
                               return_final_states=case["final"], activation="silu" if case["silu"] else None)
    out, fs = res if case["final"] else (res, None)
    assert_close(out, exp["out"].double(), torch.float32, "out", rtol=1e-6, atol=1e-6)
    if case["final"]:
        assert_bitwise(fs.to(dt), exp["final_states"].to(dt), "final_states")


@pytest.mark.parametrize("case", [c for c in golden_cases("update") if c["idx"] is None], ids=lambda c: c["name"])
def test_causal_conv1d_update_ref_matches_golden(golden, case):
    dt = DTYPES[case["dtype"]]
    inp = golden.inputs("update", case)
    exp = golden.expected("update", case)
    st = inp["conv_state"].clone()
    out = cc.causal_conv1d_update_ref(inp["x"].double(), st.double().clone(), inp["weight"].double(),
                                      None if inp.get("bias") is None else inp["bias"].double(),
                                      activation="silu" if case["silu"] else None,
                                      cache_seqlens=inp.get("cache_seqlens"))
    assert_close(out, exp["out"].double(), torch.float32, "out", rtol=1e-6, atol=1e-6)
    st64 = st.double().clone()
    cc.causal_conv1d_update_ref(inp["x"].double(), st64, inp["weight"].double(), None,
                                cache_seqlens=inp.get("cache_seqlens"))
    assert_bitwise(st64.to(dt), exp["conv_state"].to(dt), "conv_state")


@pytest.mark.parametrize("case", golden_cases("varlen"), ids=lambda c: c["name"])
def test_varlen_states_ref_matches_golden(golden, case):
    dt = DTYPES[case["dtype"]]
    inp = golden.inputs("varlen", case)
    exp = golden.expected("varlen", case)
    st = cc.causal_conv1d_varlen_states_ref(inp["x"], inp["cu_seqlens"], case["S"])
    assert st.shape == exp["states"].shape
    assert st.stride(1) == 1  # (batch, state_len, dim) storage, like upstream
    assert_bitwise(st, exp["states"].to(dt), "states")
