"""GPU parity of causal_conv1d_update (decode step) and of
causal_conv1d_varlen_states.

Golden cases come from the reference's own reference.py (float64); the
conv_state contents after an update are pure data movement and must be
bit-exact, as must untouched pool slots and padding rows.  The decode-loop
tests are ports of the reference's tests/test_update.py:70-96 and :144-171."""

from __future__ import annotations

import pytest
import torch

import oracle
from _gpu_util import seeded
from causal_conv1d_b200 import (causal_conv1d_fn, causal_conv1d_update, causal_conv1d_varlen_states,
                                causal_conv1d_varlen_states_ref)
from conftest import DTYPES, assert_bitwise, assert_close, golden_cases

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("two_d", [False, True])
@pytest.mark.parametrize("case", golden_cases("update"), ids=lambda c: c["name"])
def test_golden(golden, case, two_d):
    dt = DTYPES[case["dtype"]]
    inp = golden.inputs("update", case)
    exp = golden.expected("update", case)
    if two_d and case["L"] != 1:
        pytest.skip("2-D x means seqlen 1")
    state = inp["conv_state"].to(DEV)
    x = inp["x"].to(DEV)
    if two_d:
        x = x[..., 0]
    out = causal_conv1d_update(
        x, state, inp["weight"].to(DEV), inp["bias"].to(DEV) if "bias" in inp else None,
        activation="silu" if case["silu"] else None,
        cache_seqlens=inp["cache_seqlens"].to(DEV) if "cache_seqlens" in inp else None,
        conv_state_indices=inp["conv_state_indices"].to(DEV) if "conv_state_indices" in inp else None)
    want = exp["out"][..., 0] if two_d else exp["out"]
    assert out.shape == x.shape
    assert_close(out.cpu(), want, dt, "out")
    assert_bitwise(state.cpu(), exp["conv_state"].to(dt), "conv_state")


@pytest.mark.parametrize("D", [300, 512])  # 512: the vectorised single-token path
@pytest.mark.parametrize("mode", ["linear", "circular", "pool", "pool_circular"])
@pytest.mark.parametrize("W", [2, 4, 7, 9])
@pytest.mark.parametrize("dtype", ["fp32", "bf16", "fp16"])
def test_vs_oracle(dtype, W, mode, D):
    dt = DTYPES[dtype]
    B, L = 9, 1 if W != 7 else 3
    S = W - 1 if mode in ("linear", "pool") else W + 6
    rows = B if mode in ("linear", "circular") else 2 * B + 1
    x = seeded((B, D, L), dt, W)
    w = seeded((D, W), dt, W + 1, "uniform")
    b = seeded((D,), dt, W + 2, "uniform")
    state = seeded((rows, D, S), dt, W + 3)
    idx = None
    if mode.startswith("pool"):
        perm = torch.randperm(rows, generator=torch.Generator().manual_seed(W))[:B].to(torch.int32)
        perm[3] = -1
        idx = perm
    cache = torch.randint(-5, 1024, (B,), generator=torch.Generator().manual_seed(W), dtype=torch.int32) \
        if "circular" in mode else None
    st_g = state.to(DEV)
    out = causal_conv1d_update(x.to(DEV), st_g, w.to(DEV), b.to(DEV), activation="silu",
                               cache_seqlens=cache.to(DEV) if cache is not None else None,
                               conv_state_indices=idx.to(DEV) if idx is not None else None)
    st_o = state.clone()
    o = oracle.update(x, st_o, w, b, silu=True, cache_seqlens=cache, conv_state_indices=idx)
    assert_close(out.cpu(), o, dt, "out")
    assert_bitwise(st_g.cpu(), st_o, "conv_state")
    if idx is not None:
        assert torch.all(out[3] == 0)


@pytest.mark.parametrize("dtype", ["fp32", "bf16", "fp16"])
def test_decode_loop_matches_full_forward(dtype):
    dt = DTYPES[dtype]
    B, D, L, W = 2, 16, 24, 4
    x = torch.randn(B, D, L, dtype=dt, device=DEV)
    w = torch.randn(D, W, dtype=dt, device=DEV)
    b = torch.randn(D, dtype=dt, device=DEV)
    full = causal_conv1d_fn(x, w, b, activation="silu")
    state = torch.zeros(B, D, W - 1, dtype=dt, device=DEV)
    dec = torch.cat([causal_conv1d_update(x[:, :, t:t + 1], state, w, b, activation="silu") for t in range(L)], -1)
    # Same fp32 tap order and SiLU in both kernels: bit-exact in every dtype.
    assert torch.equal(full, dec)


@pytest.mark.parametrize("chanlast", [False, True])  # conv_state (B, D, S) or stored (B, S, D)
@pytest.mark.parametrize("row_bytes", [0, 16, 32])  # 0: state_len W-1; 16/32: whole-row kernel
@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_circular_decode_loop(dtype, row_bytes, chanlast):
    dt = DTYPES[dtype]
    B, D, L, W = 1, 8, 16, 4
    S = W - 1 if row_bytes == 0 else row_bytes // torch.tensor([], dtype=dt).element_size()
    x = torch.randn(B, D, L, dtype=dt, device=DEV)
    w = torch.randn(D, W, dtype=dt, device=DEV)
    full = causal_conv1d_fn(x, w, activation="silu")
    if chanlast:
        state = torch.zeros(B, S, D, dtype=dt, device=DEV).transpose(1, 2)
    else:
        state = torch.zeros(B, D, S, dtype=dt, device=DEV)
    outs = []
    for t in range(L):
        cs = torch.tensor([t], dtype=torch.int32, device=DEV)
        outs.append(causal_conv1d_update(x[:, :, t:t + 1], state, w, activation="silu", cache_seqlens=cs))
    assert torch.equal(torch.cat(outs, -1), full)


def test_pool_untouched_slots_exact():
    dt = torch.bfloat16
    pool, B, D, W = 7, 3, 16, 4
    x = torch.randn(B, D, dtype=dt, device=DEV)
    w = torch.randn(D, W, dtype=dt, device=DEV)
    st = torch.randn(pool, D, W - 1, dtype=dt, device=DEV)
    before = st.clone()
    idx = torch.tensor([3, 0, 5], dtype=torch.int32, device=DEV)
    causal_conv1d_update(x, st, w, activation="silu", conv_state_indices=idx)
    untouched = torch.ones(pool, dtype=torch.bool)
    untouched[[3, 0, 5]] = False
    assert torch.equal(st.cpu()[untouched], before.cpu()[untouched])


def test_padding_index_zeroes_output_and_keeps_state():
    dt = torch.float16
    B, D, W = 3, 8, 4
    x = torch.randn(B, D, dtype=dt, device=DEV)
    w = torch.randn(D, W, dtype=dt, device=DEV)
    st = torch.randn(4, D, W - 1, dtype=dt, device=DEV)
    before = st.clone()
    out = causal_conv1d_update(x, st, w, conv_state_indices=torch.tensor([0, -1, 2], dtype=torch.int32, device=DEV))
    assert torch.all(out[1] == 0)
    changed = (before != st).any(dim=(1, 2)).cpu()
    assert changed[0] and changed[2] and not changed[1] and not changed[3]


# ---- varlen states --------------------------------------------------------

@pytest.mark.parametrize("case", golden_cases("varlen"), ids=lambda c: c["name"])
def test_varlen_golden(golden, case):
    dt = DTYPES[case["dtype"]]
    inp = golden.inputs("varlen", case)
    exp = golden.expected("varlen", case)
    st = causal_conv1d_varlen_states(inp["x"].to(DEV), inp["cu_seqlens"].to(DEV), case["S"])
    assert st.shape == exp["states"].shape and st.stride(1) == 1
    assert_bitwise(st.cpu(), exp["states"].to(dt), "states")


@pytest.mark.parametrize("dtype", ["fp32", "bf16", "fp16"])
def test_varlen_random_vs_ref(dtype):
    dt = DTYPES[dtype]
    g = torch.Generator().manual_seed(3)
    lens = torch.randint(0, 300, (33,), generator=g)
    cu = torch.cat([torch.zeros(1, dtype=torch.long), lens.cumsum(0)]).to(torch.int32)
    x = torch.randn(int(cu[-1]), 200, generator=g).to(dt)
    for S in (1, 3, 8, 500):
        got = causal_conv1d_varlen_states(x.to(DEV), cu.to(DEV), S).cpu()
        assert_bitwise(got, causal_conv1d_varlen_states_ref(x, cu, S), f"S={S}")
        assert_bitwise(got, oracle.varlen_states(x, cu, S), f"S={S} (oracle)")


@pytest.mark.parametrize("D", [1024, 1000])
@pytest.mark.parametrize("row_bytes", [16, 32])
@pytest.mark.parametrize("pool", [False, True])
@pytest.mark.parametrize("dtype,W", [("bf16", 2), ("bf16", 4), ("bf16", 9), ("fp16", 5), ("fp32", 2), ("fp32", 5)])
def test_circular_serving_state_len_vs_oracle(dtype, W, pool, row_bytes, D):
    """Circular decode with the serving state lengths (rows of 16 or 32 bytes:
    8 / 16 elements for 16-bit types, 4 / 8 for fp32) -- the whole-row kernel
    -- over the full write-head range incl. negative and wrapped values; a
    ragged dim; pool rows at a channel pitch of twice the row (a dim slice)."""
    dt = DTYPES[dtype]
    S = row_bytes // torch.tensor([], dtype=dt).element_size()
    if W - 1 > S:
        pytest.skip("state shorter than the window")
    B = 7
    rows = 2 * B if pool else B
    x = seeded((B, D), dt, W)
    w = seeded((D, W), dt, W + 1, "uniform")
    b = seeded((D,), dt, W + 2, "uniform")
    state = seeded((rows, D, S), dt, W + 3)
    if pool:
        big = torch.zeros(rows, 2 * D, S, dtype=dt)
        big[:, ::2] = state
        state = big[:, ::2]
    cache = torch.tensor([0, 1, S - 1, S, 1023, -1, -S - 3], dtype=torch.int32)
    idx = None
    if pool:
        idx = torch.randperm(rows, generator=torch.Generator().manual_seed(W))[:B].to(torch.int32)
        idx[2] = -1
    if pool:
        big_g = big.to(DEV)
        st_g = big_g[:, ::2]
    else:
        st_g = state.to(DEV)
    out = causal_conv1d_update(x.to(DEV), st_g, w.to(DEV), b.to(DEV), activation="silu", cache_seqlens=cache.to(DEV),
                               conv_state_indices=idx.to(DEV) if idx is not None else None)
    st_o = state.clone()
    o = oracle.update(x, st_o, w, b, silu=True, cache_seqlens=cache, conv_state_indices=idx)
    assert_close(out.cpu(), o, dt, "out")
    assert_bitwise(st_g.cpu(), st_o, "conv_state")
    if pool:
        assert torch.count_nonzero(big_g[:, 1::2]) == 0  # the interleaved rows are never written


@pytest.mark.parametrize("pool", [False, True])
@pytest.mark.parametrize("L,S,state_layout", [
    (4, 3, "packed"), (4, 3, "chanlast"), (1, 3, "chanlast"), (8, 16, "packed"), (5, 12, "chanlast"),
    (2, 9, "packed"),       # burst shorter than the state: old values shift left
    (12, 20, "packed"),     # past the burst kernel's limits: generic kernel
])
@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_linear_burst_and_state_layouts_vs_oracle(dtype, L, S, state_layout, pool):
    """Linear-mode decode bursts (speculative decoding) and conv_state pools
    stored channel-last (strides (S*D, 1, D)): outputs within tolerance,
    state rows bit-exact, untouched and padding rows unchanged."""
    dt = DTYPES[dtype]
    B, D, W = 6, 328, 4
    rows = 2 * B if pool else B
    x = seeded((B, D, L), dt, 21)
    w = seeded((D, W), dt, 22, "uniform")
    b = seeded((D,), dt, 23, "uniform")
    state = seeded((rows, D, S), dt, 24)
    idx = None
    if pool:
        idx = torch.randperm(rows, generator=torch.Generator().manual_seed(5))[:B].to(torch.int32)
        idx[1] = -1
    if state_layout == "chanlast":
        st_g = state.transpose(1, 2).contiguous().transpose(1, 2).to(DEV)
        assert st_g.stride(1) == 1
    else:
        st_g = state.to(DEV)
    out = causal_conv1d_update(x.to(DEV), st_g, w.to(DEV), b.to(DEV), activation="silu",
                               conv_state_indices=idx.to(DEV) if idx is not None else None)
    st_o = state.clone()
    o = oracle.update(x, st_o, w, b, silu=True, cache_seqlens=None, conv_state_indices=idx)
    assert_close(out.cpu(), o, dt, "out")
    assert_bitwise(st_g.cpu(), st_o, "conv_state")
    if idx is not None:
        assert torch.all(out[1] == 0)


@pytest.mark.parametrize("pool", [False, True])
@pytest.mark.parametrize("D", [1000, 1002])  # 1002: not a multiple of 4 channels -> generic circular kernel
@pytest.mark.parametrize("dtype,W,S", [("bf16", 4, 3), ("bf16", 4, 8), ("bf16", 2, 1), ("fp16", 3, 13),
                                       ("fp32", 4, 5), ("fp32", 2, 8)])
def test_circular_chanlast_states_vs_oracle(dtype, W, S, D, pool):
    """Circular decode with conv_state stored channel-last (strides (S*D, 1, D)
    for each row; vLLM-style pools): the write head over its full range incl.
    negative and wrapped values, any state_len >= W-1, pool rows addressed by
    index with one padding entry.  Outputs within tolerance, state rows
    bit-exact, padding and unused rows untouched."""
    dt = DTYPES[dtype]
    B = 7
    rows = 2 * B if pool else B
    x = seeded((B, D), dt, 31 + W)
    w = seeded((D, W), dt, 32 + W, "uniform")
    b = seeded((D,), dt, 33 + W, "uniform")
    state = seeded((rows, D, S), dt, 34 + S)
    cache = torch.tensor([0, 1, S - 1, S, 1023, -1, -S - 3], dtype=torch.int32)
    idx = None
    if pool:
        idx = torch.randperm(rows, generator=torch.Generator().manual_seed(S))[:B].to(torch.int32)
        idx[3] = -1
    st_g = state.transpose(1, 2).contiguous().transpose(1, 2).to(DEV)
    assert st_g.stride(1) == 1
    out = causal_conv1d_update(x.to(DEV), st_g, w.to(DEV), b.to(DEV), activation="silu", cache_seqlens=cache.to(DEV),
                               conv_state_indices=idx.to(DEV) if idx is not None else None)
    st_o = state.clone()
    o = oracle.update(x, st_o, w, b, silu=True, cache_seqlens=cache, conv_state_indices=idx)
    assert_close(out.cpu(), o, dt, "out")
    assert_bitwise(st_g.cpu(), st_o, "conv_state")
    if idx is not None:
        assert torch.all(out[3] == 0)
