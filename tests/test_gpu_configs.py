"""The BASELINE.json configurations at their full sizes on the GPU.

Rows (b, c) of the conv are independent, so a channel slice of the full
problem is an exact sub-problem: the oracle checks slices (including the
dweight/dbias of the sliced channels, which sum over every batch row),
while size-independent properties (bit-exact states, determinism) cover the
whole tensors.  Inputs follow BASELINE.json: x, states, grad ~ N(0,1),
weight and bias ~ U(-0.5, 0.5)."""

from __future__ import annotations

import pytest
import torch

import oracle
from causal_conv1d_b200 import causal_conv1d_fn, causal_conv1d_update, causal_conv1d_varlen_states
from conftest import TOL, assert_bitwise, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _gen(shape, dt, g, kind="normal"):
    if kind == "normal":
        return torch.randn(*shape, generator=g, device=DEV, dtype=torch.float32).to(dt)
    return (torch.rand(*shape, generator=g, device=DEV, dtype=torch.float32) - 0.5).to(dt)


def _red_close(a, e, dt, what):
    norm = e.float().abs().max().item()
    assert_close(a, e, dt, what, atol=TOL[dt]["atol"] * max(1.0, norm))


def _check_slice(x, w, b, init, dout, dfinal, res, c0, c1, silu=True, seq=None):
    dt = x.dtype
    xs = x[:, c0:c1].cpu()
    ws, bs = w[c0:c1].cpu(), (b[c0:c1].cpu() if b is not None else None)
    ins = init[:, c0:c1].cpu() if init is not None else None
    ds = dout[:, c0:c1].cpu()
    dfs = dfinal[:, c0:c1].cpu() if dfinal is not None else None
    sq = seq.cpu() if seq is not None else None
    o, fs = oracle.fwd(xs, ws, bs, sq, ins, silu=silu, return_final_states=init is not None)
    g = oracle.bwd(xs, ws, ds, bs, sq, ins, dfs, silu=silu)
    assert_close(res["out"][:, c0:c1].cpu(), o, dt, "out")
    if fs is not None:
        assert_bitwise(res["fs"][:, c0:c1].cpu(), fs, "final_states")
    assert_close(res["dx"][:, c0:c1].cpu(), g["dx"], dt, "dx")
    _red_close(res["dw"][c0:c1].float().cpu(), g["dweight"], dt, "dweight")
    if b is not None:
        _red_close(res["db"][c0:c1].float().cpu(), g["dbias"], dt, "dbias")
    if init is not None:
        assert_close(res["dinit"][:, c0:c1].cpu(), g["dinit"], dt, "dinit")


def _fwd_bwd(x, w, b, init, dout, dfinal, silu=True, seq=None):
    xg = x.detach().requires_grad_()
    wg = w.detach().requires_grad_()
    bg = b.detach().requires_grad_() if b is not None else None
    ig = init.detach().requires_grad_() if init is not None else None
    r = causal_conv1d_fn(xg, wg, bg, seq_idx=seq, initial_states=ig, return_final_states=init is not None,
                         activation="silu" if silu else None)
    out, fs = r if init is not None else (r, None)
    outs, grads = [out], [dout]
    if fs is not None and dfinal is not None:
        outs.append(fs)
        grads.append(dfinal)
    torch.autograd.backward(outs, grads)
    return dict(out=out.detach(), fs=fs.detach() if fs is not None else None, dx=xg.grad, dw=wg.grad,
                db=bg.grad if bg is not None else None, dinit=ig.grad if ig is not None else None)


def test_c2_mamba2_prefill_channel_last():
    dt = torch.bfloat16
    B, D, L, W = 8, 5376, 2048, 4
    g = torch.Generator(device=DEV).manual_seed(0)
    x = _gen((B, L, D), dt, g).transpose(1, 2)  # channel-last: stride over dim = 1
    w = _gen((D, W), dt, g, "uniform")
    b = _gen((D,), dt, g, "uniform")
    init = _gen((B, D, W - 1), dt, g)
    dout = _gen((B, L, D), dt, g).transpose(1, 2)
    dfinal = _gen((B, D, W - 1), dt, g)
    assert x.stride(1) == 1
    res = _fwd_bwd(x, w, b, init, dout, dfinal)
    assert res["dx"].stride(1) == 1  # dx keeps x's layout
    for c0, c1 in [(0, 160), (2600, 2700), (5248, 5376)]:
        _check_slice(x, w, b, init, dout, dfinal, res, c0, c1)
    # final_states is an exact copy of the last W-1 columns.
    assert_bitwise(res["fs"], x[..., -(W - 1):], "final_states (full)")
    res2 = _fwd_bwd(x, w, b, init, dout, dfinal)
    for k in ("out", "dx", "dw", "db", "dinit"):
        assert torch.equal(res[k], res2[k]), k


@pytest.mark.parametrize("variant", ["indexed_pool", "circular"])
def test_c3_decode_update(variant):
    dt = torch.bfloat16
    B, D, W = 256, 5376, 4
    g = torch.Generator(device=DEV).manual_seed(0)
    x = _gen((B, D), dt, g)
    w = _gen((D, W), dt, g, "uniform")
    b = _gen((D,), dt, g, "uniform")
    if variant == "indexed_pool":
        state = _gen((512, D, W - 1), dt, g)
        idx = torch.randperm(512, generator=torch.Generator().manual_seed(0))[:B].to(torch.int32).to(DEV)
        cache = None
    else:
        state = _gen((B, D, 8), dt, g)
        idx = None
        cache = torch.randint(0, 1024, (B,), generator=torch.Generator().manual_seed(0), dtype=torch.int32).to(DEV)
    st_cpu = state.cpu()
    out = causal_conv1d_update(x, state, w, b, activation="silu", cache_seqlens=cache, conv_state_indices=idx)
    o = oracle.update(x.cpu(), st_cpu, w.cpu(), b.cpu(), silu=True,
                      cache_seqlens=cache.cpu() if cache is not None else None,
                      conv_state_indices=idx.cpu() if idx is not None else None)
    assert_close(out.cpu(), o, dt, "out")
    assert_bitwise(state.cpu(), st_cpu, "conv_state")


def _varlen_lengths(n=32, total=65536, seed=0):
    g = torch.Generator().manual_seed(seed)
    raw = torch.randint(256, 4097, (n,), generator=g)
    lens = (raw * total // raw.sum()).clamp(min=1)
    lens[-1] += total - lens.sum()
    return lens


def test_c4_varlen_packed_prefill():
    dt = torch.float16
    B, D, L, W = 1, 4096, 65536, 4
    lens = _varlen_lengths()
    assert int(lens.sum()) == L
    seq = torch.repeat_interleave(torch.arange(32, dtype=torch.int32), lens).view(1, L).to(DEV)
    g = torch.Generator(device=DEV).manual_seed(0)
    x = _gen((B, L, D), dt, g).transpose(1, 2)
    w = _gen((D, W), dt, g, "uniform")
    b = _gen((D,), dt, g, "uniform")
    dout = _gen((B, L, D), dt, g).transpose(1, 2)
    res = _fwd_bwd(x, w, b, None, dout, None, seq=seq)
    for c0, c1 in [(0, 64), (4032, 4096)]:
        _check_slice(x, w, b, None, dout, None, res, c0, c1, seq=seq)
    # Prefill -> decode hand-off: per-sequence conv states of the packed batch.
    cu = torch.cat([torch.zeros(1, dtype=torch.long), lens.cumsum(0)]).to(torch.int32)
    tokens = x[0].transpose(0, 1)  # (total_tokens, dim), unit stride over dim
    st = causal_conv1d_varlen_states(tokens, cu.to(DEV), W - 1)
    assert_bitwise(st[:, :64].cpu(), oracle.varlen_states(tokens[:, :64].cpu(), cu, W - 1), "varlen states")


@pytest.mark.parametrize("W,silu,B", [(4, True, 64), (3, False, 8), (2, True, 8)])
def test_c5_large_contiguous(W, silu, B):
    dt = torch.bfloat16
    D, L = 8192, 8192
    g = torch.Generator(device=DEV).manual_seed(W)
    x = _gen((B, D, L), dt, g)
    w = _gen((D, W), dt, g, "uniform")
    b = _gen((D,), dt, g, "uniform")
    init = _gen((B, D, W - 1), dt, g)
    dout = _gen((B, D, L), dt, g)
    dfinal = None
    res = _fwd_bwd(x, w, b, init, dout, dfinal, silu=silu)
    for c0, c1 in [(0, 6), (8190, 8192)]:
        _check_slice(x, w, b, init, dout, dfinal, res, c0, c1, silu=silu)
    assert_bitwise(res["fs"], x[..., -(W - 1):], "final_states (full)")
    del res
    torch.cuda.empty_cache()
