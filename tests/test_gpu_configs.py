"""The BASELINE.json configurations at their full sizes on the GPU.

Every output tensor is checked whole against an fp32 evaluation of the
pure-PyTorch reference (``causal_conv1d_ref`` with autograd, itself pinned
to the reference package's ``reference.py`` by the golden fixtures) run on
the GPU from the same bf16/fp16 inputs upcast to fp32 -- in batch chunks for
C5, whose tensors hold 2^32 elements -- with the parity tolerances of the
other tests (1e-2 for bf16/fp16 outputs; reductions against atol x max|ref|).
The comparisons run on the GPU: the C5 tensors are too large to move to the
host.  seq_idx (C4) is evaluated per packed sequence, as the reference's own
tests do (tests/_helpers.py:98-156).  On top of that, channel slices are
checked against the CPU oracle (rows (b, c) are independent, so a slice is
an exact sub-problem), states bit-exactly, and results for determinism.
Inputs follow BASELINE.json: x, states, grad ~ N(0,1), weight and bias ~
U(-0.5, 0.5)."""

from __future__ import annotations

import pytest
import torch

import oracle
from causal_conv1d_b200 import causal_conv1d_fn, causal_conv1d_ref, causal_conv1d_update, causal_conv1d_varlen_states
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


def _close_gpu(actual, expected, dt, what, atol=None):
    """|a - e| <= atol + rtol * |e| elementwise, evaluated on the device."""
    tol = dict(TOL[dt])
    if atol is not None:
        tol["atol"] = atol
    a = actual.detach().float()
    e = expected.detach().float()
    assert a.shape == e.shape, f"{what}: shape {tuple(a.shape)} vs {tuple(e.shape)}"
    diff = (a - e).abs()
    bad = ~(diff <= tol["atol"] + tol["rtol"] * e.abs())  # NaN counts as bad
    n = int(bad.sum())
    if n:
        d = torch.where(torch.isfinite(diff), diff, torch.full_like(diff, float("inf")))
        i = int(d.argmax())
        raise AssertionError(f"{what}: {n} of {a.numel()} elements out of tolerance {tol}; worst at flat index {i}: "
                             f"got {a.flatten()[i].item():.6g}, want {e.flatten()[i].item():.6g}")


def _ref_fp32(x, w, b, init, dout, dfinal, silu=True, seq=None):
    """fp32 reference forward + backward on the GPU (autograd through
    causal_conv1d_ref).  With seq_idx (batch 1, ids >= 0) each packed
    sequence is evaluated on its own and the weight gradients summed."""
    act = "silu" if silu else None
    xf = x.detach().float().requires_grad_()
    wf = w.detach().float().requires_grad_()
    bf = b.detach().float().requires_grad_() if b is not None else None
    if seq is None:
        inf = init.detach().float().requires_grad_() if init is not None else None
        r = causal_conv1d_ref(xf, wf, bf, initial_states=inf, return_final_states=init is not None, activation=act)
        out, fs = r if init is not None else (r, None)
        outs, grads = [out], [dout.float()]
        if fs is not None and dfinal is not None:
            outs.append(fs)
            grads.append(dfinal.float())
        torch.autograd.backward(outs, grads)
        return dict(out=out.detach(), dx=xf.grad, dw=wf.grad, db=bf.grad if bf is not None else None,
                    dinit=inf.grad if inf is not None else None)
    assert x.shape[0] == 1 and int(seq.min()) >= 0
    ids = seq[0]
    starts = [0] + (torch.nonzero(ids[1:] != ids[:-1]).flatten() + 1).tolist() + [ids.numel()]
    out = torch.empty_like(xf)
    for s0, s1 in zip(starts[:-1], starts[1:]):
        o = causal_conv1d_ref(xf[..., s0:s1], wf, bf, activation=act)
        o.backward(dout[..., s0:s1].float())
        out[..., s0:s1] = o.detach()
    return dict(out=out, dx=xf.grad, dw=wf.grad, db=bf.grad if bf is not None else None, dinit=None)


def _check_whole(res, ref, dt, b_sl=slice(None)):
    """Kernel results (rows b_sl of the batch) against the fp32 reference of
    those rows; the weight gradients are checked by the caller."""
    _close_gpu(res["out"][b_sl], ref["out"], dt, "out (whole tensor)")
    _close_gpu(res["dx"][b_sl], ref["dx"], dt, "dx (whole tensor)")
    if ref["dinit"] is not None:
        _close_gpu(res["dinit"][b_sl], ref["dinit"], dt, "dinitial_states (whole tensor)")


def _check_weight_grads(res, dw, db, dt):
    norm = max(dw.abs().max().item(), db.abs().max().item() if db is not None else 0.0)
    _close_gpu(res["dw"], dw, dt, "dweight (whole tensor)", atol=TOL[dt]["atol"] * max(1.0, norm))
    if db is not None:
        _close_gpu(res["db"], db, dt, "dbias (whole tensor)", atol=TOL[dt]["atol"] * max(1.0, norm))


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
    ref = _ref_fp32(x, w, b, init, dout, dfinal)
    _check_whole(res, ref, dt)
    _check_weight_grads(res, ref["dw"], ref["db"], dt)
    del ref
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
    ref = _ref_fp32(x, w, b, None, dout, None, seq=seq)
    _check_whole(res, ref, dt)
    _check_weight_grads(res, ref["dw"], ref["db"], dt)
    del ref
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
    # Whole tensors against the fp32 reference, 8 batch rows at a time (the
    # weight gradients sum over every chunk).
    dw = torch.zeros(D, W, device=DEV)
    db = torch.zeros(D, device=DEV)
    for b0 in range(0, B, 8):
        sl = slice(b0, min(B, b0 + 8))
        ref = _ref_fp32(x[sl], w, b, init[sl], dout[sl], None, silu=silu)
        _check_whole(res, ref, dt, sl)
        dw += ref["dw"]
        db += ref["db"]
        del ref
    _check_weight_grads(res, dw, db, dt)
    for c0, c1 in [(0, 6), (8190, 8192)]:
        _check_slice(x, w, b, init, dout, dfinal, res, c0, c1, silu=silu)
    assert_bitwise(res["fs"], x[..., -(W - 1):], "final_states (full)")
    del res
    torch.cuda.empty_cache()
