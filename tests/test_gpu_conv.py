"""GPU parity of causal_conv1d_fn (forward + autograd backward) on sm_100a.

* Every golden case (the reference's own reference.py evaluated in float64,
  tests/golden/make_golden.py) in four memory layouts.
* Seeded sweeps over shapes, dtypes, widths, layouts, bias/SiLU, states and
  seq_idx against the CPU oracle (oracle/), which the golden cases pin.
* Bit-exact properties: final_states, the chunked-prefill round trip and
  run-to-run determinism of the backward (no atomics).
Tolerances: north-star bar, elementwise rtol=atol=1e-5 (fp32) and 1e-2
(bf16/fp16); the reductions dweight/dbias use atol scaled by ||ref||_inf, as
the reference's own tests do (tests/_helpers.py:35-43)."""

from __future__ import annotations

import pytest
import torch

import oracle
from _gpu_util import LAYOUTS, random_seq_idx, seeded, with_layout
from causal_conv1d_b200 import _ops, causal_conv1d_fn, causal_conv1d_ref
from conftest import DTYPES, TOL, assert_bitwise, assert_close, golden_cases

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _reduction_close(actual, expected, dt, what):
    norm = expected.detach().float().abs().max().item()
    tol = TOL[dt]
    assert_close(actual, expected, dt, what, rtol=tol["rtol"], atol=tol["atol"] * max(1.0, norm))


def run_gpu(x, weight, bias, seq_idx, init, dout, dfinal, silu, want_final, layout):
    """Forward + backward on the GPU; returns CPU tensors."""
    dt = x.dtype
    W = weight.shape[1]
    L = x.shape[-1]
    xg = with_layout(x.to(DEV), layout)
    wg = weight.to(DEV)
    bg = bias.to(DEV) if bias is not None else None
    sg = seq_idx.to(DEV) if seq_idx is not None else None
    ig = init.to(DEV) if init is not None else None
    act = "silu" if silu else None
    use_autograd = not (W > 5 and L % 1024 != 0)  # API restriction kept from the reference
    res = {}
    if use_autograd:
        xg.requires_grad_(True)
        wg.requires_grad_(True)
        if bg is not None:
            bg.requires_grad_(True)
        if ig is not None:
            ig.requires_grad_(True)
        r = causal_conv1d_fn(xg, wg, bg, seq_idx=sg, initial_states=ig, return_final_states=want_final,
                             activation=act)
        out, fs = r if want_final else (r, None)
        outs, grads = [out], [with_layout(dout.to(DEV), layout)]
        if want_final and dfinal is not None:
            outs.append(fs)
            grads.append(dfinal.to(DEV))
        torch.autograd.backward(outs, grads)
        res.update(out=out, fs=fs, dx=xg.grad, dw=wg.grad, db=bg.grad if bg is not None else None,
                   dinit=ig.grad if ig is not None else None)
    else:
        out = torch.empty_like(xg)
        fs = torch.empty(x.shape[0], x.shape[1], W - 1, dtype=dt, device=DEV) if want_final else None
        _ops.fwd(xg, wg, bg, sg, ig, out, silu, fs)
        D = x.shape[1]
        dx = torch.empty_like(xg)
        dwdb = torch.empty(D * (W + 1), dtype=torch.float32, device=DEV)
        dw = torch.empty(D, W, dtype=dt, device=DEV)
        db = torch.empty(D, dtype=dt, device=DEV) if bg is not None else None
        dinit = torch.empty_like(ig) if ig is not None else None
        dfg = dfinal.to(DEV) if (want_final and dfinal is not None) else None
        _ops.bwd(xg, wg, bg, with_layout(dout.to(DEV), layout), sg, ig, dfg, dx, dwdb, dinit, dw, db, silu)
        res.update(out=out, fs=fs, dx=dx, dw=dw, db=db, dinit=dinit)
    torch.cuda.synchronize()
    return {k: (v.detach().cpu() if v is not None else None) for k, v in res.items()}


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("case", golden_cases("conv"), ids=lambda c: c["name"])
def test_golden(golden, case, layout):
    dt = DTYPES[case["dtype"]]
    inp = golden.inputs("conv", case)
    exp = golden.expected("conv", case)
    r = run_gpu(inp["x"], inp["weight"], inp.get("bias"), inp.get("seq_idx"), inp.get("initial_states"),
                inp["dout"], inp.get("dfinal"), case["silu"], case["final"], layout)
    assert_close(r["out"], exp["out"], dt, "out")
    if case["final"]:
        assert_bitwise(r["fs"], exp["final_states"].to(dt), "final_states")
    assert_close(r["dx"], exp["dx"], dt, "dx")
    _reduction_close(r["dw"], exp["dweight"], dt, "dweight")
    if case["bias"]:
        _reduction_close(r["db"], exp["dbias"], dt, "dbias")
    if case["init"]:
        assert_close(r["dinit"], exp["dinit"], dt, "dinit")


def _compare_oracle(x, w, b, seq, init, dout, dfinal, silu, want_final, layout):
    dt = x.dtype
    r = run_gpu(x, w, b, seq, init, dout, dfinal, silu, want_final, layout)
    o_out, o_fs = oracle.fwd(x, w, b, seq, init, silu=silu, return_final_states=want_final)
    g = oracle.bwd(x, w, dout, b, seq, init, dfinal if want_final else None, silu=silu)
    assert_close(r["out"], o_out, dt, "out")
    if want_final:
        assert_bitwise(r["fs"], o_fs, "final_states")
    assert_close(r["dx"], g["dx"], dt, "dx")
    _reduction_close(r["dw"].float(), g["dweight"], dt, "dweight")
    if b is not None:
        _reduction_close(r["db"].float(), g["dbias"], dt, "dbias")
    if init is not None:
        assert_close(r["dinit"], g["dinit"], dt, "dinit")


SHAPES = [(1, 8, 16), (2, 64, 128), (3, 40, 1000), (2, 520, 37), (1, 3, 5), (4, 256, 512)]


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("W", [2, 3, 4])
@pytest.mark.parametrize("dtype", ["fp32", "bf16", "fp16"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_sweep_vs_oracle(shape, dtype, W, layout):
    dt = DTYPES[dtype]
    B, D, L = shape
    seed = hash((shape, dtype, W, layout)) % 10000
    silu = (W % 2 == 0)
    x = seeded((B, D, L), dt, seed)
    w = seeded((D, W), dt, seed + 1, "uniform")
    b = seeded((D,), dt, seed + 2, "uniform") if W != 3 else None
    dout = seeded((B, D, L), dt, seed + 3)
    _compare_oracle(x, w, b, None, None, dout, None, silu, False, layout)


@pytest.mark.parametrize("layout", ["contig", "chanlast", "strided"])
@pytest.mark.parametrize("W", [2, 4])
@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("L", [1, 2, 3, 5, 300, 2100, 4096])
def test_states_vs_oracle(L, dtype, W, layout):
    dt = DTYPES[dtype]
    B, D = 2, 72
    seed = 7 * L + W
    x = seeded((B, D, L), dt, seed)
    w = seeded((D, W), dt, seed + 1, "uniform")
    b = seeded((D,), dt, seed + 2, "uniform")
    init = seeded((B, D, W - 1), dt, seed + 3)
    dout = seeded((B, D, L), dt, seed + 4)
    dfinal = seeded((B, D, W - 1), dt, seed + 5)
    _compare_oracle(x, w, b, None, init, dout, dfinal, True, True, layout)


@pytest.mark.parametrize("layout", ["contig", "chanlast", "strided"])
@pytest.mark.parametrize("W", [2, 3, 4])
@pytest.mark.parametrize("dtype", ["fp32", "bf16", "fp16"])
@pytest.mark.parametrize("L", [64, 1000])
def test_seq_idx_vs_oracle(L, dtype, W, layout):
    dt = DTYPES[dtype]
    B, D = 2, 40
    seed = 13 * L + W
    x = seeded((B, D, L), dt, seed)
    w = seeded((D, W), dt, seed + 1, "uniform")
    b = seeded((D,), dt, seed + 2, "uniform")
    dout = seeded((B, D, L), dt, seed + 4)
    seq = random_seq_idx(B, L, seed)
    _compare_oracle(x, w, b, seq, None, dout, None, W != 3, False, layout)


@pytest.mark.parametrize("shape", [(2, 64, 9), (2, 64, 255), (2, 64, 257), (3, 24, 2047), (1, 16, 5001), (2, 65, 100),
                                   (2, 65, 99)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("W", [2, 4])
@pytest.mark.parametrize("dtype", ["fp32", "bf16", "fp16"])
def test_contiguous_unaligned_rows_vs_oracle(shape, dtype, W):
    """Contiguous rows whose pitch is not a multiple of 16 bytes (the
    shifted-row TMA kernels: tiles on the tensor's 16-byte grid, row starts
    inside a lane, row ends inside a tile, long rows split into segments),
    with initial and final states.  The extents give view rows of 128 bytes
    ((2, 64, 9)), 32 bytes ((1, 16, 5001) in 16-bit types) and 16 bytes
    ((2, 65, 100) in 16-bit types); (2, 65, 99) in 16-bit types has an extent
    that is not a whole number of 16-byte units and takes the register
    kernels."""
    dt = DTYPES[dtype]
    B, D, L = shape
    seed = 7 * L + W + D
    x = seeded((B, D, L), dt, seed)
    w = seeded((D, W), dt, seed + 1, "uniform")
    b = seeded((D,), dt, seed + 2, "uniform")
    init = seeded((B, D, W - 1), dt, seed + 3)
    dout = seeded((B, D, L), dt, seed + 4)
    dfinal = seeded((B, D, W - 1), dt, seed + 5)
    _compare_oracle(x, w, b, None, init, dout, dfinal, True, True, "contig")


@pytest.mark.parametrize("dtype,W", [("bf16", 5), ("bf16", 7), ("bf16", 9), ("fp16", 9), ("fp32", 5)])
def test_contiguous_unaligned_wide_widths_vs_oracle(dtype, W):
    """Wide kernels on rows whose pitch is not a multiple of 16 bytes: the
    halo reaches up to 8 positions back, across the lane whose first tile
    element sits before the row start."""
    dt = DTYPES[dtype]
    B, D, L = 2, 48, 2047
    seed = 13 * W + L
    x = seeded((B, D, L), dt, seed)
    w = seeded((D, W), dt, seed + 1, "uniform")
    b = seeded((D,), dt, seed + 2, "uniform")
    init = seeded((B, D, W - 1), dt, seed + 3)
    dout = seeded((B, D, L), dt, seed + 4)
    dfinal = seeded((B, D, W - 1), dt, seed + 5)
    _compare_oracle(x, w, b, None, init, dout, dfinal, True, True, "contig")


@pytest.mark.parametrize("shape", [(3, 6400, 2101), (1, 5920, 4097)], ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_contiguous_unaligned_long_segments_vs_oracle(shape, dtype):
    """Unaligned contiguous rows with enough (batch, channel group) pairs
    that segments span many tiles: the shared-memory ring wraps, the last
    segment takes one tile more than its length when the row starts
    mid-unit, and (second shape) a row splits into several multi-tile
    segments."""
    dt = DTYPES[dtype]
    B, D, L = shape
    W = 4
    seed = 11 * L + D
    x = seeded((B, D, L), dt, seed)
    w = seeded((D, W), dt, seed + 1, "uniform")
    b = seeded((D,), dt, seed + 2, "uniform")
    init = seeded((B, D, W - 1), dt, seed + 3)
    dout = seeded((B, D, L), dt, seed + 4)
    dfinal = seeded((B, D, W - 1), dt, seed + 5)
    _compare_oracle(x, w, b, None, init, dout, dfinal, True, True, "contig")


@pytest.mark.parametrize("layout", ["contig", "chanlast"])
@pytest.mark.parametrize("W", [2, 4])
@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_seq_idx_long_runs_vs_oracle(dtype, W, layout):
    """Packed sequences much longer than a tile (the kernels' ungated path
    for tiles without a boundary), a padding run, boundaries inside and at
    the edges of tiles, and segment splits of long rows."""
    dt = DTYPES[dtype]
    B, D, L = 2, 48, 4096
    seed = 91 + W
    x = seeded((B, D, L), dt, seed)
    w = seeded((D, W), dt, seed + 1, "uniform")
    b = seeded((D,), dt, seed + 2, "uniform")
    dout = seeded((B, D, L), dt, seed + 4)
    runs = [[(1000, 0), (300, -1), (1, 1), (1259, 2), (1536, 3)], [(256, 0), (256, 1), (2048, 2), (1536, -1)]]
    seq = torch.empty(B, L, dtype=torch.int32)
    for r, row in enumerate(runs):
        t = 0
        for n, v in row:
            seq[r, t:t + n] = v
            t += n
        assert t == L
    _compare_oracle(x, w, b, seq, None, dout, None, True, False, layout)


@pytest.mark.parametrize("layout", ["contig", "chanlast"])
@pytest.mark.parametrize("W", [3, 4])
@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_seq_idx_reused_ids_and_step_edges_vs_oracle(dtype, W, layout):
    """seq_idx whose boundaries sit on and next to the contiguous backward's
    248-position tile steps, an id that comes back after a one- or
    two-position run of another id (taps compare ids, so a tap may reach
    across the short run), padding between runs of one id, and a row
    (second batch row) that is one sequence throughout."""
    dt = DTYPES[dtype]
    B, D, L = 2, 40, 2976  # 12 steps of 248
    seed = 57 + W
    x = seeded((B, D, L), dt, seed)
    w = seeded((D, W), dt, seed + 1, "uniform")
    b = seeded((D,), dt, seed + 2, "uniform")
    dout = seeded((B, D, L), dt, seed + 4)
    runs = [(248, 0), (1, 1), (247, 0), (248, 2), (2, 3), (250, 2), (1, -1), (495, 4), (3, -1), (248, 4), (1, 5),
            (1, 4), (1, 5), (1230, 6)]
    seq = torch.empty(B, L, dtype=torch.int32)
    t = 0
    for n, v in runs:
        seq[0, t:t + n] = v
        t += n
    assert t == L
    seq[1] = 7
    _compare_oracle(x, w, b, seq, None, dout, None, True, False, layout)


@pytest.mark.parametrize("seq", [False, True])
@pytest.mark.parametrize("W", [2, 4])
@pytest.mark.parametrize("dtype", ["fp32", "bf16", "fp16"])
def test_chanlast_odd_dim_vs_oracle(dtype, W, seq):
    """Channel-last data whose dim is not a multiple of 8 (rows not 16-byte
    aligned, so neither TMA nor vector loads apply): the register kernels,
    with a lane's channels 32 apart; several channel groups, the last one
    ragged, with initial / final states (or seq_idx)."""
    dt = DTYPES[dtype]
    B, D, L = 2, 299, 300
    seed = 31 * D + W + (7 if seq else 0)
    x = seeded((B, D, L), dt, seed)
    w = seeded((D, W), dt, seed + 1, "uniform")
    b = seeded((D,), dt, seed + 2, "uniform")
    dout = seeded((B, D, L), dt, seed + 4)
    if seq:
        _compare_oracle(x, w, b, random_seq_idx(B, L, seed), None, dout, None, True, False, "chanlast")
    else:
        init = seeded((B, D, W - 1), dt, seed + 3)
        dfinal = seeded((B, D, W - 1), dt, seed + 5)
        _compare_oracle(x, w, b, None, init, dout, dfinal, True, True, "chanlast")


@pytest.mark.parametrize("W", [5, 6, 7, 8, 9])
@pytest.mark.parametrize("layout", ["contig", "chanlast"])
def test_wide_widths_vs_oracle(W, layout):
    dt = torch.bfloat16
    B, D, L = 2, 48, 2048
    x = seeded((B, D, L), dt, W)
    w = seeded((D, W), dt, W + 1, "uniform")
    b = seeded((D,), dt, W + 2, "uniform")
    init = seeded((B, D, W - 1), dt, W + 3)
    dout = seeded((B, D, L), dt, W + 4)
    dfinal = seeded((B, D, W - 1), dt, W + 5)
    _compare_oracle(x, w, b, None, init, dout, dfinal, True, True, layout)


@pytest.mark.parametrize("shape,layout", [((1, 4, 40000), "contig"), ((1, 2, 70001), "contig"),
                                          ((3, 96, 777), "chanlast"), ((5, 264, 131), "chanlast")])
def test_long_rows_and_split_runs(shape, layout):
    """Rows split into several segments (seq layout) and time runs that
    straddle batch boundaries (channel-last layout)."""
    dt = torch.float32
    B, D, L = shape
    W = 4
    x = seeded(shape, dt, 1)
    w = seeded((D, W), dt, 2, "uniform")
    b = seeded((D,), dt, 3, "uniform")
    init = seeded((B, D, W - 1), dt, 4)
    dout = seeded(shape, dt, 5)
    dfinal = seeded((B, D, W - 1), dt, 6)
    _compare_oracle(x, w, b, None, init, dout, dfinal, True, True, layout)


@pytest.mark.parametrize("layout", ["contig", "chanlast"])
def test_backward_is_deterministic(layout):
    dt = torch.bfloat16
    B, D, L, W = 4, 320, 3000, 4
    x = with_layout(seeded((B, D, L), dt, 1, device=DEV), layout)
    w = seeded((D, W), dt, 2, "uniform", device=DEV)
    b = seeded((D,), dt, 3, "uniform", device=DEV)
    dout = with_layout(seeded((B, D, L), dt, 4, device=DEV), layout)
    results = []
    for _ in range(3):
        xg, wg, bg = x.detach().requires_grad_(), w.detach().requires_grad_(), b.detach().requires_grad_()
        causal_conv1d_fn(xg, wg, bg, activation="silu").backward(dout)
        results.append((xg.grad.clone(), wg.grad.clone(), bg.grad.clone()))
    for r in results[1:]:
        for a, e in zip(r, results[0]):
            assert torch.equal(a, e)


def test_dout_layout_differs_from_x():
    dt = torch.bfloat16
    B, D, L, W = 2, 256, 300, 4
    x = seeded((B, D, L), dt, 1)
    w = seeded((D, W), dt, 2, "uniform")
    dout = seeded((B, D, L), dt, 3)
    xg = with_layout(x.to(DEV), "chanlast").requires_grad_()
    wg = w.to(DEV).requires_grad_()
    causal_conv1d_fn(xg, wg, activation="silu").backward(dout.to(DEV).contiguous())
    g = oracle.bwd(x, w, dout, silu=True)
    assert_close(xg.grad.cpu(), g["dx"], dt, "dx")
    _reduction_close(wg.grad.float().cpu(), g["dweight"], dt, "dweight")


@pytest.mark.parametrize("layout", ["contig", "chanlast"])
@pytest.mark.parametrize("dtype", ["fp32", "bf16", "fp16"])
def test_chunked_prefill_roundtrip_is_exact(dtype, layout):
    """final_states of chunk i fed as initial_states of chunk i+1 reproduces
    the one-shot forward bit for bit (reference tests/test_fwd.py:262-291)."""
    dt = DTYPES[dtype]
    B, D, L, W = 2, 96, 1000, 4
    x = with_layout(seeded((B, D, L), dt, 1, device=DEV), layout)
    w = seeded((D, W), dt, 2, "uniform", device=DEV)
    b = seeded((D,), dt, 3, "uniform", device=DEV)
    full = causal_conv1d_fn(x, w, b, activation="silu")
    init, outs = None, []
    for s, e in [(0, 1), (1, 3), (3, 400), (400, 1000)]:
        o, init = causal_conv1d_fn(x[..., s:e], w, b, initial_states=init, return_final_states=True,
                                   activation="silu")
        outs.append(o)
    assert torch.equal(torch.cat(outs, -1), full)


@pytest.mark.parametrize("shape", [(0, 64, 128), (2, 0, 128), (2, 64, 0), (0, 0, 0)])
@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_zero_sized(shape, dtype):
    dt = DTYPES[dtype]
    B, D, L = shape
    x = torch.randn(B, D, L, dtype=dt, device=DEV, requires_grad=True)
    w = torch.randn(D, 4, dtype=dt, device=DEV, requires_grad=True)
    b = torch.randn(D, dtype=dt, device=DEV, requires_grad=True)
    out = causal_conv1d_fn(x, w, b, activation="silu")
    assert out.shape == x.shape and out.dtype == x.dtype and out.numel() == 0
    out.backward(torch.randn_like(out))
    assert x.grad.shape == x.shape and w.grad.shape == w.shape and b.grad.shape == b.shape
    assert torch.all(w.grad == 0) and torch.all(b.grad == 0)


def test_zero_length_with_states():
    dt = torch.float32
    B, D, W = 2, 8, 4
    x = torch.randn(B, D, 0, dtype=dt, device=DEV, requires_grad=True)
    w = torch.randn(D, W, dtype=dt, device=DEV, requires_grad=True)
    init = torch.randn(B, D, W - 1, dtype=dt, device=DEV, requires_grad=True)
    out, fs = causal_conv1d_fn(x, w, initial_states=init, return_final_states=True)
    assert torch.equal(fs, init)  # final = last W-1 of cat([init, x]) = init
    dfs = torch.randn_like(fs)
    torch.autograd.backward([out, fs], [torch.randn_like(out), dfs])
    assert torch.equal(init.grad, dfs)


# ---- reads like the reference's own tests (tests/test_fwd.py:28-43) --------

@pytest.mark.parametrize("shape", [(1, 8, 16), (2, 64, 128), (4, 256, 512)])
@pytest.mark.parametrize("activation", [None, "silu", "swish"])
@pytest.mark.parametrize("dtype", ["fp32", "bf16", "fp16"])
def test_contiguous_vs_causal_conv1d_ref(shape, activation, dtype):
    dt = DTYPES[dtype]
    B, D, L = shape
    x = torch.randn(B, D, L, dtype=dt, device=DEV)
    w = torch.randn(D, 4, dtype=dt, device=DEV)
    b = torch.randn(D, dtype=dt, device=DEV)
    out = causal_conv1d_fn(x, w, b, activation=activation)
    ref = causal_conv1d_ref(x.double(), w.double(), b.double(), activation=activation)
    assert_close(out, ref.to(dt), dt, "out")
