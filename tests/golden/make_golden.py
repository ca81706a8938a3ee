"""Generates the golden fixtures in this directory from the REFERENCE itself.

Run where a checkout of the reference is available, passing its root:

    python tests/golden/make_golden.py <reference-checkout>
    (or set CC1D_REFERENCE=<reference-checkout>)

It imports the reference's pure-PyTorch implementation
(src/causal_conv1d_mojo/reference.py: causal_conv1d_ref,
causal_conv1d_update_ref) by file path -- the package itself needs the Mojo
toolchain and cannot be imported here -- and evaluates it in float64 on
seeded inputs, including autograd for the backward.  seq_idx cases use the
per-segment evaluation of the reference's test helpers
(tests/_helpers.py:98-156); indexed decode pools use the gather / update /
scatter pattern of tests/test_update.py:174-243; the varlen known-answer
cases are those of tests/test_varlen.py:25-73.

Outputs (committed): golden_<group>.npz with one entry per case and array,
plus cases.json describing each case.  Inputs are stored as float32 holding
the exact dtype-rounded values; expected outputs are float32 of the float64
result.  Nothing at test time reads the reference.
"""

from __future__ import annotations

import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF_ROOT = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CC1D_REFERENCE", "reference"))
REF_PY = REF_ROOT / "src" / "causal_conv1d_mojo" / "reference.py"

DT = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


def load_reference():
    spec = importlib.util.spec_from_file_location("_cc1d_reference_py", REF_PY)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# --------------------------------------------------------------------------
# Case lists
# --------------------------------------------------------------------------

def conv_cases():
    cases = []

    def add(name, dtype, B, D, L, W, bias=True, silu=True, init=False, final=False, dfinal=False, seq=None,
            bwd=True, seed=0):
        cases.append(dict(name=name, dtype=dtype, B=B, D=D, L=L, W=W, bias=bias, silu=silu, init=init,
                          final=final, dfinal=dfinal, seq=seq, bwd=bwd, seed=seed))

    # fp32 (2, 64, 512), W=4, bias, silu, fwd + bwd.
    add("c1_fp32", "fp32", 2, 64, 512, 4)
    add("fp32_w2_plain", "fp32", 2, 16, 37, 2, bias=False, silu=False, seed=1)
    add("fp32_w3", "fp32", 1, 8, 70, 3, seed=2)
    add("fp32_w5", "fp32", 2, 8, 64, 5, seed=3)
    add("bf16_w4", "bf16", 2, 16, 100, 4, seed=4)
    add("bf16_w2_nobias", "bf16", 2, 8, 33, 2, bias=False, seed=5)
    add("fp16_w3_nosilu", "fp16", 2, 8, 50, 3, silu=False, seed=6)
    add("fp16_w4_states", "fp16", 2, 16, 64, 4, init=True, final=True, dfinal=True, seed=7)
    add("bf16_w4_states_short", "bf16", 2, 8, 2, 4, init=True, final=True, dfinal=True, seed=8)
    add("fp32_w4_final_short", "fp32", 2, 8, 2, 4, final=True, dfinal=True, seed=9)
    add("fp32_w3_states", "fp32", 2, 8, 40, 3, init=True, final=True, dfinal=True, seed=10)
    add("bf16_w4_len1_states", "bf16", 2, 8, 1, 4, init=True, final=True, dfinal=True, seed=11)
    add("fp32_w4_long", "fp32", 1, 4, 3000, 4, init=True, final=True, dfinal=True, seed=12)
    for i, pat in enumerate(["single", "two_equal", "varied", "with_padding"]):
        add(f"fp32_seq_{pat}", "fp32", 2, 16, 64, 4, seq=pat, seed=20 + i)
        add(f"bf16_seq_{pat}", "bf16", 2, 16, 64, 4, seq=pat, silu=(i % 2 == 0), seed=30 + i)
    add("fp16_seq_w3_nobias", "fp16", 1, 16, 64, 3, bias=False, seq="two_equal", seed=40)
    for W in range(5, 10):
        add(f"fp16_w{W}", "fp16", 2, 16, 64, W, seed=50 + W)
    add("bf16_w9_states", "bf16", 1, 8, 40, 9, init=True, final=True, dfinal=True, seed=60)
    return cases


def update_cases():
    cases = []

    def add(name, dtype, B, D, L, W, S, bias=True, silu=True, mode="linear", pool=None, idx=None, cache=None,
            seed=0):
        cases.append(dict(name=name, dtype=dtype, B=B, D=D, L=L, W=W, S=S, bias=bias, silu=silu, mode=mode,
                          pool=pool, idx=idx, cache=cache, seed=seed))

    for i, (dt, W) in enumerate([("fp32", 2), ("bf16", 3), ("fp16", 4), ("bf16", 4)]):
        add(f"lin_{dt}_w{W}_tok", dt, 2, 16, 1, W, W - 1, bias=(i % 2 == 0), silu=(i != 1), seed=100 + i)
    add("lin_fp32_burst", "fp32", 1, 8, 3, 4, 8, seed=110)
    add("lin_bf16_burst_gt_state", "bf16", 2, 8, 6, 4, 3, seed=111)
    add("lin_fp16_w9", "fp16", 2, 8, 1, 9, 8, seed=112)
    add("circ_fp32_w4", "fp32", 2, 16, 1, 4, 9, mode="circular", cache=[4, 12], seed=120)
    add("circ_bf16_w3_burst", "bf16", 2, 8, 2, 3, 8, mode="circular", cache=[7, 1023], seed=121)
    add("circ_fp16_exact", "fp16", 1, 8, 1, 4, 3, mode="circular", cache=[5], seed=122)
    add("circ_fp32_negative", "fp32", 2, 8, 1, 4, 6, mode="circular", cache=[-1, -8], seed=123)
    add("pool_bf16", "bf16", 3, 16, 1, 4, 3, mode="linear", pool=5, idx=[3, 0, 4], seed=130)
    add("pool_fp16_padding", "fp16", 3, 8, 1, 4, 3, mode="linear", pool=4, idx=[0, -1, 2], silu=False, seed=131)
    add("pool_circ_bf16", "bf16", 4, 16, 1, 4, 8, mode="circular", pool=6, idx=[5, -1, 0, 2], cache=[3, 9, 0, 17],
        seed=132)
    return cases


def varlen_cases():
    return [
        dict(name="kat_basic", dtype="fp32", cu=[0, 5, 7, 11], D=2, S=3, arange=True),
        dict(name="kat_empty_middle", dtype="fp32", cu=[0, 3, 3, 5], D=4, S=2, arange=True),
        dict(name="kat_state_longer", dtype="fp16", cu=[0, 2, 4], D=3, S=8, arange=True),
        dict(name="rand_bf16", dtype="bf16", cu=[0, 17, 17, 32, 80], D=64, S=10, arange=False, seed=200),
    ]


# --------------------------------------------------------------------------
# Inputs (same recipe as bench.py: fp32 draws, cast to dtype)
# --------------------------------------------------------------------------

def seq_pattern(pat, B, L):
    if pat == "single":
        s = torch.zeros(B, L, dtype=torch.int32)
    elif pat == "two_equal":
        s = torch.cat([torch.zeros(B, L // 2, dtype=torch.int32), torch.ones(B, L - L // 2, dtype=torch.int32)], 1)
    elif pat == "varied":
        s = torch.cat([torch.zeros(B, 10, dtype=torch.int32), torch.ones(B, 25, dtype=torch.int32),
                       torch.full((B, L - 35), 2, dtype=torch.int32)], 1)
    elif pat == "with_padding":
        s = torch.cat([torch.zeros(B, 16, dtype=torch.int32), torch.full((B, 16), -1, dtype=torch.int32),
                       torch.ones(B, L - 32, dtype=torch.int32)], 1)
    else:
        raise ValueError(pat)
    return s


def conv_inputs(c):
    dt = DT[c["dtype"]]
    g = torch.Generator("cpu").manual_seed(c["seed"])
    B, D, L, W = c["B"], c["D"], c["L"], c["W"]
    x = torch.randn(B, D, L, generator=g).to(dt)
    w = (torch.rand(D, W, generator=g) - 0.5).to(dt)
    b = (torch.rand(D, generator=g) - 0.5).to(dt) if c["bias"] else None
    init = torch.randn(B, D, W - 1, generator=g).to(dt) if c["init"] else None
    g1 = torch.Generator("cpu").manual_seed(c["seed"] + 1)
    dout = torch.randn(B, D, L, generator=g1).to(dt)
    dfinal = torch.randn(B, D, W - 1, generator=g1).to(dt) if c["dfinal"] else None
    seq = seq_pattern(c["seq"], B, L) if c["seq"] else None
    return dict(x=x, weight=w, bias=b, initial_states=init, dout=dout, dfinal=dfinal, seq_idx=seq)


def update_inputs(c):
    dt = DT[c["dtype"]]
    g = torch.Generator("cpu").manual_seed(c["seed"])
    B, D, L, W, S = c["B"], c["D"], c["L"], c["W"], c["S"]
    x = torch.randn(B, D, L, generator=g).to(dt)
    w = (torch.rand(D, W, generator=g) - 0.5).to(dt)
    b = (torch.rand(D, generator=g) - 0.5).to(dt) if c["bias"] else None
    rows = c["pool"] if c["pool"] else B
    state = torch.randn(rows, D, S, generator=g).to(dt)
    idx = torch.tensor(c["idx"], dtype=torch.int32) if c["idx"] is not None else None
    cache = torch.tensor(c["cache"], dtype=torch.int32) if c["cache"] is not None else None
    return dict(x=x, weight=w, bias=b, conv_state=state, conv_state_indices=idx, cache_seqlens=cache)


def varlen_inputs(c):
    dt = DT[c["dtype"]]
    total = c["cu"][-1]
    if c["arange"]:
        x = torch.arange(total * c["D"], dtype=torch.float32).reshape(total, c["D"]).to(dt)
    else:
        g = torch.Generator("cpu").manual_seed(c["seed"])
        x = torch.randn(total, c["D"], generator=g).to(dt)
    return dict(x=x, cu_seqlens=torch.tensor(c["cu"], dtype=torch.int32))


# --------------------------------------------------------------------------
# Reference evaluation (float64)
# --------------------------------------------------------------------------

def ref_conv(ref, c, inp):
    act = "silu" if c["silu"] else None
    f64 = lambda t: None if t is None else t.double().detach().clone().requires_grad_(t.dtype != torch.int32)  # noqa: E731
    x, w, b, init = f64(inp["x"]), f64(inp["weight"]), f64(inp["bias"]), f64(inp["initial_states"])
    dout = inp["dout"].double()
    res = {}
    if c["seq"] is None:
        r = ref.causal_conv1d_ref(x, w, b, initial_states=init, return_final_states=c["final"], activation=act)
        out, fs = (r if c["final"] else (r, None))
        loss = (out * dout).sum()
        if fs is not None and inp["dfinal"] is not None:
            loss = loss + (fs * inp["dfinal"].double()).sum()
        res["out"] = out.detach()
        if fs is not None:
            res["final_states"] = fs.detach()
        if c["bwd"]:
            loss.backward()
    else:
        seq = inp["seq_idx"]
        B, D, L = x.shape
        out = torch.zeros(B, D, L, dtype=torch.float64)
        for bi in range(B):
            ids = seq[bi].tolist()
            s = 0
            while s < L:
                e = s + 1
                while e < L and ids[e] == ids[s]:
                    e += 1
                if ids[s] >= 0:
                    seg = ref.causal_conv1d_ref(x[bi:bi + 1, :, s:e], w, b, activation=act)
                    out[bi:bi + 1, :, s:e] = seg.detach()
                    if c["bwd"]:
                        (seg * dout[bi:bi + 1, :, s:e]).sum().backward()
                s = e
        res["out"] = out
    if c["bwd"]:
        res["dx"] = x.grad if x.grad is not None else torch.zeros_like(x)
        res["dweight"] = w.grad if w.grad is not None else torch.zeros_like(w)
        if b is not None:
            res["dbias"] = b.grad if b.grad is not None else torch.zeros_like(b)
        if init is not None:
            res["dinit"] = init.grad if init.grad is not None else torch.zeros_like(init)
    return res


def ref_update(ref, c, inp):
    act = "silu" if c["silu"] else None
    x = inp["x"].double()
    w = inp["weight"].double()
    b = None if inp["bias"] is None else inp["bias"].double()
    state = inp["conv_state"].double().clone()
    cache = inp["cache_seqlens"]
    idx = inp["conv_state_indices"]
    B, D, L = x.shape
    out = torch.zeros(B, D, L, dtype=torch.float64)
    if idx is None:
        out = ref.causal_conv1d_update_ref(x, state, w, b, activation=act, cache_seqlens=cache)
    else:
        real = [i for i in range(B) if int(idx[i]) >= 0]
        rows = torch.tensor([int(idx[i]) for i in real], dtype=torch.long)
        sub = state[rows].clone()
        cs = cache[real] if cache is not None else None
        o = ref.causal_conv1d_update_ref(x[real], sub, w, b, activation=act, cache_seqlens=cs)
        out[real] = o
        state[rows] = sub
    return dict(out=out, conv_state=state)


def ref_varlen(c, inp):
    # Known-answer semantics of tests/test_varlen.py:25-73, evaluated directly.
    x, cu, S = inp["x"], inp["cu_seqlens"].tolist(), c["S"]
    B = len(cu) - 1
    st = torch.zeros(B, x.shape[1], S, dtype=torch.float64)
    for i in range(B):
        end = cu[i + 1]
        start = max(cu[i], end - S)
        n = end - start
        if n > 0:
            st[i, :, S - n:] = x[start:end].double().T
    return dict(states=st)


def _np(t):
    return t.detach().to(torch.float32).numpy() if t.dtype != torch.int32 else t.numpy()


def main() -> int:
    if not REF_PY.is_file():
        print(f"reference not found at {REF_PY}", file=sys.stderr)
        return 1
    ref = load_reference()
    manifest = {"reference": str(REF_PY.relative_to(REF_ROOT)), "groups": {}}
    for group, cases, mk, ev in [
        ("conv", conv_cases(), conv_inputs, lambda c, i: ref_conv(ref, c, i)),
        ("update", update_cases(), update_inputs, lambda c, i: ref_update(ref, c, i)),
        ("varlen", varlen_cases(), varlen_inputs, ref_varlen),
    ]:
        arrays = {}
        for c in cases:
            inp = mk(c)
            exp = ev(c, inp)
            for k, v in inp.items():
                if v is not None:
                    arrays[f"{c['name']}/in/{k}"] = _np(v)
            for k, v in exp.items():
                arrays[f"{c['name']}/exp/{k}"] = _np(v)
        np.savez_compressed(HERE / f"golden_{group}.npz", **arrays)
        manifest["groups"][group] = cases
    (HERE / "cases.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print("wrote", sorted(p.name for p in HERE.glob("golden_*.npz")))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
