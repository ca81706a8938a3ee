"""Production-pattern integration on the GPU: CUDA-graph capture/replay
(reference tests/test_cuda_graph.py:43-131), torch.compile(fullgraph=True)
(reference tests/test_fwd.py:494-531), launches on a non-default stream, and
that the native library -- not some fallback -- is what runs."""

from __future__ import annotations

import pytest
import torch

from causal_conv1d_b200 import _lib, causal_conv1d_fn, causal_conv1d_update

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_native_library_is_loaded():
    import ctypes

    _lib.load()
    with open("/proc/self/maps") as f:
        maps = f.read()
    assert _lib.LIB_NAME in maps
    assert isinstance(_lib.load(), ctypes.CDLL)


def test_cuda_graph_capture_and_replay_matches_eager():
    B, D, L, W = 2, 64, 128, 4
    x = torch.randn(B, D, L, dtype=torch.float16, device=DEV)
    w = torch.randn(D, W, dtype=torch.float16, device=DEV)
    b = torch.randn(D, dtype=torch.float16, device=DEV)
    causal_conv1d_fn(x, w, b, activation="silu")  # warm-up outside capture
    out_buf = torch.empty_like(x)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out_buf.copy_(causal_conv1d_fn(x, w, b, activation="silu"))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out_buf, causal_conv1d_fn(x, w, b, activation="silu"))
    x.add_(0.5)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out_buf, causal_conv1d_fn(x, w, b, activation="silu"))


def test_cuda_graph_fwd_bwd_and_update():
    B, D, L, W = 2, 256, 512, 4
    x = torch.randn(B, L, D, dtype=torch.bfloat16, device=DEV).transpose(1, 2).requires_grad_()
    w = torch.randn(D, W, dtype=torch.bfloat16, device=DEV, requires_grad=True)
    dout = torch.randn(B, L, D, dtype=torch.bfloat16, device=DEV).transpose(1, 2)
    state = torch.randn(B, D, W - 1, dtype=torch.bfloat16, device=DEV)
    xt = torch.randn(B, D, dtype=torch.bfloat16, device=DEV)

    def step():
        out = causal_conv1d_fn(x, w, activation="silu")
        gx, gw = torch.autograd.grad(out, (x, w), dout)
        y = causal_conv1d_update(xt, state, w.detach(), activation="silu")
        return gx, gw, y

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(s)
    st0 = state.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        gx, gw, y = step()
    state.copy_(st0)
    g.replay()
    torch.cuda.synchronize()
    state_after = state.clone()
    state.copy_(st0)
    ex, ew, ey = step()
    torch.cuda.synchronize()
    assert torch.equal(gx, ex) and torch.equal(gw, ew) and torch.equal(y, ey)
    assert torch.equal(state_after, state)


def test_torch_compile_fullgraph():
    B, D, L = 2, 64, 128
    x = torch.randn(B, D, L, dtype=torch.float16, device=DEV)
    w = torch.randn(D, 4, dtype=torch.float16, device=DEV)
    b = torch.randn(D, dtype=torch.float16, device=DEV)

    @torch.compile(fullgraph=True)
    def f(x, w, b):
        return causal_conv1d_fn(x, w, b, activation="silu")

    assert torch.equal(f(x, w, b), causal_conv1d_fn(x, w, b, activation="silu"))


def test_torch_compile_autograd():
    B, D, L = 2, 64, 128
    x = torch.randn(B, D, L, dtype=torch.float16, device=DEV, requires_grad=True)
    w = torch.randn(D, 4, dtype=torch.float16, device=DEV, requires_grad=True)
    b = torch.randn(D, dtype=torch.float16, device=DEV, requires_grad=True)

    @torch.compile
    def f(x, w, b):
        return causal_conv1d_fn(x, w, b, activation="silu").sum()

    f(x, w, b).backward()
    assert x.grad is not None and w.grad is not None and b.grad is not None
    x2, w2, b2 = (t.detach().clone().requires_grad_() for t in (x, w, b))
    causal_conv1d_fn(x2, w2, b2, activation="silu").sum().backward()
    assert torch.equal(x.grad, x2.grad) and torch.equal(w.grad, w2.grad)


def test_non_default_stream():
    B, D, L = 2, 128, 4096
    x = torch.randn(B, D, L, dtype=torch.bfloat16, device=DEV)
    w = torch.randn(D, 4, dtype=torch.bfloat16, device=DEV)
    ref = causal_conv1d_fn(x, w, activation="silu")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        out = causal_conv1d_fn(x, w, activation="silu")
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_pipeline_waits_never_time_out():
    """The TMA pipelines' bounded mbarrier waits all completed (the device
    counter of given-up waits stays 0) across the layouts that use them."""
    _lib.device_wait_timeouts()  # clear
    for D, L in [(256, 1000), (5376, 777), (264, 31)]:
        x = torch.randn(3, L, D, dtype=torch.bfloat16, device=DEV).transpose(1, 2).requires_grad_()
        w = torch.randn(D, 4, dtype=torch.bfloat16, device=DEV, requires_grad=True)
        init = torch.randn(3, D, 3, dtype=torch.bfloat16, device=DEV, requires_grad=True)
        out, fs = causal_conv1d_fn(x, w, initial_states=init, return_final_states=True, activation="silu")
        torch.autograd.backward([out, fs], [torch.randn_like(out), torch.randn_like(fs)])
    assert _lib.device_wait_timeouts() == 0


@pytest.mark.parametrize("layout", ["chanlast", "contig"])
def test_calls_from_a_fresh_host_thread(layout):
    """A host thread that no framework ever bound to a device (as an autograd
    worker thread of device 0 can be): the first call there goes straight to
    a TMA kernel whose launch setup is already cached, so the library itself
    must bind the device's context before encoding tensor maps.  Results
    equal the main thread's bitwise."""
    import threading

    from causal_conv1d_b200 import _ops

    B, D, L, W = 2, 512, 256, 4
    g = torch.Generator(device="cpu").manual_seed(3)

    def mk(*s):
        return torch.randn(*s, generator=g).to(torch.bfloat16).to(DEV)

    if layout == "chanlast":
        x, dout = mk(B, L, D).transpose(1, 2), mk(B, L, D).transpose(1, 2)
    else:
        x, dout = mk(B, D, L), mk(B, D, L)
    w, b = mk(D, W), mk(D)

    def run():
        out = torch.empty_like(x)
        dx = torch.empty_like(x)
        dwdb = torch.empty(D * (W + 1), dtype=torch.float32, device=DEV)
        _ops.fwd(x, w, b, None, None, out, True, None)
        _ops.bwd(x, w, b, dout, None, None, None, dx, dwdb, None, None, None, True)
        torch.cuda.synchronize()
        return out, dx, dwdb

    main = run()  # warms every launch cache on this thread
    got, errors = [], []

    def worker():
        try:
            got.append(run())
        except Exception as e:  # reported below
            errors.append(e)

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert not errors, errors
    for a, c in zip(main, got[0]):
        assert torch.equal(a, c)


def test_dependent_chains_in_one_graph_match_synchronised_eager():
    """Kernels are launched with programmatic dependent launch, so each one
    may be scheduled while its predecessor drains; every kernel must still
    see all of its predecessor's writes.  Chains whose every step consumes
    the previous step's output -- conv over conv output, backward of that,
    and 16 decode steps on one state (circular and linear) -- captured in
    one CUDA graph must equal the same chain run eagerly with a
    synchronisation after every call."""
    from causal_conv1d_b200 import _ops

    g = torch.Generator(device="cpu").manual_seed(9)
    B, D, L, W = 2, 512, 512, 4

    def mk(*s):
        return torch.randn(*s, generator=g).to(torch.bfloat16).to(DEV)

    x = mk(B, L, D).transpose(1, 2)
    w1, w2, b = mk(D, W), mk(D, W), mk(D)
    dout = mk(B, L, D).transpose(1, 2)
    xs = [mk(B, D, 1) for _ in range(16)]
    circ0, lin0 = mk(B, D, 8), mk(B, D, W - 1)
    cache = torch.arange(B, dtype=torch.int32, device=DEV)

    def chain(sync):
        y1 = torch.empty_like(x)
        y2 = torch.empty_like(x)
        dx = torch.empty_like(x)
        dwdb = torch.empty(D * (W + 1), dtype=torch.float32, device=DEV)
        circ, lin = circ0.clone(), lin0.clone()
        outs = [torch.empty(B, D, 1, dtype=torch.bfloat16, device=DEV) for _ in range(32)]

        def step(fn):
            fn()
            if sync:
                torch.cuda.synchronize()

        step(lambda: _ops.fwd(x, w1, b, None, None, y1, True, None))
        step(lambda: _ops.fwd(y1, w2, b, None, None, y2, True, None))
        step(lambda: _ops.bwd(y1, w2, b, y2, None, None, None, dx, dwdb, None, None, None, True))
        for i in range(16):
            step(lambda i=i: _ops.update(xs[i], circ, w1, b, cache + i, None, outs[2 * i], True))
            step(lambda i=i: _ops.update(xs[i], lin, w1, b, None, None, outs[2 * i + 1], True))
        return [y1, y2, dx, dwdb, circ, lin] + outs

    want = [t.clone() for t in chain(True)]
    chain(False)  # warm-up of the capture's allocations
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        got = chain(False)
    for _ in range(2):
        graph.replay()
        torch.cuda.synchronize()
        for a_, e_ in zip(got, want):
            assert torch.equal(a_, e_)
