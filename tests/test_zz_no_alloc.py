"""cc1d_bwd_noalloc: the backward entry point that allocates nothing.

It serves callers that cannot allocate device memory -- a serving engine that
has reserved almost all of HBM, an FFI caller with no access to the host
framework's allocator, or a loop that must not take cudaMalloc's implicit
synchronisation.  It uses the library's built-in static scratch array instead
of a caller-provided workspace.  These tests call it through the C ABI, twice
in a row (the shared scratch keeps the previous call's contents), and check
every output against the regular cc1d_bwd entry point within the parity
tolerances of the other tests, one channel slice against the CPU oracle, that
the device's free memory is the same before and after a call, and that
partial sums left in the scratch by a larger problem of another kernel family
do not leak into a smaller one.  The file name sorts last so that a run that
stops at the first failure has run every other test first.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

import oracle
from causal_conv1d_b200 import _lib, _ops
from conftest import TOL, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(layout, dt, B, D, L, W, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)

    def rn(*s):
        return torch.randn(*s, generator=g, device=DEV, dtype=torch.float32).to(dt)

    if layout == "chanlast":
        x = rn(B, L, D).transpose(1, 2)
        dout = rn(B, L, D).transpose(1, 2)
    else:
        x = rn(B, D, L)
        dout = rn(B, D, L)
    w = (torch.rand(D, W, generator=g, device=DEV) - 0.5).to(dt)
    b = (torch.rand(D, generator=g, device=DEV) - 0.5).to(dt)
    init = rn(B, D, W - 1)
    dfinal = rn(B, D, W - 1)
    return x, w, b, dout, init, dfinal


def _outputs(x, w, b, init):
    D, W = w.shape
    return dict(dx=torch.empty_like(x), dwdb=torch.empty(D * (W + 1), dtype=torch.float32, device=DEV),
                dinit=torch.empty_like(init), dw=torch.empty(D, W, dtype=x.dtype, device=DEV),
                db=torch.empty(D, dtype=x.dtype, device=DEV))


def _params(x, w, b, dout, init, dfinal, o):
    return _ops._bwd_params(x, w, b, dout, None, init, dfinal, o["dx"], o["dwdb"], o["dinit"], o["dw"], o["db"],
                            True)


def _run_regular(x, w, b, dout, init, dfinal):
    o = _outputs(x, w, b, init)
    _ops.bwd(x, w, b, dout, None, init, dfinal, o["dx"], o["dwdb"], o["dinit"], o["dw"], o["db"], True)
    return o


def _run_noalloc(x, w, b, dout, init, dfinal):
    o = _outputs(x, w, b, init)
    p = _params(x, w, b, dout, init, dfinal, o)
    lib = _lib.load()
    _lib.check(lib.cc1d_bwd_noalloc(ctypes.byref(p), torch.cuda.current_stream().cuda_stream), "cc1d_bwd_noalloc")
    return o


def _compare(got, want, dt):
    assert_close(got["dx"], want["dx"], dt, "dx")
    assert_close(got["dinit"], want["dinit"], dt, "dinit")
    norm = want["dwdb"].abs().max().item()
    assert_close(got["dwdb"], want["dwdb"], torch.float32, "dweight|dbias (fp32)",
                 atol=TOL[torch.float32]["atol"] * max(1.0, norm))
    assert_close(got["dw"].float(), want["dw"].float(), dt, "dweight", atol=TOL[dt]["atol"] * max(1.0, norm))
    assert_close(got["db"].float(), want["db"].float(), dt, "dbias", atol=TOL[dt]["atol"] * max(1.0, norm))


@pytest.mark.parametrize("layout,dtype,shape", [
    ("chanlast", torch.bfloat16, (8, 5376, 2048)),   # the Mamba-2 prefill shape (TMA path)
    ("contig", torch.float32, (4, 96, 3000)),         # seqlen-contiguous path
])
def test_noalloc_matches_regular_entry_point_twice(layout, dtype, shape):
    B, D, L = shape
    W = 4
    x, w, b, dout, init, dfinal = _inputs(layout, dtype, B, D, L, W, seed=11)
    want = _run_regular(x, w, b, dout, init, dfinal)
    for _ in range(2):  # the second call reuses the scratch left by the first
        got = _run_noalloc(x, w, b, dout, init, dfinal)
        torch.cuda.synchronize()
        _compare(got, want, dtype)
    # A different problem in between must not leak into the next result.
    x2, w2, b2, dout2, init2, dfinal2 = _inputs(layout, dtype, B, D, L, W, seed=12)
    want2 = _run_regular(x2, w2, b2, dout2, init2, dfinal2)
    got2 = _run_noalloc(x2, w2, b2, dout2, init2, dfinal2)
    torch.cuda.synchronize()
    _compare(got2, want2, dtype)


def test_noalloc_matches_oracle_on_a_channel_slice():
    # Rows (b, c) are independent, so channels [c0, c1) of the full problem
    # are an exact sub-problem for the CPU oracle (dweight/dbias of those
    # channels sum over every batch row).
    dt = torch.bfloat16
    B, D, L, W = 4, 1024, 1000, 4
    x, w, b, dout, init, dfinal = _inputs("chanlast", dt, B, D, L, W, seed=21)
    got = _run_noalloc(x, w, b, dout, init, dfinal)
    torch.cuda.synchronize()
    c0, c1 = 496, 560
    g = oracle.bwd(x[:, c0:c1].cpu(), w[c0:c1].cpu(), dout[:, c0:c1].cpu(), b[c0:c1].cpu(), None,
                   init[:, c0:c1].cpu(), dfinal[:, c0:c1].cpu(), silu=True)
    assert_close(got["dx"][:, c0:c1], g["dx"], dt, "dx vs oracle")
    assert_close(got["dinit"][:, c0:c1], g["dinit"], dt, "dinit vs oracle")
    norm = g["dweight"].abs().max().item()
    assert_close(got["dw"][c0:c1].float(), g["dweight"], dt, "dweight vs oracle", atol=TOL[dt]["atol"] * max(1.0, norm))
    assert_close(got["db"][c0:c1].float(), g["dbias"], dt, "dbias vs oracle", atol=TOL[dt]["atol"] * max(1.0, norm))


def test_noalloc_call_leaves_free_device_memory_unchanged():
    dt = torch.bfloat16
    B, D, L, W = 2, 2048, 512, 4
    x, w, b, dout, init, dfinal = _inputs("chanlast", dt, B, D, L, W, seed=5)
    o = _outputs(x, w, b, init)
    p = _params(x, w, b, dout, init, dfinal, o)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    # The first call on a device may load the library's device code (which
    # holds the static scratch array); every later call must allocate nothing.
    _lib.check(lib.cc1d_bwd_noalloc(ctypes.byref(p), stream), "cc1d_bwd_noalloc")
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        _lib.check(lib.cc1d_bwd_noalloc(ctypes.byref(p), stream), "cc1d_bwd_noalloc")
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes across no-allocation calls"


def test_noalloc_stale_partials_of_a_larger_problem_do_not_leak():
    # A large channel-last bf16 call fills many partial-sum slots of the
    # shared scratch; a smaller seqlen-contiguous fp32 call (another kernel
    # family, fewer slots) right after must read only its own slots.
    big = _inputs("chanlast", torch.bfloat16, 8, 5376, 2048, 4, seed=31)
    small = _inputs("contig", torch.float32, 2, 80, 700, 3, seed=32)
    _run_noalloc(*big)
    got = _run_noalloc(*small)
    torch.cuda.synchronize()
    _compare(got, _run_regular(*small), torch.float32)


def test_noalloc_empty_batch_takes_no_scratch_and_gives_zero_weight_grads():
    # Nothing to reduce: no partial-sum slot and no scratch lookup; the
    # weight/bias gradients of an empty batch are zero, as with cc1d_bwd.
    dt = torch.bfloat16
    x, w, b, dout, init, dfinal = _inputs("chanlast", dt, 0, 64, 32, 4, seed=1)
    o = _outputs(x, w, b, init)
    o["dwdb"].fill_(float("nan"))
    p = _params(x, w, b, dout, init, dfinal, o)
    lib = _lib.load()
    need = ctypes.c_size_t(1)
    assert lib.cc1d_bwd_workspace_size(ctypes.byref(p), ctypes.byref(need)) == _lib.CC1D_OK
    assert need.value == 0
    _lib.check(lib.cc1d_bwd_noalloc(ctypes.byref(p), torch.cuda.current_stream().cuda_stream), "cc1d_bwd_noalloc")
    torch.cuda.synchronize()
    assert torch.count_nonzero(o["dwdb"]) == 0


def test_noalloc_rejects_problems_larger_than_its_scratch():
    # seqlen-contiguous, 128 rows of batch: 128 * 8192 * (4+1) fp32 partial
    # sums = 21 MB > the 16 MiB built-in scratch.
    dt = torch.bfloat16
    B, D, L, W = 128, 8192, 256, 4
    x, w, b, dout, init, dfinal = _inputs("contig", dt, B, D, L, W, seed=3)
    o = _outputs(x, w, b, init)
    p = _params(x, w, b, dout, init, dfinal, o)
    lib = _lib.load()
    need = ctypes.c_size_t(0)
    assert lib.cc1d_bwd_workspace_size(ctypes.byref(p), ctypes.byref(need)) == _lib.CC1D_OK
    assert need.value > 16 * 1024 * 1024
    rc = lib.cc1d_bwd_noalloc(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.CC1D_ERR_WORKSPACE
    assert b"built-in scratch" in lib.cc1d_last_error()
