"""Batch-sharded backward on several GPUs, one process per GPU over NCCL:
the dweight/dbias reduction fused with the cross-GPU sum over NVLink peer
memory (cc1d_bwd_peer_reduce through parallel.PeerReducer).

Checked on every rank, for every call of a sequence (so both halves of the
double-buffered exchange and stale-data hazards are exercised), eagerly and
replayed from a CUDA graph:

* fp32 [dweight | dbias] is bitwise equal to the rank-order sum of the
  per-rank cc1d_bwd results (gathered with NCCL),
* the parameter-dtype dweight / dbias are that sum rounded once,
* dx / dinitial_states equal the single-GPU kernel's bitwise,
* the autograd path (causal_conv1d_fn_batch_sharded with a reducer) matches
  the unsharded causal_conv1d_fn within the dtype tolerance,
* no bounded wait gave up.

The multi-rank tests need two or more GPUs (one rank per GPU; two ranks on
one GPU are refused by PeerReducer) and are skipped otherwise; the bounded
wait of the exchange is tested on one GPU."""

from __future__ import annotations

import datetime
import os
import socket
import sys
import traceback
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent

pytestmark = pytest.mark.gpu

WORLD = min(torch.cuda.device_count(), 8) if torch.cuda.is_available() else 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case_inputs(dtype, B, D, L, W, seed, has_bias, chanlast):
    g = torch.Generator("cpu").manual_seed(seed)

    def lay(t):
        return t.transpose(1, 2).contiguous().transpose(1, 2) if chanlast else t.contiguous()

    x = lay(torch.randn(B, D, L, generator=g).to(dtype))
    w = (torch.rand(D, W, generator=g) - 0.5).to(dtype)
    b = (torch.rand(D, generator=g) - 0.5).to(dtype) if has_bias else None
    init = torch.randn(B, D, W - 1, generator=g).to(dtype)
    douts = [lay(torch.randn(B, D, L, generator=g).to(dtype)) for _ in range(4)]
    return x, w, b, init, douts


CASES = [
    # dtype, rows per rank, D, L, W, bias, channel-last
    (torch.bfloat16, 2, 512, 256, 4, True, True),
    (torch.float32, 1, 200, 77, 3, False, False),
    (torch.float16, 3, 96, 128, 2, True, True),
]


def _run_case(case, rank, world, dev):
    import torch.distributed as dist

    from causal_conv1d_b200 import _lib, _ops, causal_conv1d_fn
    from causal_conv1d_b200.parallel import PeerReducer, causal_conv1d_fn_batch_sharded, shard_range

    dtype, per, D, L, W, has_bias, chanlast = case
    B = per * world
    x, w, b, init, douts = _case_inputs(dtype, B, D, L, W, 17 + D, has_bias, chanlast)
    b0, b1 = shard_range(B, rank, world)
    to = dict(device=dev)
    xs, ws = x[b0:b1].to(**to), w.to(**to)
    bs = b.to(**to) if b is not None else None
    inits = init[b0:b1].to(**to)
    douts_s = [d[b0:b1].to(**to) for d in douts]

    def local(dout):
        dx = torch.empty_like(xs)
        dwdb = torch.empty(D * (W + 1), dtype=torch.float32, **to)
        dinit = torch.empty_like(inits)
        _ops.bwd(xs, ws, bs, dout, None, inits, None, dx, dwdb, dinit, None, None, True)
        parts = [torch.empty_like(dwdb) for _ in range(world)]
        dist.all_gather(parts, dwdb)
        total = torch.zeros_like(dwdb)
        for p in parts:
            total = total + p
        return dx, dinit, total

    reducer = PeerReducer(D, W, dev)
    try:
        dx = torch.empty_like(xs)
        dwdb = torch.empty(D * (W + 1), dtype=torch.float32, **to)
        dinit = torch.empty_like(inits)
        dw = torch.empty(D, W, dtype=dtype, **to)
        db = torch.empty(D, dtype=dtype, **to) if has_bias else None
        static_dout = torch.empty_like(douts_s[0])

        def peer():
            _ops.bwd_peer(xs, ws, bs, static_dout, inits, None, dx, dwdb, dinit, dw, db, True, *reducer.args())

        def check(i, how):
            ref_dx, ref_dinit, total = local(douts_s[i])
            tag = f"{how} call {i} rank {rank}"
            assert torch.equal(dwdb, total), tag
            assert torch.equal(dw, total[: D * W].view(D, W).to(dtype)), tag
            if has_bias:
                assert torch.equal(db, total[D * W:].to(dtype)), tag
            else:
                assert torch.count_nonzero(dwdb[D * W:]) == 0, tag
            assert torch.equal(dx, ref_dx), tag
            assert torch.equal(dinit, ref_dinit), tag

        # Eager: four calls in a row with different gradients.
        for i in range(4):
            static_dout.copy_(douts_s[i])
            peer()
            check(i, "eager")
        # Replayed from a CUDA graph: the call counters advance on the device.
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            peer()
        for i in (1, 3, 0, 2, 2):
            static_dout.copy_(douts_s[i])
            g.replay()
            check(i, "graph")
        del g

        # Autograd through the public batch-sharded function vs unsharded.
        xa = xs.clone().requires_grad_()
        wa = ws.clone().requires_grad_()
        ba = bs.clone().requires_grad_() if bs is not None else None
        out = causal_conv1d_fn_batch_sharded(xa, wa, ba, activation="silu", reducer=reducer)
        out.backward(douts_s[0])
        xf = x.to(**to).requires_grad_()
        wf = w.to(**to).requires_grad_()
        bf = b.to(**to).requires_grad_() if b is not None else None
        outf = causal_conv1d_fn(xf, wf, bf, activation="silu")
        outf.backward(douts[0].to(**to))
        tol = dict(rtol=1e-5, atol=1e-5) if dtype == torch.float32 else dict(rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(out, outf[b0:b1].detach(), **tol)
        torch.testing.assert_close(xa.grad, xf.grad[b0:b1], **tol)
        # dweight sums B*L products: compare against the fp32 reduction.
        torch.testing.assert_close(wa.grad.float(), wf.grad.float(), rtol=tol["rtol"], atol=tol["atol"] * 10)
        if ba is not None:
            torch.testing.assert_close(ba.grad.float(), bf.grad.float(), rtol=tol["rtol"], atol=tol["atol"] * 10)
        torch.cuda.synchronize(dev)
        reducer.check()  # no wait for a peer gave up
        assert _lib.device_wait_timeouts() == 0
    finally:
        reducer.close()

    # Split exchange: the backward pushes, a FINISH on a side stream waits
    # and writes dweight/dbias; each FINISH is ordered before the next PUSH.
    split = PeerReducer(D, W, dev)
    try:
        side = torch.cuda.Stream(dev)
        dx = torch.empty_like(xs)
        dwdb = torch.empty(D * (W + 1), dtype=torch.float32, **to)
        dinit = torch.empty_like(inits)
        dw = torch.empty(D, W, dtype=dtype, **to)
        db = torch.empty(D, dtype=dtype, **to) if has_bias else None
        static_dout = torch.empty_like(douts_s[0])

        def split_call():
            main = torch.cuda.current_stream(dev)
            _ops.bwd_peer(xs, ws, bs, static_dout, inits, None, dx, dwdb, dinit, dw, db, True,
                          *split.args(_lib.PEER_PUSH))
            pushed = torch.cuda.Event()
            pushed.record(main)
            with torch.cuda.stream(side):
                side.wait_event(pushed)
                _ops.bwd_peer(xs, ws, bs, static_dout, inits, None, dx, dwdb, dinit, dw, db, True,
                              *split.args(_lib.PEER_FINISH))
                done = torch.cuda.Event()
                done.record(side)
            main.wait_event(done)

        def check_split(i, how):
            ref_dx, ref_dinit, total = local(douts_s[i])
            tag = f"split {how} call {i} rank {rank}"
            assert torch.equal(dwdb, total), tag
            assert torch.equal(dw, total[: D * W].view(D, W).to(dtype)), tag
            if has_bias:
                assert torch.equal(db, total[D * W:].to(dtype)), tag
            assert torch.equal(dx, ref_dx), tag
            assert torch.equal(dinit, ref_dinit), tag

        for i in range(4):
            static_dout.copy_(douts_s[i])
            split_call()
            torch.cuda.synchronize(dev)
            check_split(i, "eager")
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            split_call()
        for i in (2, 0, 3, 1):
            static_dout.copy_(douts_s[i])
            g.replay()
            torch.cuda.synchronize(dev)
            check_split(i, "graph")
        del g
        with pytest.raises(RuntimeError, match="cannot share one reducer"):
            split.args()
        split.check()
        assert _lib.device_wait_timeouts() == 0
    finally:
        split.close()


def _run_dim_shard(rank, world, dev):
    """Dim sharding ('sharded over dim'): rank r runs
    causal_conv1d_fn on its channel slice -- a view of the channel-last
    (Mamba-layout) activations with the matching weight / bias / state
    slices -- with no collective at all.  The slices are gathered afterwards
    only to check them: out, final_states, dx and dinitial_states must equal
    the unsharded single-GPU result bitwise (rows (b, c) are independent and
    every kernel evaluates a row with the same arithmetic), dweight / dbias
    within the fp32 reduction tolerance (the partial-sum split depends on the
    number of channels).  Channel slices as the reference's
    tests/test_noncontig_layouts.py:28-43."""
    import torch.distributed as dist

    from causal_conv1d_b200 import causal_conv1d_fn
    from causal_conv1d_b200.parallel import dim_shard

    dtype, B, D, L, W = torch.bfloat16, 2, 1024, 512, 4
    x, w, b, init, douts = _case_inputs(dtype, B, D, L, W, 77, True, True)
    ws, bs, (d0, d1) = dim_shard(w, b, rank, world)
    # Every rank holds the full activations in this test; its shard is a
    # channel-slice VIEW (no copy), as a model that shards channels would pass.
    xf, dof = x.to(dev), douts[0].to(dev)
    xs = xf[:, d0:d1].detach().requires_grad_()
    wsd = ws.to(dev).requires_grad_()
    bsd = bs.to(dev).requires_grad_()
    isd = init[:, d0:d1].to(dev).requires_grad_()
    out, fs = causal_conv1d_fn(xs, wsd, bsd, initial_states=isd, return_final_states=True, activation="silu")
    out.backward(dof[:, d0:d1])
    torch.cuda.synchronize(dev)
    # Reference: the unsharded problem on this GPU.
    xa = xf.detach().requires_grad_()
    wa = w.to(dev).requires_grad_()
    ba = b.to(dev).requires_grad_()
    ia = init.to(dev).requires_grad_()
    outa, fsa = causal_conv1d_fn(xa, wa, ba, initial_states=ia, return_final_states=True, activation="silu")
    outa.backward(dof)
    torch.cuda.synchronize(dev)
    tag = f"dim shard rank {rank} channels [{d0}, {d1})"
    assert torch.equal(out, outa[:, d0:d1]), tag + " out"
    assert torch.equal(fs, fsa[:, d0:d1]), tag + " final_states"
    assert torch.equal(xs.grad, xa.grad[:, d0:d1]), tag + " dx"
    assert torch.equal(isd.grad, ia.grad[:, d0:d1]), tag + " dinitial_states"
    torch.testing.assert_close(wsd.grad.float(), wa.grad[d0:d1].float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(bsd.grad.float(), ba.grad[d0:d1].float(), rtol=1e-2, atol=1e-2)
    # The shards tile the channels: gathered slice bounds cover [0, D).
    bounds = [None] * world
    dist.all_gather_object(bounds, (d0, d1))
    assert bounds[0][0] == 0 and bounds[-1][1] == D
    assert all(bounds[r][1] == bounds[r + 1][0] for r in range(world - 1))


def _worker(rank, world, port, q):
    sys.path[:0] = [str(REPO), str(REPO / "causal-conv1d-mojo_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    case = None
    try:
        for case in CASES:
            _run_case(case, rank, world, dev)
        case = "dim shard"
        _run_dim_shard(rank, world, dev)
        q.put((rank, "ok", ""))
    except Exception:  # reported to the parent
        q.put((rank, "fail", f"case {case}\n" + traceback.format_exc()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(WORLD < 2, reason="needs two or more GPUs")
def test_peer_reduce_and_dim_shard_match_single_gpu():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(WORLD):
            rank, status, msg = q.get(timeout=600)
            results[rank] = (status, msg)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    bad = [f"rank {r}:\n{m}" for r, (s, m) in sorted(results.items()) if s != "ok"]
    if bad:
        pytest.fail("\n".join(bad), pytrace=False)
    assert len(results) == WORLD


@pytest.mark.skipif(WORLD < 2, reason="needs two or more GPUs")
def test_one_process_several_devices():
    """One process driving every GPU in turn (highest index first), forward
    and autograd backward: per-device kernel attributes and the device the
    library launches on follow the data, whichever device the calling thread
    was bound to.  All devices give bitwise identical results."""
    from causal_conv1d_b200 import causal_conv1d_fn

    B, D, L, W = 2, 512, 256, 4
    x, w, b, init, douts = _case_inputs(torch.bfloat16, B, D, L, W, 5, True, True)
    results = []
    torch.cuda.set_device(0)
    for d in reversed(range(WORLD)):
        dev = torch.device("cuda", d)
        xd = x.to(dev).requires_grad_()
        wd = w.to(dev).requires_grad_()
        bd = b.to(dev).requires_grad_()
        out = causal_conv1d_fn(xd, wd, bd, activation="silu")
        out.backward(douts[0].to(dev))
        torch.cuda.synchronize(dev)
        results.append([t.cpu() for t in (out, xd.grad, wd.grad, bd.grad)])
    for other in results[1:]:
        for a, c in zip(results[0], other):
            assert torch.equal(a, c)


def test_peer_wait_gives_up_and_reports():
    """Failure detection of the fused reduction on one GPU, with no fault: a
    'peer' buffer that nobody pushes into, so every bounded wait runs out
    after max_polls.  The outputs stay unwritten, the call counters still
    advance, the host reads the count from cc1d_device_status, and the
    context stays usable (a following single-rank call matches the local
    backward bitwise)."""
    from causal_conv1d_b200 import _lib, _ops

    dev = torch.device("cuda", 0)
    B, D, L, W = 2, 256, 64, 4
    x, w, b, init, douts = _case_inputs(torch.bfloat16, B, D, L, W, 11, True, True)
    x, w, b, init, dout = x.to(dev), w.to(dev), b.to(dev), init.to(dev), douts[0].to(dev)
    lib = _lib.load()
    nblocks = int(lib.cc1d_peer_blocks(D, W))
    _lib.device_wait_timeouts()  # reset the counter
    own = torch.zeros(int(lib.cc1d_peer_exchange_bytes(D, W, 2)) // 8, dtype=torch.int64, device=dev)
    silent = torch.zeros_like(own)
    ptrs = torch.tensor([own.data_ptr(), silent.data_ptr()], dtype=torch.int64, device=dev)
    epochs = torch.zeros(nblocks, dtype=torch.int32, device=dev)
    dx = torch.empty_like(x)
    dinit = torch.empty_like(init)
    dwdb = torch.full((D * (W + 1),), float("nan"), device=dev)
    dw = torch.full((D, W), float("nan"), dtype=torch.bfloat16, device=dev)
    db = torch.full((D,), float("nan"), dtype=torch.bfloat16, device=dev)
    _ops.bwd_peer(x, w, b, dout, init, None, dx, dwdb, dinit, dw, db, True, ptrs, epochs, 0, 2, 1024, None, 0)
    torch.cuda.synchronize(dev)
    assert _lib.device_wait_timeouts() > 0
    assert torch.isnan(dwdb).all() and torch.isnan(dw).all() and torch.isnan(db).all()
    assert torch.equal(epochs.cpu(), torch.ones(nblocks, dtype=torch.int32))
    # dx does not depend on the exchange: it is complete.
    ref_dx, ref_dwdb = torch.empty_like(x), torch.empty(D * (W + 1), device=dev)
    ref_dinit = torch.empty_like(init)
    _ops.bwd(x, w, b, dout, None, init, None, ref_dx, ref_dwdb, ref_dinit, None, None, True)
    assert torch.equal(dx, ref_dx) and torch.equal(dinit, ref_dinit)
    # The context is intact: a world of one reduces to the local result.
    one = torch.zeros_like(own)
    _ops.bwd_peer(x, w, b, dout, init, None, dx, dwdb, dinit, dw, db, True,
                  torch.tensor([one.data_ptr()], dtype=torch.int64, device=dev),
                  torch.zeros(nblocks, dtype=torch.int32, device=dev), 0, 1, 0, None, 0)
    torch.cuda.synchronize(dev)
    assert _lib.device_wait_timeouts() == 0
    assert torch.equal(dwdb, ref_dwdb)
    assert torch.equal(dw, ref_dwdb[: D * W].view(D, W).to(torch.bfloat16))


def test_batch_sharded_autograd_raises_when_a_peer_never_arrives():
    """The autograd path with a reducer whose second 'rank' never pushes (a
    buffer nobody writes, one GPU, no fault): the bounded waits give up, the
    weight/bias gradients come out NaN (never stale memory), the reducer's
    status word counts the failure and check() raises; after that the
    status is clear again."""
    from causal_conv1d_b200 import _lib
    from causal_conv1d_b200.parallel import PeerReducer, causal_conv1d_fn_batch_sharded

    dev = torch.device("cuda", 0)
    B, D, L, W = 2, 256, 64, 4
    x, w, b, init, douts = _case_inputs(torch.bfloat16, B, D, L, W, 13, True, True)
    lib = _lib.load()
    n_words = int(lib.cc1d_peer_exchange_bytes(D, W, 2)) // 8
    own = torch.zeros(n_words, dtype=torch.int64, device=dev)
    silent = torch.zeros_like(own)
    ptrs = torch.tensor([own.data_ptr(), silent.data_ptr()], dtype=torch.int64, device=dev)
    reducer = PeerReducer.from_exchange(ptrs, rank=0, dim=D, width=W, max_polls=1024)
    _lib.device_wait_timeouts(dev)  # reset the process-wide count
    xa = x.to(dev).requires_grad_()
    wa = w.to(dev).requires_grad_()
    ba = b.to(dev).requires_grad_()
    out = causal_conv1d_fn_batch_sharded(xa, wa, ba, activation="silu", reducer=reducer)
    out.backward(douts[0].to(dev))
    torch.cuda.synchronize(dev)
    assert torch.isnan(wa.grad).all() and torch.isnan(ba.grad).all()
    assert torch.isfinite(xa.grad).all()  # dx does not depend on the exchange
    assert reducer.failed_waits() > 0
    with pytest.raises(RuntimeError, match="gave up"):
        reducer.check()
    reducer.check()  # the status word was reset by the failed check
    assert _lib.device_wait_timeouts(dev) > 0
    reducer.close()


def test_split_exchange_single_rank_and_bounded_finish():
    """The split exchange on one GPU: with a world of one, PUSH then FINISH
    (any streams, in order) gives the local reduction bitwise and writes
    nothing before FINISH; with a 'peer' that never pushes, the FINISH wait
    gives up after max_polls, writes NaN, counts the failure in the status
    word and in cc1d_device_status, and the context stays usable."""
    from causal_conv1d_b200 import _lib, _ops

    dev = torch.device("cuda", 0)
    B, D, L, W = 2, 320, 96, 4
    x, w, b, init, douts = _case_inputs(torch.bfloat16, B, D, L, W, 23, True, True)
    x, w, b, init, dout = x.to(dev), w.to(dev), b.to(dev), init.to(dev), douts[0].to(dev)
    lib = _lib.load()
    nbytes = int(lib.cc1d_peer_exchange_bytes(D, W, 2))
    ref_dx, ref_dwdb, ref_dinit = torch.empty_like(x), torch.empty(D * (W + 1), device=dev), torch.empty_like(init)
    _ops.bwd(x, w, b, dout, None, init, None, ref_dx, ref_dwdb, ref_dinit, None, None, True)
    # World of one.
    one = torch.zeros(nbytes // 8, dtype=torch.int64, device=dev)
    ptrs = torch.tensor([one.data_ptr()], dtype=torch.int64, device=dev)
    ctr = torch.zeros(4, dtype=torch.int32, device=dev)
    dx, dinit = torch.empty_like(x), torch.empty_like(init)
    dwdb = torch.full((D * (W + 1),), 7.0, device=dev)
    dw = torch.full((D, W), 7.0, dtype=torch.bfloat16, device=dev)
    db = torch.full((D,), 7.0, dtype=torch.bfloat16, device=dev)
    for call in range(3):
        _ops.bwd_peer(x, w, b, dout, init, None, dx, dwdb, dinit, dw, db, True, ptrs, ctr, 0, 1, 0, None,
                      _lib.PEER_PUSH)
        torch.cuda.synchronize(dev)
        if call == 0:
            assert torch.all(dwdb == 7.0)  # PUSH writes no output
        side = torch.cuda.Stream(dev)
        with torch.cuda.stream(side):
            _ops.bwd_peer(x, w, b, dout, init, None, dx, dwdb, dinit, dw, db, True, ptrs, ctr, 0, 1, 0, None,
                          _lib.PEER_FINISH)
        torch.cuda.synchronize(dev)
        assert torch.equal(dwdb, ref_dwdb)
        assert torch.equal(dw, ref_dwdb[: D * W].view(D, W).to(torch.bfloat16))
        assert torch.equal(db, ref_dwdb[D * W:].to(torch.bfloat16))
        assert torch.equal(dx, ref_dx) and torch.equal(dinit, ref_dinit)
    assert ctr[0].item() == 3 and ctr[2].item() == 3 and ctr[1].item() == 0 and ctr[3].item() == 0
    assert _lib.device_wait_timeouts() == 0
    # A world of two whose second rank never pushes.
    own = torch.zeros(nbytes // 8, dtype=torch.int64, device=dev)
    silent = torch.zeros_like(own)
    ptrs2 = torch.tensor([own.data_ptr(), silent.data_ptr()], dtype=torch.int64, device=dev)
    ctr2 = torch.zeros(4, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _ops.bwd_peer(x, w, b, dout, init, None, dx, dwdb, dinit, dw, db, True, ptrs2, ctr2, 0, 2, 1024, status,
                  _lib.PEER_PUSH)
    _ops.bwd_peer(x, w, b, dout, init, None, dx, dwdb, dinit, dw, db, True, ptrs2, ctr2, 0, 2, 1024, status,
                  _lib.PEER_FINISH)
    torch.cuda.synchronize(dev)
    assert status.item() > 0
    assert _lib.device_wait_timeouts() > 0
    assert torch.isnan(dwdb).all() and torch.isnan(dw).all() and torch.isnan(db).all()
    assert ctr2[0].item() == 1 and ctr2[2].item() == 1
    # Still usable.
    _ops.bwd(x, w, b, dout, None, init, None, dx, dwdb, dinit, None, None, True)
    torch.cuda.synchronize(dev)
    assert torch.equal(dwdb, ref_dwdb)
