"""Host-side logic of the multi-GPU sharding (causal_conv1d_b200.parallel)
run as two gloo ranks on CPU: batch sharding, the single all-reduce of the
packed fp32 [dweight | dbias] buffer, and dim sharding without any
collective.  The per-rank compute is the CPU oracle (the kernels need a
GPU); the test checks that sharded results reassemble to the unsharded
ones.  Also covers a rank that fails before the collective: the peer gets
an error from the process-group timeout instead of hanging."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent

from causal_conv1d_b200.parallel import allreduce_weight_grads, dim_shard, shard_range, split_dwdb  # noqa: E402


def test_shard_range_covers_everything():
    for n in (0, 1, 7, 8, 64, 65):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_split_dwdb_layout():
    D, W = 5, 4
    buf = torch.arange(D * (W + 1), dtype=torch.float32)
    dw, db = split_dwdb(buf, D, W)
    assert dw.shape == (D, W) and db.shape == (D,)
    assert torch.equal(dw.flatten(), buf[: D * W]) and torch.equal(db, buf[D * W:])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs():
    g = torch.Generator().manual_seed(0)
    B, D, L, W = 4, 24, 50, 4
    x = torch.randn(B, D, L, generator=g)
    w = torch.rand(D, W, generator=g) - 0.5
    b = torch.rand(D, generator=g) - 0.5
    dout = torch.randn(B, D, L, generator=g)
    return x, w, b, dout


def _worker(rank, world, port, mode, q):
    sys.path[:0] = [str(REPO), str(REPO / "causal-conv1d-mojo_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import oracle
    from causal_conv1d_b200.parallel import allreduce_weight_grads as ar
    from causal_conv1d_b200.parallel import dim_shard as dsh
    from causal_conv1d_b200.parallel import shard_range as sr
    from causal_conv1d_b200.parallel import split_dwdb as sp

    timeout = datetime.timedelta(seconds=5 if mode == "rank_dies" else 60)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timeout)
    try:
        x, w, b, dout = _inputs()
        D, W = w.shape
        if mode == "batch":
            b0, b1 = sr(x.shape[0], rank, world)
            g = oracle.bwd(x[b0:b1].contiguous(), w, dout[b0:b1].contiguous(), b, silu=True)
            dwdb = g["dwdb"].clone()
            ar(dwdb)
            dw, db = sp(dwdb, D, W)
            q.put((rank, "batch", dw.numpy().copy(), db.numpy().copy()))
        elif mode == "dim":
            ws, bs, (d0, d1) = dsh(w, b, rank, world)
            g = oracle.bwd(x[:, d0:d1].contiguous(), ws.contiguous(), dout[:, d0:d1].contiguous(), bs.contiguous(),
                           silu=True)
            q.put((rank, "dim", (d0, d1), g["dweight"].numpy().copy(), g["dx"].numpy().copy()))
        elif mode == "rank_dies":
            if rank == 1:
                raise SystemExit(0)  # leaves before the collective
            try:
                ar(torch.zeros(D * (W + 1)))
                q.put((rank, "no-error"))
            except Exception as e:  # noqa: BLE001
                q.put((rank, "error", type(e).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail(f"rank did not finish ({mode})")
    out = []
    while not q.empty():
        out.append(q.get())
    return out


def test_batch_sharded_backward_allreduce_gloo():
    import oracle

    x, w, b, dout = _inputs()
    full = oracle.bwd(x, w, dout, b, silu=True)
    res = _run("batch")
    assert len(res) == 2
    for _, _, dw, db in res:
        dw, db = torch.from_numpy(dw), torch.from_numpy(db)
        torch.testing.assert_close(dw, full["dweight"], rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(db, full["dbias"], rtol=1e-5, atol=1e-5)


def test_dim_sharded_backward_needs_no_collective_gloo():
    import oracle

    x, w, b, dout = _inputs()
    full = oracle.bwd(x, w, dout, b, silu=True)
    res = sorted(_run("dim"), key=lambda r: r[0])
    dw = torch.cat([torch.from_numpy(r[3]) for r in res], 0)
    dx = torch.cat([torch.from_numpy(r[4]) for r in res], 1)
    assert res[0][2][0] == 0 and res[-1][2][1] == w.shape[0]
    torch.testing.assert_close(dw, full["dweight"], rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(dx, full["dx"], rtol=0, atol=0)


def test_rank_failure_surfaces_as_error_not_hang():
    res = _run("rank_dies")
    assert res, "surviving rank reported nothing"
    rank, status = res[0][0], res[0][1]
    assert rank == 0 and status == "error"


def test_allreduce_is_noop_without_process_group():
    buf = torch.ones(6)
    assert allreduce_weight_grads(buf) is buf
    assert torch.equal(buf, torch.ones(6))
    assert dim_shard(torch.zeros(10, 4), None, 1, 2)[2] == (5, 10)
