"""Sharding of causal_conv1d_fn across GPUs (one process per GPU).

Every (batch, channel) row of the conv is independent, so the work shards
with no data exchange:

* dim sharding  -- rank r owns channels [d0, d1): x, weight, bias and the
  states are sliced along dim.  Forward and backward need no collective.
* batch sharding -- rank r owns batch rows [b0, b1) and the full weights.
  The forward needs nothing; the backward produces partial weight/bias
  gradients, summed with ONE all-reduce of the fp32 buffer
  [dweight (dim, W) | dbias (dim)] that the backward kernel writes.  At the
  Mamba shapes that buffer is ~100-170 KB, so the collective is
  latency-bound.

Two implementations of that all-reduce:

* ``PeerReducer`` (GPUs on one node): the backward's final reduction kernel
  also performs the cross-GPU sum (cc1d_bwd_peer_reduce).  Each rank PUSHES
  its local sums over NVLink into every peer's IPC-mapped exchange buffer
  with plain peer stores, then reads only its OWN buffer (local memory) and
  adds the ranks' values in rank order.  One launch replaces finalize ->
  all-reduce -> dtype casts, and every rank gets bitwise identical
  gradients.  A rank that is late beyond the bounded wait (or gone) makes
  the others write NaN gradients and count the event in the reducer's status
  word, which ``PeerReducer.check()`` turns into an exception.
* ``allreduce_weight_grads``: one ``torch.distributed`` all-reduce of the
  fp32 buffer (NCCL on GPUs; the host logic is exercised with gloo on CPU).

The reference (gabrieldemarmiesse/causal-conv1d-mojo) has no multi-GPU code;
this module is the data-parallel use of its causal_conv1d_fn.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib, _ops
from ._fn import _like_layout


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) of `n` items owned by `rank` of `world`
    (the first n % world ranks get one extra item)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def dim_shard(weight: torch.Tensor, bias: torch.Tensor | None, rank: int, world: int):
    """Channel slice of the parameters owned by `rank` (views, no copy)."""
    d0, d1 = shard_range(weight.shape[0], rank, world)
    return weight[d0:d1], (bias[d0:d1] if bias is not None else None), (d0, d1)


def split_dwdb(dwdb: torch.Tensor, dim: int, width: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Views (dweight (dim, width), dbias (dim,)) of the packed fp32 buffer."""
    if dwdb.numel() != dim * (width + 1) or dwdb.dtype != torch.float32:
        raise ValueError("dwdb must be a float32 buffer of dim*(width+1) elements")
    return dwdb[: dim * width].view(dim, width), dwdb[dim * width:]


def allreduce_weight_grads(dwdb: torch.Tensor, group=None) -> torch.Tensor:
    """Sum the packed fp32 [dweight | dbias] buffer over the ranks of `group`
    (in place, one collective).  No-op when torch.distributed is not
    initialised or the group has a single rank."""
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(dwdb, op=dist.ReduceOp.SUM, group=group)
    return dwdb


def _cuda_device(device) -> torch.device:
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if dev.type != "cuda":
        raise ValueError("PeerReducer needs a CUDA device")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return dev


def _rt_check(res, what: str):
    err = res[0] if isinstance(res, tuple) else res
    if int(err) != 0:
        raise RuntimeError(f"{what} failed: {err}")
    return res[1] if isinstance(res, tuple) and len(res) == 2 else None


class PeerReducer:
    """Peer-mapped exchange buffers for the fused backward reduction over
    `group` (one process per GPU, all GPUs of one node).

    Each rank cudaMallocs one exchange buffer of
    cc1d_peer_exchange_bytes(dim, width, world) bytes (8-byte {call tag,
    value} words, two halves alternating by call parity), exports it as a
    CUDA IPC handle, gathers the peers' handles over `group` and maps them;
    the kernel stores every rank's partial sums straight into every peer's
    buffer.  Plain peer memory -- no multicast object.  Construction and
    ``close()`` are collective over `group`; every rank must then issue the
    same sequence of backward calls with the same dim/width.  The per-block
    call counters live on the device, so those calls may be captured in a
    CUDA graph and replayed.

    Split exchange: ``args(_lib.PEER_PUSH)`` makes the backward push its
    sums and return without waiting, and a later call with
    ``args(_lib.PEER_FINISH)`` and the same tensors -- typically on another
    stream, so that the wait for the slowest rank overlaps the next work --
    waits and writes dweight/dbias.  Each FINISH must be ordered before this
    rank's next PUSH (make the PUSH stream wait on an event recorded after
    FINISH).  A reducer uses either the fused or the split exchange, not
    both (the split calls count on their own 4-word counter tensor).

    Failure detection: every wait for a peer is bounded (`max_polls` polls,
    0 = the library default of about a second or more).  A wait that gives
    up writes NaN into the gradients it could not reduce and adds 1 to this
    reducer's device status word; ``check()`` -- call it at a point where the
    host synchronises anyway, e.g. right before the optimizer step -- raises
    if any call since the previous check gave up.
    """

    def __init__(self, dim: int, width: int, device: torch.device | str | int | None = None, group=None,
                 max_polls: int = 0):
        from cuda.bindings import runtime as rt

        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("PeerReducer needs an initialised torch.distributed process group")
        self._rt = rt
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 32:
            raise ValueError("PeerReducer supports at most 32 ranks")
        dev = _cuda_device(device)
        self.device, self.dim, self.width = dev, dim, width
        self.max_polls = int(max_polls)
        self._collective = True
        lib = _lib.load()
        self.nblocks = int(lib.cc1d_peer_blocks(dim, width))
        nbytes = max(int(lib.cc1d_peer_exchange_bytes(dim, width, self.world)), 16)
        _rt_check(rt.cudaSetDevice(dev.index), "cudaSetDevice")
        self._own = _rt_check(rt.cudaMalloc(nbytes), "cudaMalloc")
        _rt_check(rt.cudaMemset(self._own, 0, nbytes), "cudaMemset")
        _rt_check(rt.cudaDeviceSynchronize(), "cudaDeviceSynchronize")
        handle = bytes(_rt_check(rt.cudaIpcGetMemHandle(self._own), "cudaIpcGetMemHandle").reserved)
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        gathered: list = [None] * self.world
        dist.all_gather_object(gathered, (uuid, handle), group=group)
        if len({g[0] for g in gathered}) != self.world:
            # The reduction kernels of different ranks wait for one another;
            # two of them queued on one GPU are not guaranteed to run together.
            rt.cudaFree(self._own)
            self._own = None
            raise ValueError("PeerReducer needs one GPU per rank (two ranks share a device)")
        self._mapped = []
        ptrs = [0] * self.world
        for r, (_, h_bytes) in enumerate(gathered):
            if r == self.rank:
                ptrs[r] = int(self._own)
                continue
            h = rt.cudaIpcMemHandle_t()
            h.reserved = h_bytes
            mp = _rt_check(rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle")
            self._mapped.append(mp)
            ptrs[r] = int(mp)
        self.exchange_ptrs = torch.tensor(ptrs, dtype=torch.int64, device=dev)
        self.epochs = torch.zeros(max(self.nblocks, 1), dtype=torch.int32, device=dev)
        self.split_epochs = torch.zeros(4, dtype=torch.int32, device=dev)
        self._mode = None
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    @classmethod
    def from_exchange(cls, exchange_ptrs: torch.Tensor, rank: int, dim: int, width: int, max_polls: int = 0):
        """A reducer over exchange buffers the caller mapped itself (its own
        IPC layer, or one process owning several buffers): `exchange_ptrs`
        is an int64 device tensor of the `world` buffer addresses, each
        cc1d_peer_exchange_bytes(dim, width, world) bytes and zeroed.  No
        collective is made and ``close()`` frees nothing; the caller keeps
        the buffers alive while the reducer is used."""
        if exchange_ptrs.dtype != torch.int64 or exchange_ptrs.dim() != 1 or not exchange_ptrs.is_cuda:
            raise ValueError("exchange_ptrs must be a 1-D int64 CUDA tensor")
        world = exchange_ptrs.numel()
        if not 1 <= world <= 32 or not 0 <= rank < world:
            raise ValueError(f"bad rank {rank} for world size {world} (at most 32)")
        self = cls.__new__(cls)
        self._rt = None
        self.group = None
        self.rank, self.world = int(rank), int(world)
        self.device = exchange_ptrs.device
        self.dim, self.width = dim, width
        self.max_polls = int(max_polls)
        self._collective = False
        self.nblocks = int(_lib.load().cc1d_peer_blocks(dim, width))
        self._own = 0
        self._mapped = []
        self.exchange_ptrs = exchange_ptrs
        self.epochs = torch.zeros(max(self.nblocks, 1), dtype=torch.int32, device=self.device)
        self.split_epochs = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._mode = None
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        return self

    def args(self, flags: int = _lib.PEER_FUSED) -> tuple[torch.Tensor, torch.Tensor, int, int, int, torch.Tensor,
                                                           int]:
        """(exchange_ptrs, epochs, rank, world, max_polls, status, flags) for
        ``_ops.bwd_peer``: the fused exchange (default), or one half of the
        split exchange (_lib.PEER_PUSH / _lib.PEER_FINISH)."""
        if self._own is None:
            raise RuntimeError("PeerReducer is closed")
        if flags not in (_lib.PEER_FUSED, _lib.PEER_PUSH, _lib.PEER_FINISH):
            raise ValueError(f"unknown peer-exchange flags {flags}")
        mode = "fused" if flags == _lib.PEER_FUSED else "split"
        if self._mode is None:
            self._mode = mode
        elif self._mode != mode:
            raise RuntimeError(f"PeerReducer already used for the {self._mode} exchange; the fused and the split "
                               f"exchange cannot share one reducer")
        epochs = self.epochs if mode == "fused" else self.split_epochs
        return self.exchange_ptrs, epochs, self.rank, self.world, self.max_polls, self.status, int(flags)

    def failed_waits(self) -> int:
        """Waits for a peer that gave up since the last ``check()`` (reads
        the device word: synchronises with this device's queued work)."""
        return int(self.status.item())

    def check(self) -> None:
        """Raise if a backward call through this reducer gave up waiting for
        a peer since the previous check (its weight/bias gradients then hold
        NaN where the cross-rank sum could not be formed).  Synchronises with
        this device; resets the status word."""
        n = self.failed_waits()
        if n:
            self.status.zero_()
            raise RuntimeError(
                f"PeerReducer (rank {self.rank} of {self.world}): {n} wait(s) for a peer's partial sums gave "
                f"up (a rank late by more than the bounded wait, or gone); the weight/bias gradients of the "
                f"affected call(s) are NaN")

    def close(self) -> None:
        """Collective: unmap the peers' buffers, then free this rank's."""
        if self._own is None:
            return
        if not self._collective:
            self._own = None
            return
        rt = self._rt
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no rank still reads or signals
        _rt_check(rt.cudaSetDevice(self.device.index), "cudaSetDevice")
        for mp in self._mapped:
            _rt_check(rt.cudaIpcCloseMemHandle(mp), "cudaIpcCloseMemHandle")
        self._mapped = []
        dist.barrier(group=self.group)  # every peer has unmapped this rank's buffer
        _rt_check(rt.cudaFree(self._own), "cudaFree")
        self._own = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False


class _BatchShardedFn(torch.autograd.Function):
    """causal_conv1d_fn over a batch shard; backward sums dW/db over ranks
    (fused peer reduction when a PeerReducer is given, else all-reduce)."""

    @staticmethod
    def forward(ctx, x, weight, bias, initial_states, apply_silu, final_states_out, group, reducer):
        out = torch.empty_like(x)
        _ops.fwd(x, weight, bias, None, initial_states, out, apply_silu, final_states_out)
        ctx.save_for_backward(x, weight, bias, initial_states)
        ctx.apply_silu = apply_silu
        ctx.group = group
        ctx.reducer = reducer
        ctx.return_final_states = final_states_out is not None
        if final_states_out is not None:
            return out, final_states_out
        return out

    @staticmethod
    def backward(ctx, *grads):
        dout = grads[0]
        dfinal = grads[1] if ctx.return_final_states else None
        x, weight, bias, initial_states = ctx.saved_tensors
        D, W = weight.shape
        dout = _like_layout(dout, x)
        dx = torch.empty_like(x)
        dwdb = torch.empty(D * (W + 1), dtype=torch.float32, device=x.device)
        dinit = torch.empty_like(initial_states) if initial_states is not None else None
        if ctx.reducer is not None:
            if (ctx.reducer.dim, ctx.reducer.width) != (D, W):
                raise ValueError("PeerReducer was built for another (dim, width)")
            dw = torch.empty(D, W, dtype=weight.dtype, device=x.device)
            db = torch.empty(D, dtype=bias.dtype, device=x.device) if bias is not None else None
            _ops.bwd_peer(x, weight, bias, dout, initial_states, dfinal, dx, dwdb, dinit, dw, db, ctx.apply_silu,
                          *ctx.reducer.args())
            return dx, dw, db, dinit, None, None, None, None
        _ops.bwd(x, weight, bias, dout, None, initial_states, dfinal, dx, dwdb, dinit, None, None, ctx.apply_silu)
        allreduce_weight_grads(dwdb, ctx.group)
        dw, db = split_dwdb(dwdb, D, W)
        return (dx, dw.to(weight.dtype), db.to(bias.dtype) if bias is not None else None, dinit, None, None, None,
                None)


def causal_conv1d_fn_batch_sharded(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    initial_states: torch.Tensor | None = None,
    return_final_states: bool = False,
    activation: str | None = None,
    group=None,
    reducer: PeerReducer | None = None,
):
    """causal_conv1d_fn on this rank's batch shard `x` with replicated
    weight/bias: weight.grad / bias.grad come out summed over all ranks of
    `group` (the data-parallel gradient), x.grad stays local.  With a
    `reducer` the sum is fused into the backward kernel over NVLink peer
    memory (call ``reducer.check()`` before using the gradients, e.g. before
    the optimizer step, to turn a peer that never arrived into an error);
    otherwise one all-reduce over `group`."""
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("only activation in {None, 'silu', 'swish'} is supported")
    batch, dim, _ = x.shape
    width = weight.shape[1]
    fs = torch.empty(batch, dim, width - 1, dtype=x.dtype, device=x.device) if return_final_states else None
    return _BatchShardedFn.apply(x, weight, bias, initial_states, activation in ("silu", "swish"), fs, group, reducer)
