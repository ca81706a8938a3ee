"""Benchmark of the causal conv1d hot path on B200 (one JSON line).

Headline workload ("C2"): Mamba-2 2.7B-style
prefill, causal_conv1d_fn forward + backward, bf16, x (8, 5376, 2048) in
channel-last strides, width 4, bias, SiLU, initial_states and
return_final_states, grad_out ~ N(0,1).  One step = forward + backward of
one batch; with N GPUs every rank runs its own batch of 8 (global batch 8N,
weak scaling) and the fp32 [dweight | dbias] partials are summed across the
ranks inside the backward's reduction kernel (NVLink peer memory).

  value  -- whole-job tokens/s on device-resident inputs (CUDA events, max
            over ranks); inputs (176 MB per tensor) are larger than L2.
  e2e    -- the same step through the public API from pinned HOST buffers:
            host->device copies of the step's inputs and device->host reads
            of all its outputs inside the timed region, issued as a serving
            or training loop would: copy-in, compute and copy-out on three
            streams, device inputs double-buffered, so step i+1's upload
            overlaps step i's compute and download.
  roofline / kernels -- algorithmic HBM bytes / CUDA-event kernel time per
            op (fwd, bwd, decode update C3a/C3b, varlen C4, large C5) against
            the measured copy bandwidth of MEASURED_PEAKS.json.
  cpu_baseline -- the reference's CPU algorithm (C restatement in oracle/,
            all host threads) on a bounded sample of the same workload.

`--impl reference` times that CPU path alone as the reference arm.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path[:0] = [str(REPO / "causal-conv1d-mojo_b200"), str(REPO)]

import torch  # noqa: E402

METRIC = "fwd/bwd/update HBM GB/s vs B200 peak; tokens/s at 1/2/4/8 B200"
UNIT = "tokens/s"
B, D, L, W = 8, 5376, 2048, 4
DT = torch.bfloat16
ESZ = 2

FALLBACK_HBM_GBS = 6650.0


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def c2_bytes():
    n = B * D * L
    states = B * D * (W - 1) * ESZ
    wb = D * (W + 1) * ESZ
    fwd = 2 * n * ESZ + 2 * states + wb  # x, out, init, final, w/b
    bwd = 3 * n * ESZ + 2 * states + wb + D * (W + 1) * 4 + wb  # x, dout, dx, init, dinit, w/b, fp32 dw|db, dtype dw|db
    return fwd, bwd


# --------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# --------------------------------------------------------------------------

class Clocks:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.proc = None
        self.window = [None, None]

    def mark(self):
        """Start of the timed region (samples before it are dropped)."""
        time.sleep(0.3)  # let nvidia-smi come up
        self.window[0] = len(self.samples)

    def unmark(self):
        time.sleep(0.15)
        self.window[1] = len(self.samples)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        if self.window[0] is not None:
            lo = self.window[0]
            hi = self.window[1] if self.window[1] is not None else len(self.samples)
            self.samples = self.samples[lo:max(hi, lo + 1)]
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = sorted(float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit())
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i] == "Active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# --------------------------------------------------------------------------
# distributed plumbing
# --------------------------------------------------------------------------

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world, local):
    import datetime

    import torch.distributed as dist

    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return dist


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier_sync(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def device_rendezvous(world):
    """Align the ranks ON THE DEVICE right before a start event: a one-word
    all-reduce on the current stream completes at nearly the same moment on
    every GPU, whereas host processes leave a barrier up to ~100 us apart.
    Without it, the first cross-rank exchange of a short timed region is
    charged with that host skew on the ranks that started first."""
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(torch.zeros(1, device="cuda"))


def gather_floats(vals, world):
    """Every rank's list of floats (same length on all ranks), rank order."""
    if world == 1:
        return [list(vals)]
    import torch.distributed as dist

    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    return [p.tolist() for p in parts]


# --------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------

def make_c2(seed, device):
    g = torch.Generator(device=device).manual_seed(seed)

    def nrm(*s):
        return torch.randn(*s, generator=g, device=device, dtype=torch.float32).to(DT)

    def uni(*s):
        return (torch.rand(*s, generator=g, device=device, dtype=torch.float32) - 0.5).to(DT)

    x = nrm(B, L, D).transpose(1, 2)
    w = uni(D, W)
    b = uni(D)
    init = nrm(B, D, W - 1)
    dout = nrm(B, L, D).transpose(1, 2)
    return x, w, b, init, dout


def graph_of(fn, n=1):
    """CUDA graph of `n` calls fn(i) (captured after the caller's warm-up)."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(n):
            fn(i)
    return g


def graph_ms(g, reps, per_graph):
    """Average CUDA-event time of one of the `per_graph` launches in `g`."""
    g.replay()
    torch.cuda.synchronize()
    a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    c.record()
    torch.cuda.synchronize()
    return a.elapsed_time(c) / (reps * per_graph)


def time_c2(args, world, rank, reducer, split=None):
    """The headline step: C2 forward + backward.  With N GPUs each rank's
    backward sums dweight/dbias over the ranks through NVLink peer memory.
    The K timed steps run twice at N > 1: with the fused exchange
    (`reducer`: the reduction kernel pushes, waits for the peers and writes
    the sums) and with the split exchange (`split`: the backward pushes, and
    the wait plus the output writes run after the next step's forward, when
    the peers' sums have had the whole forward to arrive -- the pattern of a
    training loop that reads the gradients only at the optimizer step; every
    step still does one PUSH and one FINISH).  Each is timed as max over
    ranks; the faster is the job's step and both are reported."""
    from causal_conv1d_b200 import _lib, _ops

    x, w, b, init, dout = make_c2(1234 + rank, "cuda")
    out = torch.empty_like(x)
    fs = torch.empty(B, D, W - 1, dtype=DT, device="cuda")
    dx = torch.empty_like(x)
    dwdb = torch.empty(D * (W + 1), dtype=torch.float32, device="cuda")
    dw = torch.empty(D, W, dtype=DT, device="cuda")
    db = torch.empty(D, dtype=DT, device="cuda")
    dinit = torch.empty_like(init)
    K = args.steps

    def fwd(_=0):
        _ops.fwd(x, w, b, None, init, out, True, fs)

    def bwd(_=0):
        if reducer is not None:
            # dweight/dbias summed over the ranks inside the reduction kernel
            # (NVLink peer memory), written straight into dw / db.
            _ops.bwd_peer(x, w, b, dout, init, None, dx, dwdb, dinit, dw, db, True, *reducer.args())
        else:
            _ops.bwd(x, w, b, dout, None, init, None, dx, dwdb, dinit, dw, db, True)

    def step(_=0):
        fwd()
        bwd()

    def timed(step_fn):
        """Warm-up, then EXACTLY K steps replayed from a CUDA graph (captured
        once, as a serving / training loop would), between a device-side
        rendezvous and a synchronize; this rank's milliseconds."""
        for _ in range(args.warmup):
            step_fn()
        torch.cuda.synchronize()
        g_step = graph_of(step_fn)
        for _ in range(args.warmup):
            g_step.replay()
        barrier_sync(world)
        device_rendezvous(world)
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(K):
            g_step.replay()
        stop.record()
        torch.cuda.synchronize()
        barrier_sync(world)
        del g_step
        return start.elapsed_time(stop)

    exchange = {}
    with Clocks(torch.cuda.current_device()) as clk:
        # The sampler starts before the warm-up so that it is already
        # reporting when the timed steps run.
        clk.mark()
        total_ms = timed(step)
        if split is not None:
            # The same K steps with the split exchange; the faster of the two
            # (max over ranks each) is the job's step.
            def push():
                _ops.bwd_peer(x, w, b, dout, init, None, dx, dwdb, dinit, dw, db, True,
                              *split.args(_lib.PEER_PUSH))

            def finish():
                _ops.bwd_peer(x, w, b, dout, init, None, dx, dwdb, dinit, dw, db, True,
                              *split.args(_lib.PEER_FINISH))

            def split_step(_=0):
                fwd()
                finish()  # the previous step's exchange (FINISH before the next PUSH)
                push()

            fwd()
            push()  # the first step has no previous exchange to finish
            split_ms = timed(split_step)
            finish()  # the last step's exchange
            torch.cuda.synchronize()
            split.check()
            fused_max, split_max = max_over_ranks(total_ms, world), max_over_ranks(split_ms, world)
            exchange = {"fused_ms_per_step": fused_max / K, "split_ms_per_step": split_max / K,
                        "used": "split" if split_max < fused_max else "fused"}
            if split_max < fused_max:
                total_ms = split_ms
        clk.unmark()
    # Per-op kernel times: graphs of the op alone, replayed back to back.
    reps = max(20, min(200, K // 10))
    g_fwd, g_bwd = graph_of(fwd, 10), graph_of(bwd, 10)
    barrier_sync(world)
    device_rendezvous(world)
    fwd_ms = graph_ms(g_fwd, reps, 10)
    barrier_sync(world)
    device_rendezvous(world)
    bwd_ms = graph_ms(g_bwd, reps, 10)
    del g_fwd, g_bwd
    barrier_sync(world)
    extra = {}
    if world > 1:
        # Each rank's step with a local reduction only (no exchange, no
        # waiting for peers): the spread of these is the GPUs' own speed
        # difference, which a synchronous data-parallel step cannot hide.
        # The fused step's results (dwdb, dw, db hold the cross-rank sums)
        # are checked first; the local-reduction step below writes its own
        # buffers, so it cannot disturb them either way.
        extra["parity"] = peer_parity(x, w, b, dout, init, dwdb, dw, db, world)
        l_dx, l_dinit = torch.empty_like(dx), torch.empty_like(dinit)
        l_dwdb, l_dw, l_db = torch.empty_like(dwdb), torch.empty_like(dw), torch.empty_like(db)

        def local_step(_=0):
            fwd()
            _ops.bwd(x, w, b, dout, None, init, None, l_dx, l_dwdb, l_dinit, l_dw, l_db, True)

        local_ms = graph_ms(graph_of(local_step, 10), reps, 10)

        def fused_step(_=0):
            fwd()
            bwd()

        barrier_sync(world)
        device_rendezvous(world)
        fused_ms = graph_ms(graph_of(fused_step, 10), reps, 10)
        per_rank = gather_floats([total_ms / K, bwd_ms, local_ms, fused_ms], world)
        extra["per_rank"] = {
            "step_ms": [r[0] for r in per_rank],
            "bwd_with_exchange_ms": [r[1] for r in per_rank],
            "step_local_reduction_ms": [r[2] for r in per_rank],
            "step_fused_exchange_ms": [r[3] for r in per_rank],
            "note": "step_ms: the timed step (the faster exchange, see `exchange`); bwd_with_exchange_ms: the backward alone with the fused exchange; "
                    "step_fused_exchange_ms: fwd+bwd with the fused exchange (waiting inside the reduction "
                    "kernel); step_local_reduction_ms: the same fwd+bwd with the dweight/dbias reduction kept on the "
                    "rank (no exchange); its max over ranks bounds a synchronous step from below",
        }
    extra["parity_c2"] = c2_parity(x, w, b, init, dout, out, fs, dx, dinit, dw, db) if rank == 0 else None
    total_ms = max_over_ranks(total_ms, world)
    if exchange:
        extra["exchange"] = exchange
    return dict(ms_per_step=total_ms / K, fwd_ms=fwd_ms, bwd_ms=bwd_ms, clocks=clk.summary(), **extra)


def peer_parity(x, w, b, dout, init, dwdb_fused, dw_fused, db_fused, world):
    """After the timed region: every rank recomputes its shard's backward
    with the plain single-GPU reduction, the fp32 [dweight | dbias] buffers
    are gathered over NCCL and summed in rank order, and the result must be
    BITWISE equal to what the fused peer-exchange kernel left on this rank
    (fp32 and the bf16 copies).  Returns the verdict of all ranks."""
    import torch.distributed as dist

    from causal_conv1d_b200 import _ops

    torch.cuda.synchronize()
    dwdb = torch.empty_like(dwdb_fused)
    _ops.bwd(x, w, b, dout, None, init, None, torch.empty_like(x), dwdb, torch.empty_like(init), None, None, True)
    parts = [torch.empty_like(dwdb) for _ in range(world)]
    dist.all_gather(parts, dwdb)
    total = torch.zeros_like(dwdb)
    for p in parts:
        total = total + p
    ok = (torch.equal(dwdb_fused, total) and torch.equal(dw_fused, total[: D * W].view(D, W).to(DT))
          and torch.equal(db_fused, total[D * W:].to(DT)))
    flags = torch.tensor([1 if ok else 0], dtype=torch.int32, device="cuda")
    every = [torch.empty_like(flags) for _ in range(world)]
    dist.all_gather(every, flags)
    good = [int(f.item()) for f in every]
    return {"peer_dwdb_bitwise": all(good), "ranks_checked": world, "ranks_ok": sum(good),
            "how": "fused peer-exchange dweight|dbias (fp32 and bf16) == rank-order sum of per-rank "
                   "single-GPU results gathered over NCCL, on every rank"}


def c2_parity(x, w, b, init, dout, out, fs, dx, dinit, dw, db):
    """Whole-tensor check of the timed C2 step's results against an fp32
    evaluation of the pure-PyTorch reference (causal_conv1d_ref + autograd)
    on the GPU: bf16 outputs within rtol = atol = 1e-2, weight gradients
    within 1e-2 x max|ref|, final_states bit-exact.  The last replay of the
    step left its results in these buffers; the backward is rerun here with
    the local reduction so that dw/db are this rank's own (with N GPUs the
    timed buffers hold the cross-rank sums)."""
    from causal_conv1d_b200 import _ops, causal_conv1d_ref

    dwdb = torch.empty(D * (W + 1), dtype=torch.float32, device="cuda")
    dw1, db1 = torch.empty_like(dw), torch.empty_like(db)
    _ops.bwd(x, w, b, dout, None, init, None, dx, dwdb, dinit, dw1, db1, True)
    xf = x.detach().float().requires_grad_()
    wf = w.detach().float().requires_grad_()
    bf = b.detach().float().requires_grad_()
    inf = init.detach().float().requires_grad_()
    ro, rfs = causal_conv1d_ref(xf, wf, bf, initial_states=inf, return_final_states=True, activation="silu")
    ro.backward(dout.float())

    def worst(a, e, atol, rtol=1e-2):
        a, e = a.float(), e.float()
        bad = ~((a - e).abs() <= atol + rtol * e.abs())
        return int(bad.sum()), float((a - e).abs().max())

    norm = max(wf.grad.abs().max().item(), bf.grad.abs().max().item())
    checks = {"out": worst(out, ro.detach(), 1e-2), "dx": worst(dx, xf.grad, 1e-2),
              "dinit": worst(dinit, inf.grad, 1e-2), "dweight": worst(dw1, wf.grad, 1e-2 * max(1.0, norm)),
              "dbias": worst(db1, bf.grad, 1e-2 * max(1.0, norm))}
    fs_exact = torch.equal(fs, rfs.detach().to(DT))
    return {"whole_tensor_ok": all(n == 0 for n, _ in checks.values()) and fs_exact,
            "final_states_bitwise": fs_exact,
            "max_abs_err": {k: v for k, (_, v) in checks.items()},
            "out_of_tolerance": {k: n for k, (n, _) in checks.items()},
            "how": "C2 step outputs vs causal_conv1d_ref in fp32 on the GPU (bf16 inputs upcast): rtol=atol=1e-2, "
                   "weight grads atol 1e-2*max|ref|; every element of every tensor"}


C5_B, C5_D, C5_L = 64, 8192, 8192


def time_c5_sweep(world, rank, local, peak):
    """the large (64, 8192, 8192) bf16 problem,
    forward + backward with initial and final states, widths 2/3/4, SiLU on
    and off, split over the `world` GPUs two ways (strong scaling: the job is
    the whole problem at every N):

      batch -- rank r owns batch rows shard_range(64, r, N) and the full
               weights; the backward's dweight/dbias sum over the ranks runs
               inside its reduction kernel (NVLink peer exchange);
      dim   -- rank r owns channels shard_range(8192, r, N) with the matching
               weight / bias / state slices; no communication at all.

    Each op is timed alone (a CUDA graph of 4 launches replayed, device-side
    rendezvous before the start event), max over ranks.  At N = 1 both splits
    are the same single-GPU problem, reported once as "single"."""
    from causal_conv1d_b200 import _ops
    from causal_conv1d_b200.parallel import PeerReducer, shard_range

    g = torch.Generator(device="cuda").manual_seed(50 + rank)

    def rn(*sh):
        return torch.randn(*sh, generator=g, device="cuda", dtype=torch.float32).to(DT)

    def ru(*sh):
        return (torch.rand(*sh, generator=g, device="cuda", dtype=torch.float32) - 0.5).to(DT)

    def op_ms(fn):
        fn()
        torch.cuda.synchronize()
        gr = graph_of(lambda i: fn(), 4)
        barrier_sync(world)
        device_rendezvous(world)
        ms = graph_ms(gr, 2, 4)
        del gr
        barrier_sync(world)
        return max_over_ranks(ms, world)

    out_tab = {}
    for sh in (("batch", "dim") if world > 1 else ("single",)):
        if sh == "batch":
            b0, b1 = shard_range(C5_B, rank, world)
            Bl, Dl = b1 - b0, C5_D
        elif sh == "dim":
            d0, d1 = shard_range(C5_D, rank, world)
            Bl, Dl = C5_B, d1 - d0
        else:
            Bl, Dl = C5_B, C5_D
        x, dout = rn(Bl, Dl, C5_L), rn(Bl, Dl, C5_L)
        out, dx = torch.empty_like(x), torch.empty_like(x)
        n = Bl * Dl * C5_L
        rows = []
        for width in (2, 3, 4):
            w, b = ru(Dl, width), ru(Dl)
            init = rn(Bl, Dl, width - 1)
            fs, dinit = torch.empty_like(init), torch.empty_like(init)
            dwdb = torch.empty(Dl * (width + 1), dtype=torch.float32, device="cuda")
            dw = torch.empty(Dl, width, dtype=DT, device="cuda")
            db = torch.empty(Dl, dtype=DT, device="cuda")
            reducer = PeerReducer(Dl, width, torch.device("cuda", local)) if sh == "batch" else None
            for silu in (True, False):
                def fwd(silu=silu):
                    _ops.fwd(x, w, b, None, init, out, silu, fs)

                def bwd(silu=silu):
                    if reducer is not None:
                        _ops.bwd_peer(x, w, b, dout, init, None, dx, dwdb, dinit, dw, db, silu, *reducer.args())
                    else:
                        _ops.bwd(x, w, b, dout, None, init, None, dx, dwdb, dinit, dw, db, silu)

                fms, bms = op_ms(fwd), op_ms(bwd)
                fb = 4 * n + 2 * init.numel() * 2 + Dl * (width + 1) * 2
                bb = 6 * n + 2 * init.numel() * 2 + Dl * (width + 1) * (2 + 2 + 4)
                rows.append({"width": width, "silu": silu, "fwd_ms": fms, "bwd_ms": bms,
                             "tokens_per_s": C5_B * C5_L / ((fms + bms) / 1e3),
                             "fwd_frac": fb / fms / 1e6 / peak, "bwd_frac": bb / bms / 1e6 / peak,
                             "fwd_bytes_per_gpu": fb, "bwd_bytes_per_gpu": bb})
            if reducer is not None:
                if rank == 0:
                    reducer.check()
                reducer.close()
            del w, b, init, fs, dinit, dwdb, dw, db
        del x, dout, out, dx
        torch.cuda.empty_cache()
        out_tab[sh] = {"per_gpu_shape_rank0": [Bl, Dl, C5_L], "rows": rows}
    return {"workload": "BASELINE configs[4]: x (64, 8192, 8192) bf16 contiguous, fwd+bwd, initial + final states, "
                        "width 2/3/4, SiLU on/off; whole problem split over the GPUs (strong scaling)",
            "n_gpus": world, "timing": "each op alone, CUDA graph of 4 launches x 2 replays, max over ranks; "
                                       "fractions per GPU against the measured HBM copy peak",
            "shardings": out_tab}


def gpu_local_cpus(dev_index):
    """CPUs on the GPU's NUMA node (read from NVML; no setting is changed), or
    None when NVML cannot tell."""
    try:
        import pynvml

        props = torch.cuda.get_device_properties(dev_index)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            words = pynvml.nvmlDeviceGetCpuAffinity(h, 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * i + j for i, w in enumerate(words) for j in range(64) if (w >> j) & 1}
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except Exception:  # no NVML, no affinity information: leave placement alone
        return None


def pinned_near_gpu(tensors):
    """Pinned host copies of `tensors`, first touched from the CPUs next to
    the current GPU so that their pages sit on its NUMA node (the process's
    CPU affinity is restored afterwards)."""
    local = gpu_local_cpus(torch.cuda.current_device())
    before = os.sched_getaffinity(0)
    try:
        if local:
            os.sched_setaffinity(0, local)
        return {k: (v.cpu() if v.is_cuda else v).pin_memory() for k, v in tensors.items()}
    finally:
        os.sched_setaffinity(0, before)


def time_e2e(args, world, rank, reducer):
    """Public API, host buffers in and out, every step (three-stream
    pipeline: upload of step i+1 and download of step i overlap compute)."""
    from causal_conv1d_b200 import causal_conv1d_fn
    from causal_conv1d_b200.parallel import causal_conv1d_fn_batch_sharded

    xd, wd, bd, initd, doutd = make_c2(99 + rank, "cuda")
    # Channel-last activations live on the host as (B, L, D) arrays.
    host = dict(x=xd.transpose(1, 2).contiguous(), w=wd, b=bd, init=initd, dout=doutd.transpose(1, 2).contiguous())
    host = pinned_near_gpu(host)
    del xd, wd, bd, initd, doutd
    outs = pinned_near_gpu({k: torch.empty(s, dtype=DT) for k, s in dict(
        out=(B, L, D), fs=(B, D, W - 1), dx=(B, L, D), dw=(D, W), db=(D,), dinit=(B, D, W - 1)).items()})
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = sum(t.numel() * t.element_size() for t in outs.values())
    dev_in = [{k: torch.empty_like(v, device="cuda") for k, v in host.items()} for _ in range(2)]
    s_comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    for ev in in_free:
        ev.record(s_comp)

    def step(i):
        k = i % 2
        buf = dev_in[k]
        with torch.cuda.stream(s_in):
            s_in.wait_event(in_free[k])  # compute of step i-2 is done with this buffer set
            for name, t in host.items():
                buf[name].copy_(t, non_blocking=True)
            in_ready[k].record(s_in)
        s_comp.wait_event(in_ready[k])
        x = buf["x"].transpose(1, 2).detach().requires_grad_()
        w = buf["w"].detach().requires_grad_()
        b = buf["b"].detach().requires_grad_()
        init = buf["init"].detach().requires_grad_()
        dout = buf["dout"].transpose(1, 2)
        if world > 1:
            out, fs = causal_conv1d_fn_batch_sharded(x, w, b, initial_states=init, return_final_states=True,
                                                      activation="silu", reducer=reducer)
        else:
            out, fs = causal_conv1d_fn(x, w, b, initial_states=init, return_final_states=True, activation="silu")
        torch.autograd.backward([out], [dout])
        in_free[k].record(s_comp)
        results = dict(out=out.detach().transpose(1, 2), fs=fs.detach(), dx=x.grad.transpose(1, 2), dw=w.grad,
                       db=b.grad, dinit=init.grad)
        s_out.wait_stream(s_comp)
        with torch.cuda.stream(s_out):
            for name, t in results.items():
                outs[name].copy_(t, non_blocking=True)
                t.record_stream(s_out)  # keep the allocator off it until the download is done

    K = max(3, min(args.steps, 20))
    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    barrier_sync(world)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s_in)
    for i in range(K):
        step(i)
    stop.record(s_out)
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(stop), world) / K
    return dict(value=world * B * L / (ms / 1e3), unit=UNIT, h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h,
                ms_per_step=ms, steps=K,
                path="causal_conv1d_fn + autograd backward from pinned host buffers; upload, compute and download "
                     "on three streams (device inputs double-buffered)")


def _kernel_ms(fn, iters, sets):
    """Average time of fn(i), i cycling over `sets` buffer sets: a CUDA graph
    of max(sets, 8) launches replayed back to back (no host launch overhead)."""
    n = max(sets, 8)
    for i in range(sets):
        fn(i)
    torch.cuda.synchronize()
    g = graph_of(lambda i: fn(i % sets), n)
    return graph_ms(g, max(1, iters // n), n)


def decode_sweep(w, b, rn, peak):
    from causal_conv1d_b200 import _ops

    Du = w.shape[0]
    sets = 8
    out = {}
    for mode in ("c3a_indexed", "c3b_circular"):
        pts = []
        for Bs in (1, 256, 384, 512, 768, 1024):
            xs = [rn(Bs, Du, 1) for _ in range(sets)]
            outs = [torch.empty_like(xs[0]) for _ in range(sets)]
            if mode == "c3a_indexed":
                pools = [rn(2 * Bs, Du, W - 1) for _ in range(sets)]
                idx = [torch.randperm(2 * Bs, device="cuda")[:Bs].to(torch.int32) for _ in range(sets)]
                ms = _kernel_ms(lambda i: _ops.update(xs[i], pools[i], w, b, None, idx[i], outs[i], True), 800, sets)
                row = Du * (2 + 2 + 6 + 6)
                del pools, idx
            else:
                sts = [rn(Bs, Du, 8) for _ in range(sets)]
                cache = [torch.randint(0, 1024, (Bs,), device="cuda", dtype=torch.int32) for _ in range(sets)]
                ms = _kernel_ms(lambda i: _ops.update(xs[i], sts[i], w, b, cache[i], None, outs[i], True), 800, sets)
                row = Du * (2 + 2 + 6 + 2)
                del sts, cache
            pts.append((Bs, ms * 1e3, Bs * row))
            del xs, outs
        fit = [p for p in pts if p[0] >= 256]
        n = len(fit)
        mx = sum(p[0] for p in fit) / n
        my = sum(p[1] for p in fit) / n
        slope = sum((p[0] - mx) * (p[1] - my) for p in fit) / sum((p[0] - mx) ** 2 for p in fit)
        t0 = my - slope * mx
        row_bytes = pts[0][2] / pts[0][0]
        out[mode] = {"batch_us": {str(p[0]): p[1] for p in pts}, "fit_batches": [p[0] for p in fit],
                     "fit_floor_us": t0, "fit_us_per_row": slope,
                     "fit_transfer_gbs": row_bytes / (slope * 1e-6) / 1e9,
                     "fit_transfer_frac": row_bytes / (slope * 1e-6) / 1e9 / peak,
                     "row_bytes_algorithmic": row_bytes}
    torch.cuda.empty_cache()
    return out


def time_decode_sharded(world, rank, peak):
    """Decode rows of the multi-GPU table: causal_conv1d_update batch-sharded,
    no collective (pool slots stay on their GPU).  Every rank serves its own
    C3a batch (256 requests on a pool of 512 slots, indexed) and C3b batch
    (256 circular states of 8), weak scaling; each op is a CUDA graph of 8
    launches over rotating buffer sets (> L2), and the time is the max over
    ranks."""
    from causal_conv1d_b200 import _ops

    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    Bu, Du, sets = 256, D, 8

    def rn(*s):
        return torch.randn(*s, generator=g, device="cuda", dtype=torch.float32).to(DT)

    w = (torch.rand(Du, W, generator=g, device="cuda") - 0.5).to(DT)
    bias = (torch.rand(Du, generator=g, device="cuda") - 0.5).to(DT)
    xs = [rn(Bu, Du, 1) for _ in range(sets)]
    outs = [torch.empty_like(xs[0]) for _ in range(sets)]
    pools = [rn(2 * Bu, Du, W - 1) for _ in range(sets)]
    idx = [torch.randperm(2 * Bu, device="cuda", generator=g)[:Bu].to(torch.int32) for _ in range(sets)]
    states = [rn(Bu, Du, 8) for _ in range(sets)]
    cache = [torch.randint(0, 1024, (Bu,), device="cuda", dtype=torch.int32, generator=g) for _ in range(sets)]
    ops = {
        "c3a_indexed": (lambda i: _ops.update(xs[i], pools[i], w, bias, None, idx[i], outs[i], True),
                        Bu * Du * (2 + 2 + 6 + 6) + Du * (W + 1) * 2 + Bu * 4),
        "c3b_circular": (lambda i: _ops.update(xs[i], states[i], w, bias, cache[i], None, outs[i], True),
                         Bu * Du * (2 + 2 + 6 + 2) + Du * (W + 1) * 2 + Bu * 4),
    }
    res = {"workload": f"causal_conv1d_update batch-sharded: each GPU its own ({Bu}, {Du}) bf16 decode batch "
                       f"(weak scaling, no collective)", "n_gpus": world}
    for name, (fn, nbytes) in ops.items():
        for i in range(sets):
            fn(i)
        torch.cuda.synchronize()
        gr = graph_of(fn, sets)
        graph_ms(gr, 20, sets)  # warm-up replays
        ms = graph_ms(gr, 100, sets)  # no cross-rank dependency: each GPU timed on its own
        per = [v[0] for v in gather_floats([ms], world)]
        t = max(per)
        res[name] = {"ms_per_launch_max_over_ranks": t, "per_rank_ms": per,
                     "tokens_per_s": world * Bu / (t / 1e3), "frac_per_gpu": nbytes / t / 1e6 / peak,
                     "algorithmic_bytes_per_gpu": nbytes}
        del gr
    del xs, outs, pools, idx, states, cache
    torch.cuda.empty_cache()
    return res


def peak_tflops():
    p = REPO / "MEASURED_PEAKS.json"
    if p.is_file():
        return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def time_fused(peak_tf):
    """The in_proj GEMM with the conv as its epilogue (one kernel) vs cuBLAS
    GEMM + the conv kernel, C2 (Mamba-2 2.7B) shapes, W = 4, bias, SiLU,
    initial and final states.  Tensor-bound: TFLOP/s of the GEMM (2 M N K)."""
    from causal_conv1d_b200 import _ops

    peak, kind = peak_tf
    Bf, Lf, Kf, Nf = B, L, 2560, D
    g = torch.Generator(device="cuda").manual_seed(11)
    hidden = torch.randn(Bf, Lf, Kf, generator=g, device="cuda").to(DT)
    win = (torch.randn(Nf, Kf, generator=g, device="cuda") / Kf ** 0.5).to(DT)
    cw = (torch.rand(Nf, W, generator=g, device="cuda") - 0.5).to(DT)
    cb = (torch.rand(Nf, generator=g, device="cuda") - 0.5).to(DT)
    st = torch.randn(Bf, Nf, W - 1, generator=g, device="cuda").to(DT)
    out = torch.empty(Bf, Lf, Nf, dtype=DT, device="cuda")
    fs = torch.empty(Bf, Nf, W - 1, dtype=DT, device="cuda")
    y = torch.empty(Bf, Lf, Nf, dtype=DT, device="cuda")
    out2 = torch.empty_like(out)
    fused_ms = _kernel_ms(lambda i: _ops.inproj_conv(hidden, win, cw, cb, st, out, True, fs), 80, 1)
    gemm_ms = _kernel_ms(lambda i: torch.matmul(hidden, win.t(), out=y), 80, 1)

    def pair(i):
        torch.matmul(hidden, win.t(), out=y)
        _ops.fwd(y.transpose(1, 2), cw, cb, None, st, out2.transpose(1, 2), True, fs)

    pair_ms = _kernel_ms(pair, 80, 1)
    flops = 2 * Bf * Lf * Kf * Nf
    return {"ms": fused_ms, "tflops": flops / fused_ms / 1e9, "frac": flops / fused_ms / 1e9 / peak,
            "bound": "tensor", "peak_tflops": peak, "peak_source": f"{kind} bf16 GEMM",
            "unfused_ms": pair_ms, "cublas_gemm_ms": gemm_ms, "speedup_vs_unfused": pair_ms / fused_ms,
            "cublas_gemm_tflops": flops / gemm_ms / 1e9,
            "note": "hidden (8, 2048, 2560) @ in_weight (5376, 2560)^T, conv W=4 + bias + SiLU + states in the "
                    "epilogue (xBC never stored); unfused = torch.matmul (cuBLAS) + cc1d_fwd"}


def time_kernels(peak):
    """Secondary kernels of the metric, each timed alone."""
    from causal_conv1d_b200 import _ops

    res = {}
    g = torch.Generator(device="cuda").manual_seed(7)

    def rn(*s, dt=DT):
        return torch.randn(*s, generator=g, device="cuda", dtype=torch.float32).to(dt)

    def ru(*s, dt=DT):
        return (torch.rand(*s, generator=g, device="cuda", dtype=torch.float32) - 0.5).to(dt)

    # C3a: decode update, indexed pool (512, 5376, 3); rotate 8 sets (> L2).
    Bu, Du = 256, 5376
    sets = 8
    w, b = ru(Du, W), ru(Du)
    xs = [rn(Bu, Du, 1) for _ in range(sets)]
    pools = [rn(512, Du, W - 1) for _ in range(sets)]
    idx = [torch.randperm(512, device="cuda")[:Bu].to(torch.int32) for _ in range(sets)]
    outs = [torch.empty_like(xs[0]) for _ in range(sets)]
    ms = _kernel_ms(lambda i: _ops.update(xs[i], pools[i], w, b, None, idx[i], outs[i], True), 800, sets)
    nbytes = Bu * Du * (2 + 2 + 6 + 6) + Du * (W + 1) * 2 + Bu * 4
    res["update_c3a_indexed"] = dict(ms=ms, gbs=nbytes / ms / 1e6, frac=nbytes / ms / 1e6 / peak,
                                     tokens_per_s=Bu / (ms / 1e3), algorithmic_bytes=nbytes)
    del pools
    # C3b: circular (256, 5376, 8), cache_seqlens ~ U{0..1023}.
    states = [rn(Bu, Du, 8) for _ in range(sets)]
    cache = [torch.randint(0, 1024, (Bu,), device="cuda", dtype=torch.int32) for _ in range(sets)]
    ms = _kernel_ms(lambda i: _ops.update(xs[i], states[i], w, b, cache[i], None, outs[i], True), 800, sets)
    nbytes = Bu * Du * (2 + 2 + 6 + 2) + Du * (W + 1) * 2 + Bu * 4
    res["update_c3b_circular"] = dict(ms=ms, gbs=nbytes / ms / 1e6, frac=nbytes / ms / 1e6 / peak,
                                      tokens_per_s=Bu / (ms / 1e3), algorithmic_bytes=nbytes)
    del states, xs, outs
    torch.cuda.empty_cache()

    # Fixed cost of a decode step: the same two kernels over a range of batch
    # sizes in the same harness.  A least-squares line t(B) = t0 + B * s over
    # the batches whose 8 rotating buffer sets exceed L2 (B >= 256) splits
    # the C3 time into a per-launch floor t0 (launch, the dependent index ->
    # state round trips, the last wave's drain) and a transfer part whose
    # bandwidth is row_bytes / s.  B = 1 is reported alone (its data sits in
    # L2: pure fixed cost).
    res["decode_batch_sweep"] = decode_sweep(w, b, rn, peak)

    # Next rows of the path: a 4-token decode burst (speculative decoding) on
    # the C3a pool (update_lin_kernel), and the C3a / C3b steps with the
    # conv_state stored channel-last (strides (S*D, 1, D), vLLM's layout;
    # update_vec_kernel's channel-last linear and circular modes).
    Lb = 4
    xs = [rn(Bu, Du, Lb) for _ in range(sets)]
    pools = [rn(512, Du, W - 1) for _ in range(sets)]
    outs = [torch.empty_like(xs[0]) for _ in range(sets)]
    ms = _kernel_ms(lambda i: _ops.update(xs[i], pools[i], w, b, None, idx[i], outs[i], True), 800, sets)
    nbytes = Bu * Du * (2 * Lb + 2 * Lb + 6 + 6) + Du * (W + 1) * 2 + Bu * 4
    res["update_burst4_indexed"] = dict(ms=ms, gbs=nbytes / ms / 1e6, frac=nbytes / ms / 1e6 / peak,
                                        tokens_per_s=Bu * Lb / (ms / 1e3), algorithmic_bytes=nbytes,
                                        note="x (256, 5376, 4), pool (512, 5376, 3), update_lin_kernel")
    del xs, pools, outs
    xs = [rn(Bu, Du, 1) for _ in range(sets)]
    pools = [rn(512, W - 1, Du).transpose(1, 2) for _ in range(sets)]
    outs = [torch.empty_like(xs[0]) for _ in range(sets)]
    ms = _kernel_ms(lambda i: _ops.update(xs[i], pools[i], w, b, None, idx[i], outs[i], True), 800, sets)
    nbytes = Bu * Du * (2 + 2 + 6 + 6) + Du * (W + 1) * 2 + Bu * 4
    res["update_c3a_chanlast_state"] = dict(ms=ms, gbs=nbytes / ms / 1e6, frac=nbytes / ms / 1e6 / peak,
                                            tokens_per_s=Bu / (ms / 1e3), algorithmic_bytes=nbytes,
                                            note="C3a with conv_state pool stored (512, 3, 5376)")
    del pools
    states = [rn(Bu, 8, Du).transpose(1, 2) for _ in range(sets)]
    cache = [torch.randint(0, 1024, (Bu,), device="cuda", dtype=torch.int32) for _ in range(sets)]
    ms = _kernel_ms(lambda i: _ops.update(xs[i], states[i], w, b, cache[i], None, outs[i], True), 800, sets)
    nbytes = Bu * Du * (2 + 2 + 6 + 2) + Du * (W + 1) * 2 + Bu * 4
    res["update_c3b_chanlast_state"] = dict(ms=ms, gbs=nbytes / ms / 1e6, frac=nbytes / ms / 1e6 / peak,
                                            tokens_per_s=Bu / (ms / 1e3), algorithmic_bytes=nbytes,
                                            note="C3b with the circular state stored (256, 8, 5376)")
    del xs, states, outs
    torch.cuda.empty_cache()

    # C4: varlen packed prefill fp16 (1, 4096, 65536) channel-last + seq_idx.
    dt = torch.float16
    Lv, Dv = 65536, 4096
    gl = torch.Generator().manual_seed(0)
    raw = torch.randint(256, 4097, (32,), generator=gl)
    lens = (raw * Lv // raw.sum()).clamp(min=1)
    lens[-1] += Lv - lens.sum()
    seq = torch.repeat_interleave(torch.arange(32, dtype=torch.int32), lens).view(1, Lv).cuda()
    x = rn(1, Lv, Dv, dt=dt).transpose(1, 2)
    dout = rn(1, Lv, Dv, dt=dt).transpose(1, 2)
    wv, bv = ru(Dv, W, dt=dt), ru(Dv, dt=dt)
    out, dx = torch.empty_like(x), torch.empty_like(x)
    dwdb = torch.empty(Dv * (W + 1), dtype=torch.float32, device="cuda")
    dw, db = torch.empty(Dv, W, dtype=dt, device="cuda"), torch.empty(Dv, dtype=dt, device="cuda")
    n = Lv * Dv
    ms = _kernel_ms(lambda i: _ops.fwd(x, wv, bv, seq, None, out, True, None), 10, 1)
    nb = 4 * n + Lv * 4 + Dv * (W + 1) * 2
    res["fwd_c4_varlen"] = dict(ms=ms, gbs=nb / ms / 1e6, frac=nb / ms / 1e6 / peak, tokens_per_s=Lv / (ms / 1e3),
                                algorithmic_bytes=nb)
    ms = _kernel_ms(lambda i: _ops.bwd(x, wv, bv, dout, seq, None, None, dx, dwdb, None, dw, db, True), 10, 1)
    nb = 6 * n + Lv * 4 + Dv * (W + 1) * 2 * 2 + Dv * (W + 1) * 4
    res["bwd_c4_varlen"] = dict(ms=ms, gbs=nb / ms / 1e6, frac=nb / ms / 1e6 / peak, tokens_per_s=Lv / (ms / 1e3),
                                algorithmic_bytes=nb)
    # The same packed batch in the contiguous (B, D, L) layout (seqlen TMA
    # kernels with the sequence-id tiles).
    del x, dout, out, dx
    torch.cuda.empty_cache()
    xc, doutc = rn(1, Dv, Lv, dt=dt), rn(1, Dv, Lv, dt=dt)
    outc, dxc = torch.empty_like(xc), torch.empty_like(xc)
    ms = _kernel_ms(lambda i: _ops.fwd(xc, wv, bv, seq, None, outc, True, None), 10, 1)
    nb = 4 * n + Lv * 4 + Dv * (W + 1) * 2
    res["fwd_c4_contiguous"] = dict(ms=ms, gbs=nb / ms / 1e6, frac=nb / ms / 1e6 / peak,
                                    tokens_per_s=Lv / (ms / 1e3), algorithmic_bytes=nb)
    ms = _kernel_ms(lambda i: _ops.bwd(xc, wv, bv, doutc, seq, None, None, dxc, dwdb, None, dw, db, True), 10, 1)
    nb = 6 * n + Lv * 4 + Dv * (W + 1) * 2 * 2 + Dv * (W + 1) * 4
    res["bwd_c4_contiguous"] = dict(ms=ms, gbs=nb / ms / 1e6, frac=nb / ms / 1e6 / peak,
                                    tokens_per_s=Lv / (ms / 1e3), algorithmic_bytes=nb)
    x = xc.transpose(1, 2).contiguous().transpose(1, 2)  # channel-last copy for the hand-off below
    del xc, doutc, outc, dxc
    dout = out = dx = None

    # varlen states hand-off of the C4 batch: the last W-1 tokens of each of
    # the 32 packed sequences -> (32, 4096, 3) conv states.
    tok = x.transpose(1, 2)[0]  # (65536, 4096) token-major view
    cu = torch.cat([torch.zeros(1, dtype=torch.int32), lens.cumsum(0).to(torch.int32)]).cuda()
    st = torch.empty(32, W - 1, Dv, dtype=dt, device="cuda").transpose(1, 2)
    ms = _kernel_ms(lambda i: _ops.varlen_states(tok, cu, st), 200, 1)
    nb = 2 * 32 * Dv * (W - 1) * 2 + 33 * 4
    res["varlen_states_c4"] = dict(ms=ms, gbs=nb / ms / 1e6, frac=nb / ms / 1e6 / peak, algorithmic_bytes=nb,
                                   note="32 sequences, state_len 3, dim 4096 fp16; launch-latency bound")
    del x, dout, out, dx
    torch.cuda.empty_cache()

    # C2 shape with an odd length in the contiguous layout: row pitch
    # 2047 * 2 bytes is not a multiple of 16 (shifted-row TMA kernels).
    Bo, Do, Lo = 8, 5376, 2047
    xo, douto = rn(Bo, Do, Lo), rn(Bo, Do, Lo)
    wo, bo = ru(Do, W), ru(Do)
    inito = rn(Bo, Do, W - 1)
    outo, dxo, fso, dinito = torch.empty_like(xo), torch.empty_like(xo), torch.empty_like(inito), torch.empty_like(inito)
    dwdbo = torch.empty(Do * (W + 1), dtype=torch.float32, device="cuda")
    dwo, dbo = torch.empty(Do, W, dtype=DT, device="cuda"), torch.empty(Do, dtype=DT, device="cuda")
    n = Bo * Do * Lo
    ms = _kernel_ms(lambda i: _ops.fwd(xo, wo, bo, None, inito, outo, True, fso), 40, 1)
    nb = 4 * n + 2 * inito.numel() * 2 + Do * (W + 1) * 2
    res["fwd_c2_odd_len_contiguous"] = dict(ms=ms, gbs=nb / ms / 1e6, frac=nb / ms / 1e6 / peak,
                                            tokens_per_s=Bo * Lo / (ms / 1e3), algorithmic_bytes=nb,
                                            note="(8, 5376, 2047) bf16 contiguous: row pitch not 16-byte aligned")
    ms = _kernel_ms(lambda i: _ops.bwd(xo, wo, bo, douto, None, inito, None, dxo, dwdbo, dinito, dwo, dbo, True), 40, 1)
    nb = 6 * n + 2 * inito.numel() * 2 + Do * (W + 1) * (2 + 2 + 4)
    res["bwd_c2_odd_len_contiguous"] = dict(ms=ms, gbs=nb / ms / 1e6, frac=nb / ms / 1e6 / peak,
                                            tokens_per_s=Bo * Lo / (ms / 1e3), algorithmic_bytes=nb)
    del xo, douto, outo, dxo
    torch.cuda.empty_cache()

    # Fused neighbour (next row of the path): the in_proj GEMM of the C2
    # block, xBC = hidden (16384 x 2560) @ in_weight^T (2560 x 5376), with the
    # conv as its epilogue, against the pair it replaces timed alongside:
    # cuBLAS GEMM (torch.matmul, xBC stored in bf16), then the conv kernel.
    # Timed last: these tensor-core kernels run at the 1 kW power cap and
    # leave the clocks low for a moment, which would bias HBM lines after them.
    res["inproj_conv_fused_c2"] = time_fused(peak_tflops())
    torch.cuda.empty_cache()
    return res


# --------------------------------------------------------------------------
# CPU path (oracle port): baseline leg and reference arm
# --------------------------------------------------------------------------

def host_cores():
    """Host threads available to this process (torchrun sets
    OMP_NUM_THREADS=1 for its workers, so OpenMP's default is not used)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_sample_step(state):
    """One sample step of the reference CPU algorithm: forward + backward of
    batch row 0 of C2 (1, 5376, 2048), float accumulation, all host threads."""
    import oracle

    x, w, b, init, dout = state
    n = host_cores()
    oracle.fwd(x, w, b, None, init, silu=True, return_final_states=True, acc64=False, nthreads=n)
    oracle.bwd(x, w, dout, b, None, init, None, silu=True, acc64=False, nthreads=n)


def cpu_setup():
    import oracle

    oracle.load()
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, L, D, generator=g).to(DT).transpose(1, 2)
    w = (torch.rand(D, W, generator=g) - 0.5).to(DT)
    b = (torch.rand(D, generator=g) - 0.5).to(DT)
    init = torch.randn(1, D, W - 1, generator=g).to(DT)
    dout = torch.randn(1, L, D, generator=g).to(DT).transpose(1, 2)
    return (x, w, b, init, dout), host_cores()


def cpu_baseline(budget_s=10.0):
    state, cores = cpu_setup()
    cpu_sample_step(state)
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter_ns()
        cpu_sample_step(state)
        times.append((time.perf_counter_ns() - t0) / 1e9)
        if len(times) >= 200:
            break
    best = min(times)
    return {"value": L / best, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"C2 batch row 0 (1, {D}, {L}) fwd+bwd, bf16, min of {len(times)} runs "
                      f"({best * 1e3:.1f} ms each); oracle/cc1d_oracle.c float accumulation, OpenMP"}


def c2_config(world):
    """The workload both arms report (the reference arm times a bounded
    sample of it, described in its cpu_baseline.sample)."""
    return {
        "workload": "C2 Mamba-2 2.7B prefill: causal_conv1d_fn fwd+bwd, bf16, x (8, 5376, 2048) channel-last, "
                    "width 4, bias, SiLU, initial_states, return_final_states",
        "global_batch": world * B, "seq_len": L, "dim": D, "width": W,
        "parallelism": f"batch-sharded x{world}" + (
            ", dweight|dbias summed over ranks inside the reduction kernel over NVLink peer memory"
            if world > 1 else ""),
        "l2": "inputs larger than L2 (x and grad_out are 176 MB each; L2 is 126 MB)",
    }


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    state, cores = cpu_setup()
    for _ in range(args.warmup):
        cpu_sample_step(state)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter_ns()
        cpu_sample_step(state)
        times.append((time.perf_counter_ns() - t0) / 1e9)
    # The reference's own CPU timing method: the minimum over samples of
    # perf_counter_ns around each call (scripts/plot_bench.py:225-243).
    ms = 1e3 * min(times)
    value = L / (ms / 1e3)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "ms_per_step_unit": f"one step = one C2 batch row (1, {D}, {L}) fwd+bwd on the host cores, the minimum "
                            f"over the {len(times)} timed steps; the C2 batch has {B} such rows",
        "ms_per_step_mean": 1e3 * sum(times) / len(times),
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": c2_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"batch row 0 (1, {D}, {L}) of C2 per step (tokens/s of that row, all host "
                                   f"threads, min over steps); reference CPU algorithm (oracle/cc1d_oracle.c, "
                                   f"restating fwd_cpu/bwd_full_cpu kernel.mojo)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_only(args):
    """Launch one op of one config `args.reps` times (for profilers); prints
    the average CUDA-event time per launch."""
    from causal_conv1d_b200 import _ops

    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(5)

    def rn(*s, dt=DT):
        return torch.randn(*s, generator=g, device="cuda", dtype=torch.float32).to(dt)

    def ru(*s, dt=DT):
        return (torch.rand(*s, generator=g, device="cuda", dtype=torch.float32) - 0.5).to(dt)

    op = args.only
    if op in ("fwd_c2", "bwd_c2"):
        x, w, b, init, dout = make_c2(0, "cuda")
        out, fs, dx = torch.empty_like(x), torch.empty_like(init), torch.empty_like(x)
        dwdb = torch.empty(D * (W + 1), dtype=torch.float32, device="cuda")
        dw, db, dinit = torch.empty(D, W, dtype=DT, device="cuda"), torch.empty(D, dtype=DT, device="cuda"), \
            torch.empty_like(init)
        fn = (lambda: _ops.fwd(x, w, b, None, init, out, True, fs)) if op == "fwd_c2" else \
            (lambda: _ops.bwd(x, w, b, dout, None, init, None, dx, dwdb, dinit, dw, db, True))
    elif op in ("fwd_c5", "bwd_c5"):
        B5, D5, L5 = args.c5_batch, 8192, 8192
        x, dout = rn(B5, D5, L5), rn(B5, D5, L5)
        w5, b5, init = ru(D5, W), ru(D5), rn(B5, D5, W - 1)
        out, dx, fs, dinit = torch.empty_like(x), torch.empty_like(x), torch.empty_like(init), torch.empty_like(init)
        dwdb = torch.empty(D5 * (W + 1), dtype=torch.float32, device="cuda")
        dw, db = torch.empty(D5, W, dtype=DT, device="cuda"), torch.empty(D5, dtype=DT, device="cuda")
        fn = (lambda: _ops.fwd(x, w5, b5, None, init, out, True, fs)) if op == "fwd_c5" else \
            (lambda: _ops.bwd(x, w5, b5, dout, None, init, None, dx, dwdb, dinit, dw, db, True))
    elif op in ("fwd_c4", "bwd_c4"):
        dt = torch.float16
        Lv, Dv = 65536, 4096
        gl = torch.Generator().manual_seed(0)
        raw = torch.randint(256, 4097, (32,), generator=gl)
        lens = (raw * Lv // raw.sum()).clamp(min=1)
        lens[-1] += Lv - lens.sum()
        seq = torch.repeat_interleave(torch.arange(32, dtype=torch.int32), lens).view(1, Lv).cuda()
        x, dout = rn(1, Lv, Dv, dt=dt).transpose(1, 2), rn(1, Lv, Dv, dt=dt).transpose(1, 2)
        wv, bv = ru(Dv, W, dt=dt), ru(Dv, dt=dt)
        out, dx = torch.empty_like(x), torch.empty_like(x)
        dwdb = torch.empty(Dv * (W + 1), dtype=torch.float32, device="cuda")
        dw, db = torch.empty(Dv, W, dtype=dt, device="cuda"), torch.empty(Dv, dtype=dt, device="cuda")
        fn = (lambda: _ops.fwd(x, wv, bv, seq, None, out, True, None)) if op == "fwd_c4" else \
            (lambda: _ops.bwd(x, wv, bv, dout, seq, None, None, dx, dwdb, None, dw, db, True))
    elif op in ("update_c3a", "update_c3b", "update_burst4", "update_c3a_chanlast", "update_c3b_chanlast"):
        Bu, Du = 256, 5376
        w, b = ru(Du, W), ru(Du)
        x = rn(Bu, Du, 4 if op == "update_burst4" else 1)
        out = torch.empty_like(x)
        if op in ("update_burst4", "update_c3a_chanlast"):
            pool = rn(512, Du, W - 1) if op == "update_burst4" else rn(512, W - 1, Du).transpose(1, 2)
            idx = torch.randperm(512, device="cuda")[:Bu].to(torch.int32)
            fn = lambda: _ops.update(x, pool, w, b, None, idx, out, True)  # noqa: E731
        elif op == "update_c3a":
            pool = rn(512, Du, W - 1)
            idx = torch.randperm(512, device="cuda")[:Bu].to(torch.int32)
            fn = lambda: _ops.update(x, pool, w, b, None, idx, out, True)  # noqa: E731
        else:
            state = rn(Bu, Du, 8) if op == "update_c3b" else rn(Bu, 8, Du).transpose(1, 2)
            cache = torch.randint(0, 1024, (Bu,), device="cuda", dtype=torch.int32)
            fn = lambda: _ops.update(x, state, w, b, cache, None, out, True)  # noqa: E731
    else:
        raise SystemExit(f"unknown op {op}")
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.reps):
        fn()
    c.record()
    torch.cuda.synchronize()
    print(json.dumps({"op": op, "reps": args.reps, "ms_per_launch_eager": a.elapsed_time(c) / args.reps}))
    return 0


def load_traffic():
    p = REPO / "profiles" / "ncu_traffic.json"
    if p.is_file():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return {}
    return {}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-kernels", action="store_true", help="skip the secondary kernel table")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-c5", action="store_true", help="skip the C5 sweep (BASELINE configs[4])")
    ap.add_argument("--skip-decode", action="store_true", help="skip the batch-sharded decode rows")
    ap.add_argument("--only", default=None,
                    help="launch one op alone (fwd_c2, bwd_c2, update_c3a, update_c3b, update_burst4, "
                         "update_c3a_chanlast, update_c3b_chanlast, fwd_c4, bwd_c4, fwd_c5, bwd_c5) --reps times, for profilers; "
                         "prints no contract line")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--c5-batch", type=int, default=64, help="batch of the C5 shape in --only mode")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.only:
        return run_only(args)
    if args.impl == "reference":
        return run_reference(args)

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = init_dist(world, local)
    peak, peak_kind = peaks()
    fwd_bytes, bwd_bytes = c2_bytes()

    reducer = split_reducer = None
    if world > 1:
        from causal_conv1d_b200.parallel import PeerReducer

        reducer = PeerReducer(D, W, torch.device("cuda", local))
        split_reducer = PeerReducer(D, W, torch.device("cuda", local))
    r = time_c2(args, world, rank, reducer, split_reducer)
    e2e = None if args.skip_e2e else time_e2e(args, world, rank, reducer)
    c5 = None if args.skip_c5 else time_c5_sweep(world, rank, local, peak)
    decode = None if args.skip_decode else time_decode_sharded(world, rank, peak)
    kernels = None
    if rank == 0 and not args.skip_kernels:
        kernels = time_kernels(peak)
    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        cpu = cpu_baseline()
    if world > 1:
        dist.barrier()

    if rank == 0:
        fwd_gbs = fwd_bytes / r["fwd_ms"] / 1e6
        bwd_gbs = bwd_bytes / r["bwd_ms"] / 1e6
        traffic = load_traffic().get("bwd_chan_kernel/C2")
        ktab = {
            "fwd_c2": dict(ms=r["fwd_ms"], gbs=fwd_gbs, frac=fwd_gbs / peak, algorithmic_bytes=fwd_bytes),
            "bwd_c2": dict(ms=r["bwd_ms"], gbs=bwd_gbs, frac=bwd_gbs / peak, algorithmic_bytes=bwd_bytes,
                           note="bwd kernel + dweight/dbias finalize kernel" + (
                               " (fused with the cross-rank sum, so it includes waiting for peers)"
                               if world > 1 else "")),
        }
        if kernels:
            ktab.update(kernels)
        if c5 is not None and world == 1:
            # The sweep's width-4 SiLU row on one GPU is the C5 kernel line.
            row = next(x for x in c5["shardings"]["single"]["rows"] if x["width"] == W and x["silu"])
            for op in ("fwd", "bwd"):
                ms, nb = row[f"{op}_ms"], row[f"{op}_bytes_per_gpu"]
                ktab[f"{op}_c5_large"] = dict(ms=ms, gbs=nb / ms / 1e6, frac=nb / ms / 1e6 / peak,
                                              tokens_per_s=C5_B * C5_L / (ms / 1e3), algorithmic_bytes=nb)
        line = {
            "metric": METRIC,
            "value": world * B * L / (r["ms_per_step"] / 1e3),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": r["ms_per_step"],
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": c2_config(world),
            "roofline": {
                "bound": "hbm", "achieved": bwd_gbs, "peak": peak, "unit": "GB/s", "frac": bwd_gbs / peak,
                "traffic": traffic, "kernel": "bwd (bwd_chan_kernel + finalize_kernel), C2",
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback 6.65 TB/s",
                "algorithmic_bytes_per_launch": bwd_bytes,
            },
            "kernels": ktab,
            "gpu_launches": (4 if r.get("exchange", {}).get("used") == "split" else 3) * args.steps,
            "clocks": r["clocks"],
            "parity": {k: v for k, v in (("peer_reduction", r.get("parity")), ("c2_step", r.get("parity_c2")))
                       if v is not None},
        }
        if "per_rank" in r:
            line["per_rank"] = r["per_rank"]
        if "exchange" in r:
            line["exchange"] = r["exchange"]
        if c5 is not None:
            line["c5_sweep"] = c5
        if decode is not None:
            line["decode_sharded"] = decode
        if e2e is not None:
            line["e2e"] = e2e
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        reducer.close()
        split_reducer.close()
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
