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


def time_c2(args, world, rank, reducer):
    from causal_conv1d_b200 import _ops

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

    with Clocks(torch.cuda.current_device()) as clk:
        # The sampler starts before the warm-up so that it is already
        # reporting when the timed steps run.
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        # The timed step is replayed from a CUDA graph (captured once), as a
        # serving / training loop would; every replay launches the same
        # kernels on the same buffers.
        g_step = graph_of(step)
        for _ in range(args.warmup):
            g_step.replay()
        barrier_sync(world)
        clk.mark()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(K):
            g_step.replay()
        stop.record()
        torch.cuda.synchronize()
        clk.unmark()
    total_ms = start.elapsed_time(stop)
    # Per-op kernel times: graphs of the op alone, replayed back to back.
    reps = max(20, min(200, K // 10))
    fwd_ms = graph_ms(graph_of(fwd, 10), reps, 10)
    bwd_ms = graph_ms(graph_of(bwd, 10), reps, 10)
    del g_step
    barrier_sync(world)
    total_ms = max_over_ranks(total_ms, world)
    return dict(ms_per_step=total_ms / K, fwd_ms=fwd_ms, bwd_ms=bwd_ms, clocks=clk.summary())


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

    # Next rows of the path: a 4-token decode burst (speculative decoding) on
    # the C3a pool, and the C3a step with a channel-last conv_state pool
    # (strides (3*D, 1, D)); both use the generic update kernel.
    Lb = 4
    xs = [rn(Bu, Du, Lb) for _ in range(sets)]
    pools = [rn(512, Du, W - 1) for _ in range(sets)]
    outs = [torch.empty_like(xs[0]) for _ in range(sets)]
    ms = _kernel_ms(lambda i: _ops.update(xs[i], pools[i], w, b, None, idx[i], outs[i], True), 800, sets)
    nbytes = Bu * Du * (2 * Lb + 2 * Lb + 6 + 6) + Du * (W + 1) * 2 + Bu * 4
    res["update_burst4_indexed"] = dict(ms=ms, gbs=nbytes / ms / 1e6, frac=nbytes / ms / 1e6 / peak,
                                        tokens_per_s=Bu * Lb / (ms / 1e3), algorithmic_bytes=nbytes,
                                        note="x (256, 5376, 4), pool (512, 5376, 3), generic update kernel")
    del xs, pools, outs
    xs = [rn(Bu, Du, 1) for _ in range(sets)]
    pools = [rn(512, W - 1, Du).transpose(1, 2) for _ in range(sets)]
    outs = [torch.empty_like(xs[0]) for _ in range(sets)]
    ms = _kernel_ms(lambda i: _ops.update(xs[i], pools[i], w, b, None, idx[i], outs[i], True), 800, sets)
    nbytes = Bu * Du * (2 + 2 + 6 + 6) + Du * (W + 1) * 2 + Bu * 4
    res["update_c3a_chanlast_state"] = dict(ms=ms, gbs=nbytes / ms / 1e6, frac=nbytes / ms / 1e6 / peak,
                                            tokens_per_s=Bu / (ms / 1e3), algorithmic_bytes=nbytes,
                                            note="C3a with conv_state pool stored (512, 3, 5376), generic kernel")
    del xs, pools, outs
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

    # C5: large contiguous (64, 8192, 8192) bf16, width 4, SiLU, states on.
    B5, D5, L5 = 64, 8192, 8192
    x = rn(B5, D5, L5)
    out = torch.empty_like(x)
    w5, b5 = ru(D5, W), ru(D5)
    init = rn(B5, D5, W - 1)
    fs = torch.empty_like(init)
    n = B5 * D5 * L5
    ms = _kernel_ms(lambda i: _ops.fwd(x, w5, b5, None, init, out, True, fs), 5, 1)
    nb = 4 * n + 2 * init.numel() * 2 + D5 * (W + 1) * 2
    res["fwd_c5_large"] = dict(ms=ms, gbs=nb / ms / 1e6, frac=nb / ms / 1e6 / peak,
                               tokens_per_s=B5 * L5 / (ms / 1e3), algorithmic_bytes=nb)
    dout = out  # reuse the buffer as grad_out (values irrelevant for timing)
    dx = torch.empty_like(x)
    dwdb = torch.empty(D5 * (W + 1), dtype=torch.float32, device="cuda")
    dw, db, dinit = torch.empty(D5, W, dtype=DT, device="cuda"), torch.empty(D5, dtype=DT, device="cuda"), \
        torch.empty_like(init)
    ms = _kernel_ms(lambda i: _ops.bwd(x, w5, b5, dout, None, init, None, dx, dwdb, dinit, dw, db, True), 5, 1)
    nb = 6 * n + 2 * init.numel() * 2 + D5 * (W + 1) * (2 + 2 + 4)
    res["bwd_c5_large"] = dict(ms=ms, gbs=nb / ms / 1e6, frac=nb / ms / 1e6 / peak,
                               tokens_per_s=B5 * L5 / (ms / 1e3), algorithmic_bytes=nb)
    del x, out, dx
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
    ms = 1e3 * sum(times) / len(times)
    value = L / (ms / 1e3)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": c2_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"batch row 0 (1, {D}, {L}) of C2 per step (tokens/s of that row, all host "
                                   f"threads); reference CPU algorithm (oracle/cc1d_oracle.c, restating "
                                   f"fwd_cpu/bwd_full_cpu kernel.mojo)"},
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
    elif op in ("update_c3a", "update_c3b", "update_burst4", "update_c3a_chanlast"):
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
            state = rn(Bu, Du, 8)
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
    ap.add_argument("--only", default=None,
                    help="launch one op alone (fwd_c2, bwd_c2, update_c3a, update_c3b, update_burst4, "
                         "update_c3a_chanlast, fwd_c4, bwd_c4, fwd_c5, bwd_c5) --reps times, for profilers; "
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

    reducer = None
    if world > 1:
        from causal_conv1d_b200.parallel import PeerReducer

        reducer = PeerReducer(D, W, torch.device("cuda", local))
    r = time_c2(args, world, rank, reducer)
    e2e = None if args.skip_e2e else time_e2e(args, world, rank, reducer)
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
            "gpu_launches": 3 * args.steps,
            "clocks": r["clocks"],
        }
        if e2e is not None:
            line["e2e"] = e2e
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        reducer.close()
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
