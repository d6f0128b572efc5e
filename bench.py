"""Benchmark of the hyper-connections hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {b200,reference}]

Headline workload (one "step" = one forward + one backward of the fused
hyper-connection step over one batch): x [16,1024,4,768] bf16 streams, f
[16,1024,768] bf16 layer output, per-token H [.,4,4] = expm(skew), alpha/beta
= softmax, all float32, upstream gradients ~ N(0,1); seeded synthetic data
(the reference publishes no dataset for this path).

Metric: algorithmic HBM bytes of the fused forward + backward per second,
where every tensor is counted once:
  fwd  T*((2nD + 2D)*2 + (n^2 + 2n)*4)  bytes  (read x, f, H, alpha, beta; write u, x_out)
  bwd  T*((3nD + 3D)*2 + 2(n^2 + 2n)*4) bytes  (read g_u, g_x, x, f, H, alpha, beta;
                                                write grad_x, grad_f, grad_H, grad_alpha, grad_beta)
The batched matrix exponential (65,536 skew 4x4, forward + Frechet backward)
is reported alongside in matrices/s.

Timing: CUDA events on the launching stream around each kernel, L2 flushed
between steps outside the events (a 256 MiB write, then a 256 MiB read that
writes the flush's dirty lines back; ``write_flush`` repeats the step after
the write alone), barrier + synchronize
around the K timed steps, max over ranks. Under torchrun every rank runs one
full batch of the workload on its own GPU (its shard of an N x 16,384-token
global batch, seeded by rank) with no collective on the data path (weak
scaling); value = N * bytes / max-rank time.

``--impl reference`` times the reference's own CPU path for the same work,
the whole 16,384-token batch per step, with every host thread, on rank 0
only: the reference's read einsum (hyperconnections/cghc.py:410), write
einsum (:417) and its layer's eager stream mix (_stream_mix_eager,
:365-392) under bf16 autocast, with autograd backward. The reference is
imported from baseline/_ref (baseline/install_reference.py); where it is
absent, the oracle's op-for-op restatement of the same path runs instead and
the line says so ("kind": "port").
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import threading
import time

import numpy as np
import torch

METRIC = "stream-mix fwd+bwd HBM GB/s (% of 8 TB/s); batched expm matrices/sec"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
ROOT = os.path.dirname(os.path.abspath(__file__))

# ---------------------------------------------------------------- workloads
BATCH, SEQ, N_STREAMS, BLOCK = 16, 1024, 4, 768
TOKENS = BATCH * SEQ
EXPM_BATCH, EXPM_N = 65536, 4


def fused_bytes(T: int, n: int, D: int, esize: int = 2) -> tuple[int, int]:
    """Algorithmic bytes (each tensor touched once) of the fused fwd and bwd."""
    small = (n * n + 2 * n) * 4
    fwd = T * ((2 * n * D + 2 * D) * esize + small)
    bwd = T * ((3 * n * D + 3 * D) * esize + 2 * small)
    return fwd, bwd


def fused_workload(T: int, n: int, D: int, dtype=torch.bfloat16, seed: int = 0):
    """x, f, H, alpha, beta, g_u, g_x drawn in this order from one CPU generator:
    x, f ~ N(0,1); H = expm(S - S^T), S = strict upper triangle of 0.5*N(0,1)
    (a skew-symmetric generator whose off-diagonal entries are N(0, 0.5^2));
    alpha, beta = softmax of N(0,1) logits; g_u, g_x ~ N(0,1)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, n, D, generator=g).to(dtype)
    f = torch.randn(T, D, generator=g).to(dtype)
    S = torch.triu(0.5 * torch.randn(T, n, n, generator=g), 1)
    H = torch.linalg.matrix_exp(S - S.mT).contiguous()
    alpha = torch.softmax(torch.randn(T, n, generator=g), -1)
    beta = torch.softmax(torch.randn(T, n, generator=g), -1)
    g_u = torch.randn(T, D, generator=g).to(dtype)
    g_x = torch.randn(T, n, D, generator=g).to(dtype)
    return x, f, H, alpha, beta, g_u, g_x


def expm_workload(B: int, n: int, seed: int = 0):
    """A = 0.5 (G - G^T) / 2 with G ~ N(0,1), then an upstream gradient ~ N(0,1)."""
    g = torch.Generator().manual_seed(seed)
    M = torch.randn(B, n, n, generator=g)
    A = (0.5 * (M - M.mT) / 2).contiguous()
    G = torch.randn(B, n, n, generator=g)
    return A, G


# ---------------------------------------------------------------- clocks
_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
    0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML (read-only) in a
    background thread; ``window(t0, t1)`` summarises the samples taken while
    the timed region ran."""

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples: list[tuple[float, int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(visible.split(",")[device_index]) if visible else device_index
            self._h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self._nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML missing: report no clocks rather than guess
            self._nvml = None
        self.period = period_s

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((time.perf_counter(), mhz, reasons))
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def window(self, t0: float, t1: float) -> dict:
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        if not inside:  # very short windows: take the nearest samples
            inside = sorted(self.samples, key=lambda s: min(abs(s[0] - t0), abs(s[0] - t1)))[:3]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mask = 0
        for s in inside:
            mask |= s[2]
        reasons = [name for bit, name in _REASONS.items() if mask & bit and name != "gpu_idle"]
        return {
            "sm_mhz": float(np.median([s[1] for s in inside])),
            "sm_max_mhz": self.max_mhz,
            "reasons": reasons,
            "samples": len(inside),
        }


# ---------------------------------------------------------------- helpers
def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def committed_traffic(kernel: str):
    """DRAM bytes per launch from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as fh:
            return json.load(fh).get(kernel)
    except Exception:
        return None


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(value: float, world: int, device) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def gather_ranks(value: float, world: int, device) -> list:
    """Every rank's value, in rank order (one all-gather; [value] at N = 1)."""
    if world == 1:
        return [value]
    t = torch.tensor([value], dtype=torch.float64, device=device)
    out = [torch.zeros_like(t) for _ in range(world)]
    torch.distributed.all_gather(out, t)
    return [float(x.item()) for x in out]


def barrier(world: int):
    if world > 1:
        torch.distributed.barrier()


class numa_local:
    """Runs its body on the host CPUs nearest to a GPU (NVML's CPU affinity of
    the device, read-only), then restores the thread's affinity. Pinned host
    buffers allocated inside land on that GPU's NUMA node (first touch), so
    their DMA does not cross the socket interconnect. No-op where NVML or
    sched_setaffinity is unavailable."""

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.saved = None

    def _gpu_cpus(self):
        import pynvml

        pynvml.nvmlInit()
        visible = os.environ.get("CUDA_VISIBLE_DEVICES")
        idx = int(visible.split(",")[self.device_index]) if visible else self.device_index
        h = pynvml.nvmlDeviceGetHandleByIndex(idx)
        words = (os.cpu_count() + 63) // 64
        mask = pynvml.nvmlDeviceGetCpuAffinity(h, words)
        return {64 * w + b for w, m in enumerate(mask) for b in range(64) if (m >> b) & 1}

    def __enter__(self):
        try:
            cpus = self._gpu_cpus() & os.sched_getaffinity(0)
            if cpus:
                self.saved = os.sched_getaffinity(0)
                os.sched_setaffinity(0, cpus)
        except Exception:
            self.saved = None
        return self

    def __exit__(self, *exc):
        if self.saved is not None:
            os.sched_setaffinity(0, self.saved)
        return False


# ---------------------------------------------------------------- B200 arm
class FusedRunner:
    """Direct C-ABI launches of the fused forward and backward on resident
    device buffers (the kernels timed for ``value``)."""

    def __init__(self, device, T=TOKENS, n=N_STREAMS, D=BLOCK, seed=0, shard=None):
        from hyperconnections_b200 import _lib

        self.lib = _lib.lib()
        host = fused_workload(T, n, D, seed=seed)
        if shard is not None:  # (rank, world): this rank's contiguous slice of the seeded batch
            rank, world = shard
            lo, hi = T * rank // world, T * (rank + 1) // world
            host = [t[lo:hi].contiguous() for t in host]
            T = hi - lo
        self.T, self.n, self.D = T, n, D
        self.x, self.f, self.H, self.alpha, self.beta, self.g_u, self.g_x = [t.to(device) for t in host]
        dt = self.x.dtype
        self.u = torch.empty(T, D, dtype=dt, device=device)
        self.x_out = torch.empty_like(self.x)
        self.grad_x = torch.empty_like(self.x)
        self.grad_f = torch.empty(T, D, dtype=dt, device=device)
        self.grad_H = torch.empty(T, n, n, device=device)
        self.grad_a = torch.empty(T, n, device=device)
        self.grad_b = torch.empty(T, n, device=device)
        self.code = _lib.dtype_code(dt)
        self.stream = torch.cuda.current_stream(device).cuda_stream
        self._check = _lib.check

    def fwd(self):
        rc = self.lib.hc_fused_fwd(
            self.x.data_ptr(), self.f.data_ptr(), self.H.data_ptr(), self.alpha.data_ptr(),
            self.beta.data_ptr(), self.u.data_ptr(), self.x_out.data_ptr(), self.T, self.n, self.D,
            self.code, self.stream)
        self._check(rc, "hc_fused_fwd")

    def bwd(self):
        rc = self.lib.hc_fused_bwd(
            self.g_u.data_ptr(), self.g_x.data_ptr(), self.x.data_ptr(), self.f.data_ptr(),
            self.H.data_ptr(), self.alpha.data_ptr(), self.beta.data_ptr(), self.grad_x.data_ptr(),
            self.grad_f.data_ptr(), self.grad_H.data_ptr(), self.grad_a.data_ptr(), self.grad_b.data_ptr(),
            self.T, self.n, self.D, self.code, self.stream)
        self._check(rc, "hc_fused_bwd")


class L2Flush:
    """Evicts L2 (126 MB) between timed steps, outside the events. "clean"
    (the default): a 256 MiB write, so that no input of the step stays in L2,
    then a 256 MiB read of another buffer, which writes the first buffer's
    dirty lines back before the step starts; the step begins cold on a clean
    L2, the state ncu's cache control gives a profiled kernel. "write": the
    write alone; the timed step then also pays the write-back of up to ~126 MB
    of the flush's own dirty lines."""

    def __init__(self, device, mode: str = "clean"):
        words = 256 * 1024 * 1024 // 4
        self.w = torch.empty(words, dtype=torch.float32, device=device)
        self.r = torch.ones(words, dtype=torch.float32, device=device) if mode == "clean" else None
        self.sink = torch.empty((), dtype=torch.float32, device=device)

    def __call__(self, i: int):
        self.w.fill_(float(i))
        if self.r is not None:
            torch.sum(self.r, dim=0, out=self.sink)


def time_fused(device, steps, warmup, world, T=TOKENS, n=N_STREAMS, D=BLOCK, seed=0, shard=None, flush_mode="clean"):
    """Two timed passes of `steps` fused steps each, L2 flushed before every
    step outside the events. Pass 1 records events only around the step
    (forward then backward back to back, as a training step runs them: the
    backward's CTAs may start on SMs the forward has left, programmatic
    dependent launch); its times are the headline. Pass 2 adds an event between
    the kernels for the per-kernel split and the dominant kernel's roofline."""
    runner = FusedRunner(device, T=T, n=n, D=D, seed=seed, shard=shard)
    flush = L2Flush(device, flush_mode)
    for i in range(warmup):
        flush(i)
        runner.fwd()
        runner.bwd()
    torch.cuda.synchronize(device)
    barrier(world)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    steps_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(steps)]
    for i in range(steps):
        flush(i)  # evict L2 between steps, outside the events
        e = steps_ev[i]
        e[0].record()
        runner.fwd()
        runner.bwd()
        e[1].record()
    torch.cuda.synchronize(device)
    barrier(world)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    for i in range(steps):
        flush(i)
        e = evs[i]
        e[0].record()
        runner.fwd()
        e[1].record()
        runner.bwd()
        e[2].record()
    torch.cuda.synchronize(device)
    t2 = time.perf_counter()
    step_ms = [e[0].elapsed_time(e[1]) for e in steps_ev]
    fwd_ms = [e[0].elapsed_time(e[1]) for e in evs]
    bwd_ms = [e[1].elapsed_time(e[2]) for e in evs]
    del flush
    return {"step_ms": step_ms, "fwd_ms": fwd_ms, "bwd_ms": bwd_ms, "wall": (t0, t2), "launches": 2 * steps}


class ExpmRunner:
    """Direct C-ABI launches of the batched T18 expm forward and backward
    (global scaling, the reference's semantics) on resident device buffers."""

    def __init__(self, device, B=EXPM_BATCH, n=EXPM_N, seed=0):
        from hyperconnections_b200 import _lib

        self.lib = _lib.lib()
        self.B, self.n = B, n
        self.A, self.G = (t.to(device) for t in expm_workload(B, n, seed=seed))
        self.E = torch.empty_like(self.A)
        self.dA = torch.empty_like(self.A)
        self.words = max(1, self.lib.hc_expm_t18_scratch_words(B, n))
        self.scratch = torch.empty(self.words, dtype=torch.float32, device=device)
        self.stream = torch.cuda.current_stream(device).cuda_stream
        self._check = _lib.check

    def fwd(self):
        rc = self.lib.hc_expm_t18_fwd(self.A.data_ptr(), self.E.data_ptr(), self.B, self.n,
                                      self.scratch.data_ptr(), self.words, 0, self.stream)
        self._check(rc, "hc_expm_t18_fwd")

    def bwd(self):
        # mode 2: reuse the partial maxima of A that the forward left in scratch
        rc = self.lib.hc_expm_t18_bwd(self.A.data_ptr(), self.G.data_ptr(), self.dA.data_ptr(), self.B, self.n,
                                      self.scratch.data_ptr(), self.words, 2, self.stream)
        self._check(rc, "hc_expm_t18_bwd")


def time_expm(device, steps, warmup, B=EXPM_BATCH, n=EXPM_N, split=False):
    """Device time of one expm forward + backward over B resident matrices
    (C-ABI launches), L2 flushed between steps; ms per step (and, with
    split=True, also the forward's ms per step)."""
    runner = ExpmRunner(device, B, n)
    flush = L2Flush(device)
    for _ in range(warmup):
        runner.fwd()
        runner.bwd()
    torch.cuda.synchronize(device)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    for i in range(steps):
        flush(i)
        evs[i][0].record()
        runner.fwd()
        evs[i][1].record()
        runner.bwd()
        evs[i][2].record()
    torch.cuda.synchronize(device)
    del flush
    step = [e[0].elapsed_time(e[2]) for e in evs]
    return (step, [e[0].elapsed_time(e[1]) for e in evs]) if split else step


def time_expm_api(device, steps, warmup):
    """The same work through the public API (``expm_t18`` + autograd, whose
    Function is C++ over the C ABI), which adds the host cost of autograd and
    of allocating outputs and scratch."""
    from hyperconnections_b200.ops import expm_t18

    A, G = (t.to(device) for t in expm_workload(EXPM_BATCH, EXPM_N))

    def step():
        a = A.detach().requires_grad_(True)
        E = expm_t18(a)
        E.backward(G)
        return a.grad

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize(device)
    return e0.elapsed_time(e1) / steps


def time_e2e(device, steps, warmup):
    """The same fused step through the public API (autograd) with inputs in
    pinned host memory: every step copies its inputs host->device and reads
    every output back device->host.

    Three streams, as a training input pipeline would run it: the upload of
    step i+1 (copy stream) overlaps the download of step i (download
    stream), so both PCIe directions are busy at once; the kernels run on the
    current stream between them, ordered by events."""
    from hyperconnections_b200.ops import stream_mix_fused

    with numa_local(device.index):
        host = [t.pin_memory() for t in fused_workload(TOKENS, N_STREAMS, BLOCK, seed=1)]
    h2d = sum(t.numel() * t.element_size() for t in host)
    comp = torch.cuda.current_stream(device)
    up = torch.cuda.Stream(device)
    down = torch.cuda.Stream(device)
    outs_host = None

    def step():
        nonlocal outs_host
        with torch.cuda.stream(up):
            dev = [t.to(device, non_blocking=True) for t in host]
        comp.wait_stream(up)
        for t in dev:
            t.record_stream(comp)
        x, f, H, a, b, g_u, g_x = dev
        leaves = [t.requires_grad_(True) for t in (x, f, H, a, b)]
        u, x_out = stream_mix_fused(*leaves)
        torch.autograd.backward([u, x_out], [g_u, g_x])
        outs = [u.detach(), x_out.detach()] + [t.grad for t in leaves]
        if outs_host is None:
            with numa_local(device.index):
                outs_host = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in outs]
        down.wait_stream(comp)
        with torch.cuda.stream(down):
            for dst, src in zip(outs_host, outs):
                src.record_stream(down)
                dst.copy_(src, non_blocking=True)
        return sum(o.numel() * o.element_size() for o in outs)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    up.wait_stream(comp)
    down.wait_stream(comp)
    d2h = 0
    for _ in range(steps):
        d2h = step()
    comp.wait_stream(down)
    e1.record(comp)
    torch.cuda.synchronize(device)
    return e0.elapsed_time(e1) / steps, h2d, d2h


def time_host_copies(device, steps, warmup):
    """The end-to-end leg's host<->device traffic alone, its ceiling: every
    step copies the same pinned inputs host->device on one stream while
    output-shaped device buffers are copied device->host on another (both
    PCIe directions at once, as in time_e2e), with no kernels and no autograd.
    Returns ms per step."""
    with numa_local(device.index):
        host_in = [t.pin_memory() for t in fused_workload(TOKENS, N_STREAMS, BLOCK, seed=1)]
    x, f, H, a, b, g_u, g_x = host_in
    # the step's outputs: u, x', grad_x, grad_f, grad_H, grad_alpha, grad_beta
    dev_in = [torch.empty(t.shape, dtype=t.dtype, device=device) for t in host_in]
    dev_out = [torch.zeros(t.shape, dtype=t.dtype, device=device) for t in (g_u, g_x, x, f, H, a, b)]
    with numa_local(device.index):
        host_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in dev_out]
    comp = torch.cuda.current_stream(device)
    up = torch.cuda.Stream(device)
    down = torch.cuda.Stream(device)

    def step():
        with torch.cuda.stream(up):
            for dst, src in zip(dev_in, host_in):
                dst.copy_(src, non_blocking=True)
        with torch.cuda.stream(down):
            for dst, src in zip(host_out, dev_out):
                dst.copy_(src, non_blocking=True)

    up.wait_stream(comp)
    down.wait_stream(comp)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    up.wait_stream(comp)
    down.wait_stream(comp)
    for _ in range(steps):
        step()
    comp.wait_stream(up)
    comp.wait_stream(down)
    e1.record(comp)
    torch.cuda.synchronize(device)
    return e0.elapsed_time(e1) / steps


# ---------------------------------------------------------------- CPU baseline
def reference_cpu_path():
    """The reference's own eager CPU path for the fused step and for
    expm_t18, imported from baseline/_ref: returns (fused_step, expm_step,
    kind). Each step runs forward + autograd backward on CPU tensors. Falls
    back to the oracle's restatement (kind "port") when the reference is not
    installed."""
    try:
        from baseline import reference_env

        if reference_env.available():
            hc = reference_env.import_reference()
            from einops import einsum

            from hyperconnections.ops.expm import expm_t18

            body = expm_t18._torchdynamo_orig_callable  # uncompiled body of ops/expm.py:69-106
            layer = hc.cghc.ContinuousGenHyperConnections(N_STREAMS, 1, N_STREAMS * BLOCK, BLOCK, torch.nn.Identity(),
                                                          use_triton=False)

            def fused_step(x, f, H, alpha, beta, g_u, g_x):
                x, f, H, alpha, beta = (t.detach().requires_grad_(True) for t in (x, f, H, alpha, beta))
                with torch.autocast("cpu", dtype=torch.bfloat16):  # as the reference trains (experiments/cifar.py:272)
                    u = einsum(alpha[:, None, :], x, "b m n, b n d -> b m d")             # cghc.py:410
                    Y = einsum(beta[:, :, None], f[:, None, :], "b n m, b m d -> b n d")  # cghc.py:417
                    out = layer._stream_mix_eager(x, H, Y, None)                          # cghc.py:365-392
                torch.autograd.backward([u, out], [g_u[:, None, :].to(u.dtype), g_x.to(out.dtype)])
                return u, out

            def expm_step(A, G):
                A = A.detach().requires_grad_(True)
                E = body(A)
                E.backward(G)
                return E, A.grad

            return fused_step, expm_step, "reference"
    except Exception as exc:  # an unusable install: say so and use the restatement
        print(f"reference import failed ({exc!r}); timing the oracle's restatement", flush=True)
    from oracle.torch_ref import expm_t18_cpu, fused_step_cpu

    return fused_step_cpu, expm_t18_cpu, "port"


def cpu_fused_sample(tokens: int, budget_s: float, min_reps: int = 3):
    """The reference's CPU path on `tokens` tokens of the workload; returns
    (median seconds per rep, reps, threads, kind)."""
    fused_step, _, kind = reference_cpu_path()
    torch.set_num_threads(os.cpu_count() or 1)
    x, f, H, a, b, g_u, g_x = fused_workload(tokens, N_STREAMS, BLOCK, seed=2)
    fused_step(x, f, H, a, b, g_u, g_x)  # warm-up
    times = []
    t_start = time.perf_counter()
    while len(times) < min_reps or (time.perf_counter() - t_start < budget_s and len(times) < 50):
        t0 = time.perf_counter()
        fused_step(x, f, H, a, b, g_u, g_x)
        times.append(time.perf_counter() - t0)
    return float(np.median(times)), len(times), torch.get_num_threads(), kind


def cpu_expm_sample(batch: int, budget_s: float, min_reps: int = 3):
    _, expm_step, kind = reference_cpu_path()
    torch.set_num_threads(os.cpu_count() or 1)
    A, G = expm_workload(batch, EXPM_N, seed=3)
    expm_step(A, G)
    times = []
    t_start = time.perf_counter()
    while len(times) < min_reps or (time.perf_counter() - t_start < budget_s and len(times) < 50):
        t0 = time.perf_counter()
        expm_step(A, G)
        times.append(time.perf_counter() - t0)
    return float(np.median(times)), len(times), torch.get_num_threads(), kind


def cpu_model():
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


CONFIG = {
    "workload": "fused hyper-connection step fwd+bwd: x[16,1024,4,768] bf16, f[16,1024,768] bf16, "
                "H[16,1024,4,4]=expm(skew) fp32, alpha/beta[16,1024,4]=softmax fp32, seed 0",
    "tokens": TOKENS, "n_streams": N_STREAMS, "block_size": BLOCK,
    "l2": ("flushed between steps outside the timed events: a 256 MiB write, then a 256 MiB read that writes "
           "the flush's own dirty lines back (inputs cold, L2 clean); write_flush repeats the step with the "
           "write alone"),
}


def run_reference(args):
    """The reference arm: W untimed + K timed steps of the reference's CPU
    path over the whole workload (16,384 tokens per step)."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    fused_step, _, kind = reference_cpu_path()
    torch.set_num_threads(os.cpu_count() or 1)
    x, f, H, a, b, g_u, g_x = fused_workload(TOKENS, N_STREAMS, BLOCK, seed=0)
    for _ in range(args.warmup):
        fused_step(x, f, H, a, b, g_u, g_x)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fused_step(x, f, H, a, b, g_u, g_x)
    sec = (time.perf_counter() - t0) / args.steps
    fb, bb = fused_bytes(TOKENS, N_STREAMS, BLOCK)
    gbs = (fb + bb) / sec / 1e9
    what = ("the reference's own code from baseline/_ref: einops read einsum cghc.py:410, write einsum :417, "
            "ContinuousGenHyperConnections._stream_mix_eager :365-392" if kind == "reference" else
            "the oracle's op-for-op restatement of cghc.py:410, :417, :365-392 (reference not installed)")
    sample = (f"all {TOKENS} tokens of the workload per step, {args.steps} steps; {what}; bf16 autocast, "
              "autograd backward")
    line = {
        "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": CONFIG, "impl": "reference",
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": kind,
                         "sample": sample, "cpu": cpu_model()},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def time_model(spec, device, world, rank, steps, warmup):
    """One end-to-end training workload (e2e_models): tokens/s of the whole job
    at this N, step time as the max over ranks; for N > 1 also the all-reduce
    share: the step with every micro-batch under no_sync (no gradient
    all-reduce) timed after the real steps, and one NCCL all-reduce of the
    step's gradient volume on its own."""
    import e2e_models as em

    tr = em.Trainer(spec, device, world, rank)
    ms, loss, _ = em.time_steps(tr, steps, warmup, sync=True, barrier=lambda: barrier(world))
    step = float(np.mean(ms))
    step_max = max_over_ranks(step, world, device)
    out = {**em.describe(spec), "n_gpus": world, "local_batch": tr.local_batch, "micro_batch": tr.micro_batch,
           "params": tr.params, "steps": steps, "warmup": warmup, "ms_per_step": step_max,
           "rank_ms_per_step": gather_ranks(step, world, device),
           "tokens_per_s": tr.tokens_per_step / (step_max * 1e-3), "loss": loss, "loss_uniform": em.sanity(spec),
           "model_tflops_per_s": em.flops_per_token(spec) * tr.tokens_per_step / (step_max * 1e-3) / 1e12,
           "scaling": "strong (fixed global batch split over the ranks)"}
    if world > 1:
        ms_c, _, _ = em.time_steps(tr, max(2, steps // 2), 1, sync=False, barrier=lambda: barrier(world))
        comp_max = max_over_ranks(float(np.mean(ms_c)), world, device)
        ar_ms = max_over_ranks(em.time_allreduce(tr.grad_bytes, device, world), world, device)
        busbw = 2 * (world - 1) / world * tr.grad_bytes / (ar_ms * 1e-3) / 1e9
        out["allreduce"] = {"grad_bytes": tr.grad_bytes, "step_without_allreduce_ms": comp_max,
                            "exposed_ms": step_max - comp_max, "exposed_share": (step_max - comp_max) / step_max,
                            "standalone_ms": ar_ms, "standalone_bus_gbs": busbw,
                            "standalone_share_if_not_overlapped": ar_ms / step_max,
                            "how": "DDP bucketed NCCL all-reduce overlapped with the backward; exposed = step - "
                                   "step with every micro-batch under no_sync"}
    del tr
    torch.cuda.empty_cache()
    return out


def run_b200(args):
    world, rank, local = dist_env()
    if world > 1:
        from datetime import timedelta

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)

    from hyperconnections_b200 import _lib

    _lib.lib()  # fail loudly when the kernels are missing

    sampler = ClockSampler(local)
    sampler.start()
    if args.fused_only and (args.n, args.block) != (N_STREAMS, BLOCK):
        # another point of the n x D grid, 16,384 tokens (profiling captures)
        res = time_fused(device, args.steps, args.warmup, world, n=args.n, D=args.block, seed=dist_env()[1])
        fb, bb = fused_bytes(TOKENS, args.n, args.block)
        t0, t1 = res["wall"]
        if rank == 0:
            step = float(np.mean(res["step_ms"]))
            print(json.dumps({"fused_only": True, "tokens": TOKENS, "n": args.n, "D": args.block, "ms_per_step": step,
                              "value": (fb + bb) / (step * 1e-3) / 1e9, "unit": "GB/s",
                              "kernels_ms": {"hc_fused_fwd": float(np.mean(res["fwd_ms"])),
                                             "hc_fused_bwd": float(np.mean(res["bwd_ms"]))},
                              "clocks": sampler.window(t0, t1)}), flush=True)
        sampler.stop()
        return
    # rank r's shard: its own seeded batch of the workload (seed r)
    res = time_fused(device, args.steps, args.warmup, world, seed=dist_env()[1])
    t0, t1 = res["wall"]
    clocks = sampler.window(t0, t1)

    fwd_ms = float(np.mean(res["fwd_ms"]))
    bwd_ms = float(np.mean(res["bwd_ms"]))
    step_ms = float(np.mean(res["step_ms"]))
    step_ms_max = max_over_ranks(step_ms, world, device)
    rank_ms = gather_ranks(step_ms, world, device)
    fb, bb = fused_bytes(TOKENS, N_STREAMS, BLOCK)
    value = world * (fb + bb) / (step_ms_max * 1e-3) / 1e9

    if args.fused_only:  # the headline step alone (profiling captures, quick comparisons)
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                              "warmup": args.warmup, "ms_per_step": step_ms_max, "fused_only": True,
                              "kernels_ms": {"hc_fused_fwd": fwd_ms, "hc_fused_bwd": bwd_ms},
                              "rank_ms_per_step": rank_ms, "clocks": clocks}), flush=True)
        sampler.stop()
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return

    # the same step with the global batch fixed: rank r keeps its contiguous 1/N slice of the seed-0 batch
    if world > 1:
        strong = time_fused(device, args.steps, args.warmup, world, seed=0, shard=(rank, world))
        strong_ms = max_over_ranks(float(np.mean(strong["step_ms"])), world, device)
    else:
        strong_ms = step_ms_max
    strong_value = (fb + bb) / (strong_ms * 1e-3) / 1e9
    # the same step after a write-only L2 flush (see L2Flush)
    wf = time_fused(device, args.steps, args.warmup, world, seed=dist_env()[1], flush_mode="write")
    wf_ms = max_over_ranks(float(np.mean(wf["step_ms"])), world, device)
    write_flush = {"value": world * (fb + bb) / (wf_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": wf_ms,
                   "kernels_ms": {"hc_fused_fwd": float(np.mean(wf["fwd_ms"])),
                                  "hc_fused_bwd": float(np.mean(wf["bwd_ms"]))}}

    expm_ms, expm_fwd_ms = time_expm(device, max(5, min(args.steps, 50)), max(3, args.warmup), split=True)
    expm_step = float(np.mean(expm_ms))
    expm_step_max = max_over_ranks(expm_step, world, device)
    expm_rate = world * EXPM_BATCH / (expm_step_max * 1e-3)
    expm_fwd_max = max_over_ranks(float(np.mean(expm_fwd_ms)), world, device)
    expm_api_ms = max_over_ranks(time_expm_api(device, 50, 10), world, device)

    # 20 steps: the pipeline's fill and drain (one transfer each that nothing
    # overlaps) are then a small share of the timed region
    e2e_ms, h2d, d2h = time_e2e(device, max(3, min(args.steps, 20)), 2)
    e2e_ms_max = max_over_ranks(e2e_ms, world, device)
    e2e_value = world * (fb + bb) / (e2e_ms_max * 1e-3) / 1e9
    # the same copies without the step: the ceiling the host link puts on e2e
    # at this N (every rank copies at once); context only, so a failure here
    # records its reason instead of ending the run
    copy_err = None
    try:
        copy_ms = time_host_copies(device, max(3, min(args.steps, 20)), 2)
    except Exception as exc:  # noqa: BLE001
        copy_ms, copy_err = float("nan"), f"{type(exc).__name__}: {exc}"[:200]
    copy_ms_max = max_over_ranks(copy_ms, world, device)
    sampler.stop()

    models = {}
    if not args.no_models:
        import e2e_models as em

        for spec in (em.VIT, em.LM):
            models[spec.name] = time_model(spec, device, world, rank, steps=max(3, min(args.steps, 5)),
                                           warmup=3)

    if rank == 0:
        peak, peak_kind = measured_peak()
        dom_name, dom_ms, dom_bytes = ("hc_fused_bwd", bwd_ms, bb) if bwd_ms >= fwd_ms else ("hc_fused_fwd", fwd_ms, fb)
        achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": step_ms_max,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded)",
            "config": CONFIG,
            "pct_of_8tbs": 100.0 * value / world / NOMINAL_HBM_GBS,
            "pct_of_measured_hbm": 100.0 * value / world / peak,
            "kernels_ms": {"hc_fused_fwd": fwd_ms, "hc_fused_bwd": bwd_ms,
                           "note": "separate pass with an event between the kernels"},
            "rank_ms_per_step": rank_ms,
            "write_flush": write_flush,
            "strong_scaling": {"value": strong_value, "unit": "GB/s", "ms_per_step": strong_ms,
                               "tokens_per_rank": TOKENS // world,
                               "what": "the same step with the 16,384-token batch split over the ranks "
                                       "(rank r keeps its contiguous 1/N slice of the seed-0 batch)"},
            "roofline": {
                "bound": "hbm", "kernel": dom_name, "achieved": achieved, "peak": peak,
                "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                "traffic": committed_traffic(dom_name), "algorithmic_bytes": dom_bytes,
            },
            "expm": {"metric": "batched expm fwd+bwd matrices/s", "value": expm_rate, "unit": "matrices/s",
                     "ms_per_step": expm_step_max, "batch": EXPM_BATCH, "n": EXPM_N,
                     "scaling": "global (reference semantics)",
                     "fwd": {"value": world * EXPM_BATCH / (expm_fwd_max * 1e-3), "unit": "matrices/s",
                             "ms_per_step": expm_fwd_max},
                     "api": {"value": world * EXPM_BATCH / (expm_api_ms * 1e-3), "unit": "matrices/s",
                             "ms_per_step": expm_api_ms,
                             "path": "hyperconnections_b200.ops.expm_t18 + autograd (C++ Function)"}},
            "e2e": {"value": e2e_value, "unit": "GB/s", "ms_per_step": e2e_ms_max,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "hyperconnections_b200.ops.stream_mix_fused + autograd, pinned host buffers, "
                            "upload of step i+1 overlapping download of step i",
                    "copy_ceiling": ({"value": world * (fb + bb) / (copy_ms_max * 1e-3) / 1e9, "unit": "GB/s",
                                      "ms_per_step": copy_ms_max,
                                      "what": "the same H2D and D2H copies per step on two streams at once, "
                                              "no kernels, every rank at once"}
                                     if copy_ms_max == copy_ms_max and copy_ms_max > 0
                                     else {"unavailable": copy_err or "no finite time"})},
            "gpu_launches": res["launches"],
            "clocks": clocks,
        }
        if models:
            line["e2e_models"] = models
        if world == 1 and not args.no_cpu_baseline:
            sec, reps, threads, kind = cpu_fused_sample(TOKENS, budget_s=10.0)
            line["cpu_baseline"] = {
                "value": (fb + bb) / sec / 1e9, "unit": "GB/s", "cores": threads, "kind": kind,
                "sample": f"all {TOKENS} tokens of the workload per rep, median of {reps} reps (the reference's "
                          "eager CPU path: read einsum, write einsum, _stream_mix_eager; bf16 autocast, autograd)",
                "cpu": cpu_model(),
            }
            esec, ereps, ethreads, ekind = cpu_expm_sample(EXPM_BATCH, budget_s=8.0)
            line["expm"]["cpu_baseline"] = {
                "value": EXPM_BATCH / esec, "unit": "matrices/s", "cores": ethreads, "kind": ekind,
                "sample": f"{EXPM_BATCH} matrices per rep, median of {ereps} reps (the reference's uncompiled "
                          "expm_t18 body, ops/expm.py:69-106, + autograd)",
            }
            line["expm"]["speedup_vs_cpu"] = expm_rate / (EXPM_BATCH / esec)
        print(json.dumps(line), flush=True)

    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def rw_bytes(T: int, n: int, m: int, D: int, proj: bool, esize: int = 2) -> dict:
    """Algorithmic bytes (each tensor once) of the read and mix-write halves."""
    return {
        "read_fwd": T * ((n + m) * D * esize + m * n * 4),
        "read_bwd": T * ((m + 2 * n) * D * esize + 2 * m * n * 4),
        "mix_write_fwd": T * ((2 * n + m) * D * esize + (n * n + n * m + (n if proj else 0)) * 4),
        "mix_write_bwd": T * ((3 * n + 2 * m) * D * esize + (2 * (n * n + n * m) + (2 * n if proj else 0)) * 4),
    }


class RwRunner:
    """Direct C-ABI launches of the read and mix-write kernels (two-phase
    layer: read before the wrapped module, mix + write after it)."""

    def __init__(self, device, T, n, m, D, proj, seed=0):
        from hyperconnections_b200 import _lib

        self.lib, self._check = _lib.lib(), _lib.check
        self.T, self.n, self.m, self.D = T, n, m, D
        g = torch.Generator().manual_seed(seed)
        bf = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16).to(device)  # noqa: E731
        self.x, self.f, self.g_u, self.g_x = bf(T, n, D), bf(T, m, D), bf(T, m, D), bf(T, n, D)
        self.R = torch.rand(T, m, n, generator=g).to(device)
        self.W = torch.rand(T, n, m, generator=g).to(device)
        self.H = torch.rand(T, n, n, generator=g).to(device)
        self.v = torch.rand(T, n, generator=g).to(device) if proj else None
        self.u = torch.empty(T, m, D, dtype=torch.bfloat16, device=device)
        self.out = torch.empty_like(self.x)
        self.grad_x = torch.empty_like(self.x)
        self.grad_f = torch.empty_like(self.f)
        self.grad_R = torch.empty(T, m, n, device=device)
        self.grad_H = torch.empty(T, n, n, device=device)
        self.grad_W = torch.empty(T, n, m, device=device)
        self.grad_v = torch.empty(T, n, device=device) if proj else None
        self.code = _lib.dtype_code(torch.bfloat16)
        self.stream = torch.cuda.current_stream(device).cuda_stream
        self._ptr = _lib.ptr

    def read_fwd(self):
        self._check(self.lib.hc_read_fwd(self.R.data_ptr(), self.x.data_ptr(), self.u.data_ptr(), self.T, self.n,
                                         self.m, self.D, self.code, self.stream), "hc_read_fwd")

    def read_bwd(self):
        self._check(self.lib.hc_read_bwd(self.g_u.data_ptr(), self.R.data_ptr(), self.x.data_ptr(),
                                         self.grad_x.data_ptr(), self.grad_R.data_ptr(), self.T, self.n, self.m,
                                         self.D, self.code, self.stream), "hc_read_bwd")

    def mix_write_fwd(self):
        self._check(self.lib.hc_mix_write_fwd(self.H.data_ptr(), self.x.data_ptr(), self.W.data_ptr(),
                                              self.f.data_ptr(), self._ptr(self.v), self.out.data_ptr(), self.T,
                                              self.n, self.m, self.D, self.code, self.stream), "hc_mix_write_fwd")

    def mix_write_bwd(self):
        self._check(self.lib.hc_mix_write_bwd(self.g_x.data_ptr(), self.H.data_ptr(), self.x.data_ptr(),
                                              self.W.data_ptr(), self.f.data_ptr(), self._ptr(self.v),
                                              self.grad_x.data_ptr(), self.grad_f.data_ptr(),
                                              self.grad_H.data_ptr(), self.grad_W.data_ptr(),
                                              self._ptr(self.grad_v), self.T, self.n, self.m, self.D, self.code,
                                              self.stream), "hc_mix_write_bwd")


def time_launches(device, fns, steps, warmup, flush_mode="clean"):
    """Mean device ms of each callable in `fns`, L2 flushed between steps."""
    flush = L2Flush(device, flush_mode)
    for _ in range(warmup):
        for fn in fns:
            fn()
    torch.cuda.synchronize(device)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(fns) + 1)] for _ in range(steps)]
    for i in range(steps):
        flush(i)
        evs[i][0].record()
        for k, fn in enumerate(fns):
            fn()
            evs[i][k + 1].record()
    torch.cuda.synchronize(device)
    del flush
    return [float(np.mean([e[k].elapsed_time(e[k + 1]) for e in evs])) for k in range(len(fns))]


# (n, D, projection) of stream_mix_add at 9 <= n <= 32, 2,048 tokens of bf16 streams
BIG_SWEEP = ((9, 1536, False), (12, 1536, True), (16, 1536, False), (16, 1536, True), (24, 1536, False),
             (32, 1536, False), (32, 1536, True))


def large_n_line(device, N, D, proj, steps, warmup, B=2048):
    """stream_mix_add forward + backward at 9 <= N <= 32, bf16 streams and
    Phi (the reference benchmark's dtypes and write flush): GB/s of 3 N D
    elements a token (+ the N x N fp32 grad_Phi in the backward)."""
    fwd_ms, bwd_ms = time_stream_mix(device, B, N, D, torch.bfloat16, proj, steps, warmup)
    nb = 3 * B * N * D * 2
    return {"sweep": "stream_mix_add_large_n", "tokens": B, "n": N, "D": D, "dtype": "bf16", "proj": proj,
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms, "fwd_gbs": nb / (fwd_ms * 1e-3) / 1e9,
            "bwd_gbs": (nb + B * N * N * 4) / (bwd_ms * 1e-3) / 1e9}


# (n, m, D, projection) of the two-phase sweep; the first is the fused step's shape
RW_SWEEP = ((4, 1, 768, False), (4, 1, 768, True), (4, 2, 768, False), (4, 4, 512, False), (6, 3, 1024, True),
            (2, 1, 2048, False), (8, 4, 1024, False))

def time_sinkhorn(device, B, n, iters, steps, warmup):
    """Sinkhorn-Knopp fwd + bwd over B matrices: the two kernels through the
    C-ABI, and for context the same op sequence as eager torch on the GPU
    (exp, then iters x (row sum, divide, column sum, divide), autograd)."""
    from hyperconnections_b200 import _lib

    lib = _lib.lib()
    g = torch.Generator().manual_seed(0)
    H = (torch.randn(B, n, n, generator=g) + 2.0 * torch.eye(n)).to(device)
    G = torch.randn(B, n, n, generator=g).to(device)
    P, dH = torch.empty_like(H), torch.empty_like(H)
    stream = torch.cuda.current_stream(device).cuda_stream

    def kernels():
        _lib.check(lib.hc_sinkhorn_fwd(H.data_ptr(), P.data_ptr(), B, n, iters, stream), "hc_sinkhorn_fwd")
        _lib.check(lib.hc_sinkhorn_bwd(H.data_ptr(), G.data_ptr(), dH.data_ptr(), B, n, iters, stream),
                   "hc_sinkhorn_bwd")

    def eager():
        h = H.detach().requires_grad_(True)
        x = h.exp()
        for _ in range(iters):
            x = x / x.sum(dim=-1, keepdim=True)
            x = x / x.sum(dim=-2, keepdim=True)
        x.backward(G)

    k_ms, e_ms = time_launches(device, [kernels, eager], steps, warmup)
    return {"sweep": "sinkhorn", "batch": B, "n": n, "iters": iters, "kernels_ms": k_ms, "matrices_per_s": B / (k_ms * 1e-3),
            "torch_eager_gpu_ms": e_ms}


# The reference's published stream_mix_add forward numbers (A100 80GB PCIe,
# benchmarks/stream_mix_bench.py -> benchmark_small_n_exhaustive_4_3_2026.log):
# (tokens B, N, D, dtype, projection, GB/s in the reference's byte model, log line)
PUBLISHED_FWD = (
    (2048, 4, 1024, "fp32", False, 947.2, 2129),
    (2048, 4, 1024, "fp32", True, 967.4, 2130),
    (2048, 4, 768, "fp32", False, 489.4, 2127),
    (2048, 8, 1024, "fp32", False, 1031.8, 2169),
    (2048, 16, 1536, "fp32", False, 1542.1, 2211),
    (2048, 4, 768, "fp16", False, 244.9, 2248),
    (2048, 4, 1024, "fp16", False, 248.3, 2250),
    (2048, 8, 1024, "fp16", False, 923.0, 2290),
)


def reference_model_bytes(B, N, D, elem, proj):
    """The reference benchmark's byte model (stream_mix_bench.py:329-336)."""
    return elem * (B * N * N + 3 * B * N * D + (B * N if proj else 0))


def time_stream_mix(device, B, N, D, dtype, proj, steps, warmup):
    """stream_mix_add forward and backward through the C-ABI on resident
    buffers, 256 MiB write flush between steps (as do_bench does)."""
    from hyperconnections_b200 import _lib

    lib = _lib.lib()
    g = torch.Generator().manual_seed(0)
    Phi = torch.randn(B, N, N, generator=g).to(dtype).to(device)
    x, Y, G = (torch.randn(B, N, D, generator=g).to(dtype).to(device) for _ in range(3))
    v = torch.nn.functional.normalize(torch.randn(B, N, generator=g), dim=-1).to(dtype).to(device) if proj else None
    out, gx = torch.empty_like(x), torch.empty_like(x)
    gP = torch.empty(B, N, N, device=device)
    gv = torch.empty(B, N, device=device) if proj else None
    code = _lib.dtype_code(dtype)
    st = torch.cuda.current_stream(device).cuda_stream

    def fwd():
        _lib.check(lib.hc_stream_mix_fwd(Phi.data_ptr(), x.data_ptr(), Y.data_ptr(), _lib.ptr(v), out.data_ptr(),
                                         B, N, D, code, code, st), "hc_stream_mix_fwd")

    def bwd():
        _lib.check(lib.hc_stream_mix_bwd(G.data_ptr(), Phi.data_ptr(), x.data_ptr(), _lib.ptr(v), gx.data_ptr(),
                                         gP.data_ptr(), _lib.ptr(gv), B, N, D, code, code, st), "hc_stream_mix_bwd")

    return time_launches(device, [fwd, bwd], steps, warmup, flush_mode="write")


def time_pade(device, B, n, steps, warmup):
    """Pade [7/7] matrix exponential (the replacement of torch.linalg.matrix_exp
    in the CGHC layer) forward + backward over B matrices of the expm workload:
    the two kernels through the C-ABI, and for context torch.linalg.matrix_exp
    with autograd on the same GPU."""
    from hyperconnections_b200 import _lib

    lib = _lib.lib()
    A, G = (t.to(device) for t in expm_workload(B, n, seed=3))
    E, dA = torch.empty_like(A), torch.empty_like(A)
    st = torch.cuda.current_stream(device).cuda_stream

    def kernels():
        _lib.check(lib.hc_expm_pade_fwd(A.data_ptr(), E.data_ptr(), B, n, st), "hc_expm_pade_fwd")
        _lib.check(lib.hc_expm_pade_bwd(A.data_ptr(), G.data_ptr(), dA.data_ptr(), B, n, st), "hc_expm_pade_bwd")

    def eager():
        At = A.detach().requires_grad_(True)
        torch.autograd.grad(torch.linalg.matrix_exp(At), At, G)

    k_ms, t_ms = time_launches(device, [kernels, eager], steps, warmup)
    return {"sweep": "expm_pade", "batch": B, "n": n, "kernels_ms": k_ms, "matrices_per_s": B / (k_ms * 1e-3),
            "torch_matrix_exp_gpu_ms": t_ms}


def time_generator(device, T, n, steps, warmup):
    """CGHC's generator (conservative + PSD dissipation, the reference's
    default type, scalar dt) forward + backward over T tokens: the kernel pair
    through the C-ABI, the same through the public API with autograd (host
    cost included), and for context the same steps as eager torch ops."""
    from hyperconnections_b200.ops import cghc_generator

    from hyperconnections_b200 import _lib

    lib = _lib.lib()
    g = torch.Generator().manual_seed(0)
    M, R, G = (torch.randn(T, n, n, generator=g).to(device) for _ in range(3))
    lc, ld = (torch.randn(T, 1, generator=g).to(device) for _ in range(2))
    A, dM, dR = (torch.empty_like(M) for _ in range(3))
    dlc, dld = torch.empty_like(lc), torch.empty_like(ld)
    st = torch.cuda.current_stream(device).cuda_stream
    ranges = (0.001, 1.0, 0.001, 1.0)

    def kernels():  # the C-ABI pair: forward, then backward
        _lib.check(lib.hc_cghc_generator_fwd(M.data_ptr(), lc.data_ptr(), R.data_ptr(), None, None, ld.data_ptr(),
                                             A.data_ptr(), T, n, 0, 3, *ranges, st), "hc_cghc_generator_fwd")
        _lib.check(lib.hc_cghc_generator_bwd(M.data_ptr(), lc.data_ptr(), R.data_ptr(), None, None, ld.data_ptr(),
                                             G.data_ptr(), dM.data_ptr(), dlc.data_ptr(), dR.data_ptr(), None, None,
                                             dld.data_ptr(), T, n, 0, 3, *ranges, st), "hc_cghc_generator_bwd")

    def api():
        ins = [t.detach().requires_grad_(True) for t in (M, lc, R, ld)]
        out = cghc_generator(M=ins[0], logit_conserv=ins[1], R=ins[2], logit_diss=ins[3])
        torch.autograd.grad(out, ins, G)

    def eager():
        ins = [t.detach().requires_grad_(True) for t in (M, lc, R, ld)]
        dt_c = 0.001 + 0.999 * torch.sigmoid(ins[1])
        dt_d = 0.001 + 0.999 * torch.sigmoid(ins[3])
        A = dt_c.unsqueeze(-1) * (ins[0] - ins[0].transpose(-1, -2))
        A = A - dt_d.unsqueeze(-1) * (ins[2] @ ins[2].transpose(-1, -2) / n ** 0.5)
        torch.autograd.grad(A, ins, G)

    k_ms, a_ms, e_ms = time_launches(device, [kernels, api, eager], steps, warmup)
    return {"sweep": "cghc_generator", "tokens": T, "n": n, "type": "conservative_psd_diss", "kernels_ms": k_ms,
            "api_autograd_ms": a_ms, "torch_eager_gpu_ms": e_ms}


SWEEP_N = (2, 3, 4, 6, 8)
SWEEP_D = (512, 1024, 2048, 4096)


def run_sweep(args):
    """The small-n sweep at 16,384 tokens, bf16: one JSON line per (n, D) with
    the fused fwd+bwd GB/s and its fraction of the HBM peak; one line per
    (n, m, D, projection) for the two-phase read / mix-write kernels; the
    Sinkhorn-Knopp projection at n = 2, 4, 8; then one line per n for the
    per-token batched expm (16,384 matrices, fwd+bwd), T18 and Pade."""
    _, _, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from hyperconnections_b200 import _lib

    _lib.lib()
    peak, peak_kind = measured_peak()
    steps = max(5, min(args.steps, 50))
    for n in SWEEP_N:
        for D in SWEEP_D:
            res = time_fused(device, steps, args.warmup, 1, T=TOKENS, n=n, D=D)
            fwd_ms, bwd_ms = float(np.mean(res["fwd_ms"])), float(np.mean(res["bwd_ms"]))
            fb, bb = fused_bytes(TOKENS, n, D)
            gbs = (fb + bb) / (float(np.mean(res["step_ms"])) * 1e-3) / 1e9
            print(json.dumps({
                "sweep": "fused", "tokens": TOKENS, "n": n, "D": D, "step_ms": float(np.mean(res["step_ms"])),
                "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
                "fwd_gbs": fb / (fwd_ms * 1e-3) / 1e9, "bwd_gbs": bb / (bwd_ms * 1e-3) / 1e9, "gbs": gbs,
                "frac_of_peak": gbs / peak, "peak": peak, "peak_kind": peak_kind,
                "pct_of_8tbs": 100.0 * gbs / NOMINAL_HBM_GBS, "bytes": fb + bb}), flush=True)
    dt = {"fp32": torch.float32, "fp16": torch.float16}
    for B, N, D, name, proj, ref_gbs, line_no in PUBLISHED_FWD:
        fwd_ms, bwd_ms = time_stream_mix(device, B, N, D, dt[name], proj, steps, args.warmup)
        elem = 4 if name == "fp32" else 2
        gbs = reference_model_bytes(B, N, D, elem, proj) / (fwd_ms * 1e-3) / 1e9
        print(json.dumps({"sweep": "stream_mix_add_published", "tokens": B, "n": N, "D": D, "dtype": name,
                          "proj": proj, "fwd_ms": fwd_ms, "bwd_ms": bwd_ms, "fwd_gbs_reference_model": gbs,
                          "reference_a100_gbs": ref_gbs, "ratio": gbs / ref_gbs,
                          "reference_source": f"benchmark_small_n_exhaustive_4_3_2026.log:{line_no}"}),
              flush=True)
    for N, D, proj in BIG_SWEEP:
        print(json.dumps(large_n_line(device, N, D, proj, steps, args.warmup)), flush=True)
    for n, m, D, proj in RW_SWEEP:
        r = RwRunner(device, TOKENS, n, m, D, proj)
        names = ("read_fwd", "read_bwd", "mix_write_fwd", "mix_write_bwd")
        ms = time_launches(device, [getattr(r, k) for k in names], steps, args.warmup)
        nbytes = rw_bytes(TOKENS, n, m, D, proj)
        line = {"sweep": "read/mix_write", "tokens": TOKENS, "n": n, "m": m, "D": D, "proj": proj,
                "peak": peak, "peak_kind": peak_kind}
        for k, t in zip(names, ms):
            line[f"{k}_ms"] = t
            line[f"{k}_gbs"] = nbytes[k] / (t * 1e-3) / 1e9
        line["gbs"] = sum(nbytes.values()) / (sum(ms) * 1e-3) / 1e9
        line["frac_of_peak"] = line["gbs"] / peak
        print(json.dumps(line), flush=True)
        del r
    for n in (2, 4, 8):
        line = time_sinkhorn(device, TOKENS, n, 20, steps, args.warmup)
        print(json.dumps(line), flush=True)
    for n in (4, 8):
        print(json.dumps(time_generator(device, TOKENS, n, steps, args.warmup)), flush=True)
    for n in SWEEP_N:
        ms = float(np.mean(time_expm(device, steps, args.warmup, B=TOKENS, n=n)))
        print(json.dumps({"sweep": "expm_t18", "batch": TOKENS, "n": n, "ms_per_step": ms,
                          "matrices_per_s": TOKENS / (ms * 1e-3)}), flush=True)
    for n in SWEEP_N:
        print(json.dumps(time_pade(device, TOKENS, n, steps, args.warmup)), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-models", action="store_true", help="skip the end-to-end ViT / LM training legs")
    ap.add_argument("--fused-only", action="store_true",
                    help="time the headline fused step alone and print a short line (profiling, comparisons)")
    ap.add_argument("--n", type=int, default=N_STREAMS, help="with --fused-only: streams (16,384 tokens)")
    ap.add_argument("--block", type=int, default=BLOCK, help="with --fused-only: block size D")
    ap.add_argument("--sweep", action="store_true", help="print the n x D sweep (16,384 tokens) instead")
    ap.add_argument("--large-n", type=int, default=0,
                    help="stream_mix_add at this 9 <= n <= 32 alone (2,048 tokens, D = 1536, bf16; ncu captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.sweep:
        run_sweep(args)
    elif args.large_n:
        device = torch.device("cuda", 0)
        torch.cuda.set_device(device)
        print(json.dumps(large_n_line(device, args.large_n, 1536, False, args.steps, args.warmup)), flush=True)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
