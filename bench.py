#!/usr/bin/env python
"""Benchmark of the persistent micro-op runtime on the reference's headline workload.

Workload (one step = one flush): 4096 independent fp32 requests of 4096 contiguous
elements each, a, b ~ U(-1, 1) from a fixed seed, op 50/50 add/mul, a separate output
buffer per request, submitted with submit_add / submit_mul and one flush(sync=True).
Inputs + outputs are 201 MB per step (> 126 MB L2), so every step streams from HBM.

Printed JSON line (rank 0):
  value     micro-ops/s of the whole job, inputs resident in HBM, timed with CUDA events
            on the current stream around K steps (submit calls included), max over ranks,
            summed over ranks (weak scaling: every rank runs the full workload on its GPU)
  e2e       the same through the public API with host (pinned) buffers: H2D of a and b and
            D2H of out inside every step
  roofline  the worker kernel: algorithmic bytes (12 B per element) / launch duration,
            launches timed with CUDA events on the worker's stream in drain mode (from launch
            to grid exit), each launch carrying 8 steps of requests; against
            MEASURED_PEAKS.json hbm_gbs.  traffic: 8 x the DRAM bytes of a one-step launch
            (committed ncu summary; traffic grows with the tiles processed).  One step per
            launch is reported beside it
  baselines GPU per-op torch eager (same stream of requests as individual launches) and
            the CPU path (PyTorch CPU eager over the same requests on the host cores)
  latency   p50/p99 submit->done of single 4096-element requests: back to back (sync flush
            each), and open loop at 25/50/80% of that rate (asynchronous flushes, polled)
  copy ceiling  the e2e step's H2D and D2H copies alone (what e2e can reach over PCIe)

--impl reference runs the reference's CPU path (PyTorch CPU eager over the identical
request stream, all host threads) and prints the same metric.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import datetime
import json
import os
import statistics
import sys
import threading
import time

# the persistent worker holds one hardware work queue; give other streams their own
os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")

import torch  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "aggregated micro-ops/s"
UNIT = "micro-ops/s"
WORKLOAD = "4096 fp32 requests x 4096 contiguous elements, add/mul 50/50, one flush per step"
BYTES_PER_ELEM = 12  # read a, read b, write out (fp32)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--requests", type=int, default=4096)
    p.add_argument("--numel", type=int, default=4096)
    p.add_argument("--worker-mode", choices=["persistent", "drain"], default="persistent")
    p.add_argument("--no-extras", action="store_true", help="skip baselines, latency, e2e (profiling runs)")
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--latency-samples", type=int, default=2000)
    p.add_argument("--workload", choices=["c1", "c2", "c3", "c4", "c5"], default="c1",
                   help="c1: the headline workload (default).  c2-c4: the mixed-op, strided/broadcast "
                        "mixed-dtype and reduction streams, one GPU, measured for the kernel's roofline.  "
                        "c5: dependent chains over N runtimes with an NVRTC op_mul switched in at request "
                        "50000, a dual-slot switch and a rollback (torchrun for N > 1)")
    p.add_argument("--e2e-chunks", type=int, default=4, help="chunks per step of the e2e pipeline")
    p.add_argument("--config-requests", type=int, default=0,
                   help="c2-c4: requests per step (default: the configuration's full count)")
    return p.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def rank_max(dist, x: float, device: str) -> float:
    """Max of a per-rank timing over all ranks (identity without a process group)."""
    if dist is None:
        return x
    t = torch.tensor([x], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_rate(units_per_rank: float, world: int, elapsed_ms: float) -> float:
    """Whole-job rate under weak scaling: every rank processed `units_per_rank` units, and the job
    took the slowest rank's time."""
    return units_per_rank * world / (elapsed_ms / 1e3)


def profiled_traffic():
    """DRAM bytes (read + write) of one worker launch on this workload, from the committed ncu
    summary (profiles/gpuos_batch_worker_c1_drain.json), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "gpuos_batch_worker_c1_drain.json")) as f:
            return float(json.load(f)["dram_bytes_per_launch"])
    except Exception:
        return None


def workload(rank: int, R: int, N: int):
    g = torch.Generator().manual_seed(1234 + 1 + rank)
    A = torch.rand(R, N, generator=g) * 2 - 1
    B = torch.rand(R, N, generator=g) * 2 - 1
    ops = torch.randint(0, 2, (R,), generator=g)
    return A, B, ops


class Clocks:
    """SM clock and clock-event reasons sampled through NVML every 20 ms while a timed region
    runs."""

    REASONS = (("hw_slowdown", "nvmlClocksThrottleReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksThrottleReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksThrottleReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksThrottleReasonSwPowerCap"),
               ("hw_power_brake", "nvmlClocksThrottleReasonHwPowerBrakeSlowdown"))

    def __init__(self, index: int):
        self.index = index
        self.samples = []  # (sm_mhz, reasons bitmask)
        self.sm_max = None
        self.stop_evt = threading.Event()
        self.thread = None
        self.nvml = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(vis.split(",")[self.index]) if vis else self.index
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.sm_max = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.nvml = pynvml
        except Exception:
            self.nvml = None
            return
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def _run(self):
        nv = self.nvml
        while not self.stop_evt.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                try:
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                except Exception:
                    r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle)
                self.samples.append((sm, r))
            except Exception:
                pass
            self.stop_evt.wait(0.02)

    def stop(self):
        self.stop_evt.set()
        if self.thread is not None:
            self.thread.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.sm_max, "reasons": ["clock sampling unavailable"], "samples": 0}
        nv = self.nvml
        reasons = sorted({name for _, r in self.samples for name, attr in self.REASONS
                          if hasattr(nv, attr) and r & getattr(nv, attr)})
        return {"sm_mhz": statistics.median(sm for sm, _ in self.samples), "sm_max_mhz": self.sm_max,
                "reasons": reasons, "samples": len(self.samples)}


_CPU = {}


def _cpu_init(A, B, out, ops):
    torch.set_num_threads(1)
    _CPU.update(A=A, B=B, out=out, ops=ops)


def _cpu_slice(bounds):
    lo, hi = bounds
    A, B, out, ops = _CPU["A"], _CPU["B"], _CPU["out"], _CPU["ops"]
    for i in range(lo, hi):
        if ops[i] == 0:
            torch.add(A[i], B[i], out=out[i])
        else:
            torch.mul(A[i], B[i], out=out[i])
    return hi - lo


class CpuPath:
    """The request stream in PyTorch CPU eager, split over `procs` host processes (spawned,
    tensors in shared memory; Python threads would serialise on the GIL)."""

    def __init__(self, A, B, out, ops, procs: int):
        self.procs = procs
        R = A.shape[0]
        self.chunks = [(k * R // procs, (k + 1) * R // procs) for k in range(procs)]
        if procs > 1:
            for t in (A, B, out):
                t.share_memory_()
            ctx = torch.multiprocessing.get_context("spawn")
            self.pool = ctx.Pool(procs, initializer=_cpu_init, initargs=(A, B, out, ops))
        else:
            _cpu_init(A, B, out, ops)
            self.pool = None

    def run(self):
        if self.pool is None:
            _cpu_slice(self.chunks[0])
        else:
            self.pool.map(_cpu_slice, self.chunks)

    def close(self):
        if self.pool is not None:
            self.pool.close()
            self.pool.join()


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def bind_to_gpu_cores(index: int):
    """Restrict this process to the CPU cores NVML reports as local to GPU `index`; returns the
    previous CPU set (None when NVML or the mapping is unavailable)."""
    try:
        import pynvml
        pynvml.nvmlInit()
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        phys = int(vis.split(",")[index]) if vis else index
        h = pynvml.nvmlDeviceGetHandleByIndex(phys)
        words = ((os.cpu_count() or 64) + 63) // 64
        masks = pynvml.nvmlDeviceGetCpuAffinity(h, words)
        before = os.sched_getaffinity(0)
        cpus = {64 * i + bit for i, m in enumerate(masks) for bit in range(64) if (m >> bit) & 1} & before
        if cpus and cpus != before:
            os.sched_setaffinity(0, cpus)
            return before
    except Exception:
        pass
    return None


def time_cpu_path(cpu: CpuPath, warm_passes: int, min_passes: int, seconds: float, warm_seconds: float = 3.0):
    """Steady-state rate of the CPU path: warm-up until both `warm_passes` passes and
    `warm_seconds` have gone by (process pool, page faults, clocks), then time passes until both
    `min_passes` passes and `seconds` have gone by.  Returns (passes timed, seconds)."""
    t0 = time.perf_counter()
    k = 0
    while k < warm_passes or time.perf_counter() - t0 < warm_seconds:
        cpu.run()
        k += 1
    n = 0
    t0 = time.perf_counter()
    while n < min_passes or time.perf_counter() - t0 < seconds:
        cpu.run()
        n += 1
    return n, time.perf_counter() - t0


def run_reference(args, rank, world):
    """The reference's CPU path: PyTorch CPU eager over the identical request stream, timed over
    the same steady-state window as the cpu_baseline leg of the GPU arm."""
    if rank != 0:
        return None
    import oracle.reference_semantics  # noqa: F401  (CPU path lives with the oracle)
    threads = cpu_threads()
    A, B, ops = workload(0, args.requests, args.numel)
    out = torch.empty_like(A)
    cpu = CpuPath(A, B, out, ops.tolist(), threads)
    passes, dt = time_cpu_path(cpu, args.warmup, args.steps, args.cpu_seconds)
    cpu.close()
    ok = torch.equal(out, torch.where(ops[:, None] == 0, A + B, A * B))
    v = args.requests * passes / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / passes * 1e3, "timed_passes": passes,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded U(-1,1))",
        "config": {"workload": WORKLOAD, "requests": args.requests, "numel": args.numel, "l2": "inputs > L2"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{passes} passes x {args.requests} requests in {dt:.1f} s after >= 3 s of "
                                   f"warm-up (full workload)"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "correct": bool(ok),
    }
    return line


# ---- secondary workloads (one GPU): the request streams of the other configurations ----------
def open_loop_latency(g, x, y, z, capacity_per_s: float, samples: int, fracs=(0.25, 0.5, 0.8)):
    """p50/p99 submit->done of single 4096-element requests arriving on a fixed schedule at a
    stated fraction of the back-to-back request rate (an open loop: an arrival does not wait
    for earlier requests).  Each request is one submit_add plus an asynchronous flush; its
    completion is seen by polling the highest completed flush ticket between arrivals, so a
    latency includes up to one polling pass (about a microsecond)."""
    out = {}
    for frac in fracs:
        period = 1e9 / (capacity_per_s * frac)
        pending, lat = [], []
        n = 0
        t0 = time.perf_counter_ns()
        nxt = t0
        while len(lat) < samples:
            now = time.perf_counter_ns()
            if n < samples and now >= nxt:
                g.submit_add(x, y, z)
                pending.append((g.flush(), now))
                n += 1
                nxt += period
            if pending:
                done = g.completed()
                now = time.perf_counter_ns()
                while pending and pending[0][0] <= done:
                    lat.append((now - pending[0][1]) / 1e3)
                    pending.pop(0)
        lat.sort()
        out[f"{int(frac * 100)}%"] = {"offered_req_per_s": round(capacity_per_s * frac),
                                      "p50": lat[len(lat) // 2], "p99": lat[int(len(lat) * 0.99)]}
    out["what"] = ("open loop: single 4096-element fp32 add requests on a fixed schedule at the stated fraction "
                   "of the back-to-back rate, submit_add + asynchronous flush each, completion polled")
    return out


def ulp_distance(got: torch.Tensor, ref: torch.Tensor) -> torch.Tensor:
    """|ulp distance| between two float32 tensors (same sign ordering as the integers)."""
    def key(t):
        i = t.float().contiguous().view(torch.int32).to(torch.int64)
        return torch.where(i < 0, -(i & 0x7FFFFFFF), i)
    return (key(got) - key(ref)).abs()


def log_uniform(g, lo: float, hi: float) -> int:
    import math
    return int(math.exp(math.log(lo) + torch.rand(1, generator=g).item() * (math.log(hi) - math.log(lo))))


def aligned(n: int, es: int) -> int:
    """Elements of a slice of n elements rounded up to 512 bytes: requests sit in one buffer
    at the alignment separate allocations would have."""
    per = 512 // es
    return (n + per - 1) // per * per


def _c2_ops():
    """name, op-code attribute, binary, (p0, p1), bit-exact against PyTorch CPU, PyTorch op"""
    import torch.nn.functional as F
    return [
        ("relu", "EW_RELU", False, (), True, lambda x, y: torch.relu(x)),
        ("sigmoid", "EW_SIGMOID", False, (), False, lambda x, y: torch.sigmoid(x)),
        ("tanh", "EW_TANH", False, (), False, lambda x, y: torch.tanh(x)),
        ("exp", "EW_EXP", False, (), False, lambda x, y: torch.exp(x)),
        ("log", "EW_LOG", False, (), False, lambda x, y: torch.log(x)),
        ("sqrt", "EW_SQRT", False, (), False, lambda x, y: torch.sqrt(x)),
        ("gelu", "EW_GELU", False, (), False, lambda x, y: F.gelu(x)),
        ("hardswish", "EW_HARDSWISH", False, (), True, lambda x, y: F.hardswish(x)),
        ("leaky_relu", "EW_LEAKY_RELU", False, (0.01,), True, lambda x, y: F.leaky_relu(x, 0.01)),
        ("elu", "EW_ELU", False, (1.0,), False, lambda x, y: F.elu(x)),
        ("softplus", "EW_SOFTPLUS", False, (1.0, 20.0), False, lambda x, y: F.softplus(x)),
        ("clamp", "EW_CLAMP", False, (-0.5, 0.5), True, lambda x, y: torch.clamp(x, -0.5, 0.5)),
        ("add", "EW_ADD", True, (), True, lambda x, y: x + y),
        ("sub", "EW_SUB", True, (), True, lambda x, y: x - y),
        ("mul", "EW_MUL", True, (), True, lambda x, y: x * y),
        ("div", "EW_DIV", True, (), True, lambda x, y: x / y),
        ("maximum", "EW_MAXIMUM", True, (), True, lambda x, y: torch.maximum(x, y)),
        ("minimum", "EW_MINIMUM", True, (), True, lambda x, y: torch.minimum(x, y)),
        ("pow", "EW_POW", True, (), False, lambda x, y: torch.pow(x, y)),
    ]


def _within(got, ref, exact, x, name) -> bool:
    if exact:
        return bool(torch.equal(got.float().view(torch.int32), ref.float().contiguous().view(torch.int32)))
    d = ulp_distance(got, ref)
    if name == "gelu":  # PyTorch CPU's own GELU error reaches ~6 |x| 2**-24
        d = torch.where((got.float() - ref.float()).abs() <= 8 * x.abs() * 2.0 ** -24, torch.zeros_like(d), d)
    return int(d.max()) <= 2


def build_c2(g_ext, seed=1234 + 2, n_req=16384):
    """16384 fp32 requests, numel log-uniform 256..32768, ops uniform over the 19 operators,
    inputs in each operator's domain; 512-byte-aligned slices of one buffer per operand."""
    ops = _c2_ops()
    g = torch.Generator().manual_seed(seed)
    sizes = [log_uniform(g, 256, 32768) for _ in range(n_req)]
    kinds = torch.randint(0, len(ops), (n_req,), generator=g).tolist()
    offs, o = [], 0
    for n in sizes:
        offs.append(o)
        o += aligned(n, 4)
    X = torch.rand(o, generator=g) * 8 - 4
    Y = torch.rand(o, generator=g) * 8 - 4
    for k, (n, off) in enumerate(zip(sizes, offs)):
        name = ops[kinds[k]][0]
        x, y = X[off:off + n], Y[off:off + n]
        if name in ("log", "sqrt"):
            x.abs_().add_(1e-3)
        elif name == "div":
            y.copy_(torch.rand(n, generator=g) * 1.5 + 0.5)
        elif name == "pow":
            x.copy_(torch.rand(n, generator=g) * 1.9 + 0.1)
            y.copy_(torch.rand(n, generator=g) * 1.5 + 0.5)
    Xd, Yd = X.cuda(), Y.cuda()
    Od = torch.empty_like(Xd)
    reqs, nbytes = [], 0
    for k, (n, off) in enumerate(zip(sizes, offs)):
        name, code, binary, params, exact, fn = ops[kinds[k]]
        reqs.append((getattr(g_ext, code), Xd[off:off + n], Yd[off:off + n] if binary else None,
                     Od[off:off + n], params))
        nbytes += (12 if binary else 8) * n

    def check(sample):
        ok = True
        for k in sample:
            n, off = sizes[k], offs[k]
            name, code, binary, params, exact, fn = ops[kinds[k]]
            x, y = X[off:off + n], Y[off:off + n]
            ok &= _within(Od[off:off + n].cpu(), fn(x, y), exact, x, name)
        return ok
    desc = ("16384 fp32 requests, numel log-uniform 256..32768, ops uniform over 19 (12 unary, 7 binary), "
            "x ~ U(-4,4) (log/sqrt on |x|+1e-3, pow base U(0.1,2) exponent U(0.5,2), divisor U(0.5,2))")
    extra = {"ops": ops, "kinds": kinds, "X": Xd, "Y": Yd, "sizes": sizes, "offs": offs}
    return reqs, nbytes, check, desc, extra


def build_c3(g_ext, seed=1234 + 3, n_req=8192):
    """8192 requests over 32 shape pairs: a = [C,R] fp16 viewed transposed as [R,C], b = [C]
    bf16 broadcast along dim 0, out [R,C] fp32 contiguous; op add/mul/maximum/gelu(a)."""
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(seed)
    pairs = [(int(torch.randint(1, 257, (1,), generator=g)), int(torch.randint(32, 2049, (1,), generator=g)))
             for _ in range(32)]
    opk = torch.randint(0, 4, (n_req,), generator=g).tolist()
    shapes = [pairs[k % 32] for k in range(n_req)]
    na = sum(aligned(R * C, 2) for R, C in shapes)
    nb = sum(aligned(C, 2) for R, C in shapes)
    no = sum(aligned(R * C, 4) for R, C in shapes)
    gd = torch.Generator(device="cuda").manual_seed(seed)
    Ad = torch.randn(na, generator=gd, device="cuda").half()
    Bd = torch.randn(nb, generator=gd, device="cuda").bfloat16()
    Od = torch.empty(no, device="cuda")
    codes = [g_ext.EW_ADD, g_ext.EW_MUL, g_ext.EW_MAXIMUM, g_ext.EW_GELU]
    reqs, views, nbytes = [], [], 0
    oa = ob = oo = 0
    for k, (R, C) in enumerate(shapes):
        a = Ad[oa:oa + R * C].view(C, R).t()
        b = Bd[ob:ob + C]
        o = Od[oo:oo + R * C].view(R, C)
        op = opk[k]
        reqs.append((codes[op], a, b if op < 3 else None, o, ()))
        views.append((op, a, b, o))
        nbytes += R * C * 6 + (2 * C if op < 3 else 0)
        oa += aligned(R * C, 2)
        ob += aligned(C, 2)
        oo += aligned(R * C, 4)

    def check(sample):
        ok = True
        for k in sample:
            op, a, b, o = views[k]
            ac, bc = a.cpu().float(), b.cpu().float()
            ref = [lambda: ac + bc, lambda: ac * bc, lambda: torch.maximum(ac, bc), lambda: F.gelu(ac)][op]()
            ok &= _within(o.cpu(), ref, op < 3, ac, "gelu")
        return ok
    desc = ("8192 requests over 32 shape pairs R 1..256, C 32..2048: a = [C,R] fp16 viewed transposed, "
            "b = [C] bf16 broadcast along dim 0, out [R,C] fp32; op add/mul/maximum/gelu(a); N(0,1)")
    return reqs, nbytes, check, desc, {}


def build_c4(g_ext, seed=1234 + 4, n_req=8192):
    """8192 sum/mean reductions over the last axis of [R,C]: R log-uniform 1..1024, C log-uniform
    32..4096, fp32 and bf16, half of them stride-2 views of [R,2C], keepdim at random; the output
    has the input's dtype."""
    g = torch.Generator().manual_seed(seed)
    cases = []
    for k in range(n_req):
        R = log_uniform(g, 1, 1024)
        C = log_uniform(g, 32, 4096)
        dt = torch.float32 if k % 2 == 0 else torch.bfloat16
        keep = bool(torch.randint(0, 2, (1,), generator=g))
        mean = bool(torch.randint(0, 2, (1,), generator=g))
        cases.append((R, C, dt, keep, mean, (k // 2) % 2 == 0))
    es = {torch.float32: 4, torch.bfloat16: 2}
    n_in = {torch.float32: 0, torch.bfloat16: 0}
    n_out = {torch.float32: 0, torch.bfloat16: 0}
    for R, C, dt, keep, mean, strided in cases:
        n_in[dt] += aligned(R * (2 * C if strided else C), es[dt])
        n_out[dt] += aligned(R, es[dt])
    gd = torch.Generator(device="cuda").manual_seed(seed)
    IN = {dt: torch.randn(n, generator=gd, device="cuda").to(dt) for dt, n in n_in.items()}
    OUT = {dt: torch.empty(n, device="cuda", dtype=dt) for dt, n in n_out.items()}
    oi = {torch.float32: 0, torch.bfloat16: 0}
    oo = {torch.float32: 0, torch.bfloat16: 0}
    reqs, views, nbytes = [], [], 0
    for R, C, dt, keep, mean, strided in cases:
        w = 2 * C if strided else C
        buf = IN[dt][oi[dt]:oi[dt] + R * w].view(R, w)
        x = buf[:, ::2] if strided else buf
        o = OUT[dt][oo[dt]:oo[dt] + R]
        o = o.view(R, 1) if keep else o.view(R)
        oi[dt] += aligned(R * w, es[dt])
        oo[dt] += aligned(R, es[dt])
        reqs.append(("reduce", g_ext.RED_MEAN if mean else g_ext.RED_SUM, x, o, keep))
        views.append((x, o, keep, mean, dt, C))
        nbytes += R * C * es[dt] + R * es[dt]

    def check(sample):
        ok = True
        for k in sample:
            x, o, keep, mean, dt, C = views[k]
            xc = x.cpu().float()
            ref = xc.mean(-1, keepdim=keep) if mean else xc.sum(-1, keepdim=keep)
            scale = xc.abs().sum(-1, keepdim=keep) / (C if mean else 1)
            tol = 1e-5 if dt == torch.float32 else 1e-2
            ok &= bool(((o.cpu().float() - ref).abs() <= tol * torch.maximum(scale, ref.abs()) + 1e-6).all())
        return ok
    desc = ("8192 sum/mean over the last axis of [R,C], R log-uniform 1..1024, C log-uniform 32..4096, "
            "fp32/bf16 N(0,1), half stride-2 views of [R,2C], keepdim at random, fp32 accumulation")
    return reqs, nbytes, check, desc, {}


# ---- config 5: dependent chains over per-GPU runtimes with an online switch, a dual-slot switch
# and a rollback (test/online_switch.cpp:170-228, test/dual_slot_switch.cpp:139-168) -------------
C5_SWITCH = (50000, 55000, 60000)   # global request index at which phases 1, 2, 3 begin
C5_SENTINEL = 1234.5678              # initial value of every chain output (a lost request keeps it)


def c5_workload(chains=2048, depth=32, n=4096, seed=1234 + 5):
    """Op of step k of chain c drawn uniformly from the 19 config-2 operators; a chain's start
    value ~ U(-4,4); binary operators take a per-chain second operand (U(0.5,2) for div and
    pow's exponent, U(-4,4) otherwise).  Values can leave every operator's domain on the way
    (log of a negative, exp overflow): IEEE results (NaN, inf) are compared like any other."""
    g = torch.Generator().manual_seed(seed)
    kinds = torch.randint(0, 19, (chains, depth), generator=g)
    y0 = torch.rand(chains, n, generator=g) * 8 - 4
    yg = torch.rand(chains, n, generator=g) * 8 - 4
    yp = torch.rand(chains, n, generator=g) * 1.5 + 0.5
    return kinds, y0, yg, yp


def _rows_within(got, ref, exact, x, name):
    """Per-row check (bool per row): bit-exact, or within 2 ulp (GELU: PyTorch CPU's own error
    bound); NaN matches NaN."""
    gn, rn = torch.isnan(got), torch.isnan(ref)
    gi = got.contiguous().view(torch.int32).to(torch.int64)
    ri = ref.contiguous().view(torch.int32).to(torch.int64)
    gi = torch.where(gi < 0, -(gi & 0x7FFFFFFF), gi)
    ri = torch.where(ri < 0, -(ri & 0x7FFFFFFF), ri)
    d = (gi - ri).abs()
    ok = d == 0 if exact else d <= 2
    if name == "gelu":
        ok |= (got - ref).abs() <= 8 * x.abs() * 2.0 ** -24
    ok = torch.where(gn | rn, gn & rn, ok)
    return ok.all(dim=1)


def c5_run(g, rank, world, barrier, chains=2048, depth=32, n=4096, n_probe=2, reps=1, warmup=0):
    """Runs the config-5 stream `warmup + reps` times on this rank's chains and returns a dict of
    measurements and checks.  Every pass: slot 0 = add, alias 0 = 0 at the start; a multiply
    compiled by NVRTC for sm_100a is staged (compiled and linked) before the pass and committed
    into slot 0 at request 50000 (online switch); at 55000 slot 0 returns to add and logical 0
    is routed to physical slot 1 holding the compiled multiply (dual-slot switch); at 60000 the
    alias is rolled back.  Each phase change is an epoch fence: every rank completes its requests
    below the index, all ranks meet (barrier), switch, and meet again."""
    ops = _c2_ops()
    kinds_all, y0, yg, yp = c5_workload(chains, depth, n)
    mine = [c for c in range(chains) if c % world == rank]
    m = len(mine)
    kinds = kinds_all[mine]
    kl = kinds.tolist()
    Yd = torch.full((depth + 1, m, n), C5_SENTINEL, device="cuda")
    YG, YP = yg[mine].cuda(), yp[mine].cuda()
    i = torch.arange(n, dtype=torch.float32)
    PA, PB = (0.5 * i).cuda(), (1.0 + (torch.arange(n) % 5).float()).cuda()
    codes = [getattr(g, o[1]) for o in ops]
    binary = [o[2] for o in ops]
    params = [o[3] for o in ops]
    uses_p = [o[0] in ("div", "pow") for o in ops]
    sub_ew, sub_bin, flush = g.submit_elementwise, g.submit_binary, g.flush
    add0, mul1 = g.builtin_op_address(0), g.builtin_op_address(1)
    # global order: request index k * chains + c (step k of chain c)
    plan = [[(j, k * chains + c) for j, c in enumerate(mine)] for k in range(depth)]
    results = []
    for rep in range(warmup + reps):
        Yd[1:].fill_(C5_SENTINEL)
        Yd[0].copy_(y0[mine].cuda())
        g.set_slot(0, add0)
        g.set_slot(1, mul1)
        g.set_alias(0, 0)
        t_stage = time.perf_counter()
        staged = g.jit_stage("A * B", 2)        # compiled + linked ahead of the switch point
        t_stage = time.perf_counter() - t_stage
        probes = []                              # (phase, output)
        lat = []
        fences = []
        phase = 0
        jit_addr = None
        # per-request row views made before the timed region (indexing a tensor per request
        # would cost the submit loop about as much as the submit itself)
        rows = [list(Yd[k].unbind(0)) for k in range(depth + 1)]
        yrows = [list(YG.unbind(0)), list(YP.unbind(0))]
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        for k in range(depth):
            row_in, row_out = rows[k], rows[k + 1]
            segs = [[]]
            for j, gi in plan[k]:
                if phase + len(segs) - 1 < len(C5_SWITCH) and gi >= C5_SWITCH[phase + len(segs) - 1]:
                    segs.append([])
                segs[-1].append(j)
            for si, seg in enumerate(segs):
                if si > 0:
                    # epoch fence: everything below the switch index is complete on every rank
                    tf = time.perf_counter()
                    barrier()
                    phase += 1
                    if phase == 1:
                        g.jit_commit(staged, 0)              # online switch: slot 0 multiplies
                        jit_addr = g.get_slot(0)
                    elif phase == 2:
                        g.set_slot(0, add0)                  # undo, then route 0 -> physical slot 1
                        g.set_slot(1, jit_addr)
                        g.set_alias(0, 1)
                    else:
                        g.set_alias(0, 0)                    # rollback
                    barrier()
                    fences.append((time.perf_counter() - tf) * 1e3)
                ts = []
                for j in seg:
                    kd = kl[j][k]
                    y = yrows[uses_p[kd]][j] if binary[kd] else None
                    ts.append(time.perf_counter_ns())
                    sub_ew(codes[kd], row_in[j], y, row_out[j], *params[kd])
                for _ in range(n_probe if seg else 0):
                    o = torch.empty_like(PA)
                    sub_bin(0, PA, PB, o)
                    probes.append((phase, o))
                flush(True)
                te = time.perf_counter_ns()
                lat.extend((te - t) / 1e3 for t in ts)
        while phase < len(C5_SWITCH):  # a rank with no request past an index still takes part
            barrier()
            phase += 1
            barrier()
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        results.append({"elapsed_s": elapsed, "lat": lat, "fences_ms": fences, "probes": probes,
                        "stage_s": t_stage})
    # restore the table
    g.set_alias(0, 0)
    g.set_slot(0, add0)
    g.set_slot(1, mul1)
    # ---- checks of the last pass: every request against PyTorch CPU on the GPU's own input ----
    Y = Yd.cpu()
    YGc, YPc = YG.cpu(), YP.cpu()
    lost = wrong = 0
    wrong_by_op, wrong_examples = {}, []
    for k in range(depth):
        for kd, (name, code, bin_, prm, exact, fn) in enumerate(ops):
            rows = (kinds[:, k] == kd).nonzero().flatten()
            if rows.numel() == 0:
                continue
            x = Y[k][rows]
            y = (YPc if uses_p[kd] else YGc)[rows] if bin_ else None
            ref = fn(x, y)
            got = Y[k + 1][rows]
            ok = _rows_within(got, ref, exact, x, name)
            untouched = (got == C5_SENTINEL).all(dim=1) & ~(ref == C5_SENTINEL).all(dim=1)
            lost += int(untouched.sum())
            bad = ~ok & ~untouched
            nb = int(bad.sum())
            wrong += nb
            if nb:
                wrong_by_op[name] = wrong_by_op.get(name, 0) + nb
                r0 = int(bad.nonzero()[0])
                gr, rr, xr = got[r0], ref[r0], x[r0]
                diff = (gr != rr) & ~(torch.isnan(gr) & torch.isnan(rr))
                e0 = int(diff.nonzero()[0]) if bool(diff.any()) else 0
                if len(wrong_examples) < 8:
                    wrong_examples.append({"op": name, "step": k, "x": float(xr[e0]), "got": float(gr[e0]),
                                           "ref": float(rr[e0])})
    padd, pmul = (PA + PB).cpu(), (PA * PB).cpu()
    last = results[-1]
    mis = 0
    per_phase = [0, 0, 0, 0]
    for ph, o in last["probes"]:
        per_phase[ph] += 1
        ref = pmul if ph in (1, 2) else padd
        if not torch.equal(o.cpu(), ref):
            mis += 1
    finite = float(torch.isfinite(Y[depth]).float().mean())
    return {"requests": m * depth, "results": results, "lost": lost, "wrong": wrong, "misdispatched": mis,
            "wrong_by_op": wrong_by_op, "wrong_examples": wrong_examples,
            "probes_per_phase": per_phase, "finite_fraction_final": finite}


def run_c5_bench(args):
    """Config 5 at N GPUs (one rank per GPU under torchrun): the 2048 x 32 chain stream split
    round-robin over the ranks' runtimes ("strong" scaling: the total work is fixed).  Fences
    and the max over ranks use a gloo group (host only: a barrier needs no SM of a GPU whose
    worker is running).  value = all requests / slowest rank's pass time, fences included."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    torch.cuda.set_device(local if world > 1 else 0)
    from gpuos_b200 import gpuos_ext as g
    g.init(capacity=8192, threads_per_block=256)

    def barrier():
        if dist is not None:
            dist.barrier()

    l0 = g.launches()
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    r = c5_run(g, rank, world, barrier, reps=args.steps, warmup=max(0, args.warmup))
    clk = clocks.stop()
    launches = g.launches() - l0
    res = r["results"][max(0, args.warmup):]
    el = [x["elapsed_s"] for x in res]
    lat = [v for x in res for v in x["lat"]]
    tot = torch.tensor([r["lost"], r["wrong"], r["misdispatched"], r["requests"]], dtype=torch.float64)
    mx = torch.tensor(el + [max(f for x in res for f in x["fences_ms"])], dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(tot)
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        lat_t = torch.tensor(lat, dtype=torch.float64)
        gathered = [torch.zeros_like(lat_t) for _ in range(world)]
        dist.all_gather(gathered, lat_t)
        lat = torch.cat(gathered).tolist()
    g.shutdown()
    if rank == 0:
        ms = statistics.median(mx[:-1].tolist()) * 1e3
        lat.sort()
        q = lambda p: lat[min(len(lat) - 1, int(p * len(lat)))]  # noqa: E731
        total = int(tot[3])
        line = {
            "metric": METRIC, "value": total / (ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": len(res),
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32 compute", "data": "synthetic (seeded)",
            "config": {"workload": "config 5: 2048 chains x 32 dependent element-wise ops on [4096] fp32 "
                                   "(ops uniform over the 19 config-2 operators), one sync flush per chain step, "
                                   "chains round-robin over the ranks' runtimes; NVRTC op_mul committed into slot 0 "
                                   "at request 50000, dual-slot switch at 55000, rollback at 60000",
                       "requests": total, "switch_at": list(C5_SWITCH),
                       "parallelism": f"{world} independent runtimes, host gloo barriers at the switch points"},
            "latency_us": {"p50": q(0.5), "p99": q(0.99), "what": "submit call to return of the step's sync flush"},
            "lost": int(tot[0]), "wrong": int(tot[1]), "misdispatched": int(tot[2]),
            "probes_per_phase_rank0": r["probes_per_phase"], "fence_ms_max": float(mx[-1]),
            "stage_s_rank0": statistics.median(x["stage_s"] for x in res),
            "finite_fraction_final_rank0": r["finite_fraction_final"],
            "gpu_launches": launches, "clocks": clk,
            "what": "value: all requests of a pass / slowest rank's pass (host clock, fences included); "
                    "every request checked against PyTorch CPU on its GPU input; probes through op 0 per segment",
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_config(args):
    """One GPU: every request of the configuration submitted through the runtime's calls, then
    one flush(sync=True) per step.  `value` is requests/s with the submit calls; `device` is the
    span of the step's flushes on the GPU (first tile staged to last tile accounted, from the
    %globaltimer stamps of their tickets)."""
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("--workload c2..c4 runs on one GPU")
    torch.cuda.set_device(0)
    if args.worker_mode == "drain":
        # every launch (the one at init included) exits as soon as its work is done
        os.environ["GPUOS_IDLE_QUIESCE_MS"] = "0"
    from gpuos_b200 import gpuos_ext as g
    # a ring large enough for a whole step (a strided request is many tiles): one flush per step
    g.init(capacity=65536, threads_per_block=256)
    if args.worker_mode == "drain":
        g.set_idle_quiesce_ms(0)
    build = {"c2": build_c2, "c3": build_c3, "c4": build_c4}[args.workload]
    kw = {"n_req": args.config_requests} if args.config_requests > 0 else {}
    reqs, nbytes, check, desc, extra = build(g, **kw)
    torch.cuda.synchronize()
    sub_ew, sub_red = g.submit_elementwise, g.submit_reduction

    def step():
        first = g.completed() + 1  # every earlier flush is complete (sync flushes)
        for r in reqs:
            if r[0] == "reduce":
                sub_red(r[1], r[2], r[3], [-1], r[4])
            else:
                sub_ew(r[0], r[1], r[2], r[3], *r[4])
        return first, g.flush(sync=True)

    for _ in range(max(3, args.warmup)):
        step()
    n_req = len(reqs)
    sample = torch.randperm(n_req, generator=torch.Generator().manual_seed(99))[:96].tolist()
    correct = check(sample)
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    l0 = g.launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    seqs = [step() for _ in range(args.steps)]
    e1.record()
    e1.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    dev_ms, nflush = [], []
    for first, last in seqs:
        ts = [g.flush_times(sq) for sq in range(first, last + 1)]
        dev_ms.append((max(t1 for _, t1 in ts) - min(t0 for t0, _ in ts)) / 1e6)
        nflush.append(last - first + 1)
    dmed = statistics.median(dev_ms)
    peak, peak_kind = peaks()
    gbs = nbytes / (dmed * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": n_req / (ms * 1e-3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 compute", "data": "synthetic (seeded)",
        "config": {"workload": desc, "requests": n_req, "algorithmic_bytes_per_step": nbytes,
                   "l2": "inputs larger than L2" if nbytes > 126e6 else "fits in L2"},
        "device": {"flush_ms": dmed, "hbm_gbs": gbs, "frac": gbs / peak, "peak": peak, "peak_kind": peak_kind,
                   "what": "every request of a step: first tile staged to last tile accounted "
                           "(%globaltimer ticket stamps), persistent worker"},
        "flushes_per_step": max(nflush),
        "gpu_launches": g.launches() - l0, "clocks": clk, "correct": bool(correct),
        "correct_sample": f"{len(sample)} requests against PyTorch CPU eager",
    }
    g.shutdown()
    if args.workload == "c2" and not args.no_extras:
        line["scheduler_e2e"] = c2_scheduler(args, extra, native=True)
        line["scheduler_e2e_python_mode"] = c2_scheduler(args, extra, native=False)
    print(json.dumps(line), flush=True)


def c2_scheduler(args, extra, native):
    """The same 16384 requests as PyTorch calls under scheduler_context(size_threshold=1<<15,
    auto_flush_ms=2.0), then flush(sync=True): requests/s through the dispatch plugin (the C++
    dispatcher intercept when `native`, else the Python dispatch mode)."""
    from gpuos_b200.scheduler import scheduler_context
    ops, kinds, X, Y, sizes, offs = (extra[k] for k in ("ops", "kinds", "X", "Y", "sizes", "offs"))
    calls = [(ops[kinds[k]][5], X[off:off + n], Y[off:off + n]) for k, (n, off) in enumerate(zip(sizes, offs))]
    times = []
    with torch.no_grad(), scheduler_context(size_threshold=1 << 15, auto_flush_ms=2.0, native=native) as s:
        for _ in range(1 + max(1, args.steps // 4)):
            t0 = time.perf_counter()
            outs = [fn(x, y) for fn, x, y in calls]
            s.flush(sync=True)
            times.append(time.perf_counter() - t0)
            del outs
        stats = dict(s.stats)
    dt = statistics.median(times[1:])
    return {"value": len(calls) / dt, "unit": UNIT, "ms_per_step": dt * 1e3,
            "scheduled": stats.get("scheduled"), "fallbacks": stats.get("fallbacks"),
            "intercept": "C++ dispatcher fallback" if s.native else "Python dispatch mode",
            "what": "same requests as PyTorch calls under scheduler_context, host wall clock per pass"}


def main():
    args = parse()
    if args.workload == "c5" and args.impl == "ours":
        run_c5_bench(args)
        return
    if args.workload not in ("c1", "c5"):
        run_config(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    dist = None
    host_cpus = None
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        # each rank's submit loop on the cores of its GPU's NUMA node (pinned buffers and the
        # mapped queue words local to the link the GPU reads them over)
        host_cpus = bind_to_gpu_cores(local)
    else:
        torch.cuda.set_device(0)
    dev = torch.cuda.current_device()
    if args.worker_mode == "drain":
        # every launch (the one at init included) exits as soon as its work is done
        os.environ["GPUOS_IDLE_QUIESCE_MS"] = "0"
    from gpuos_b200 import gpuos_ext as g

    R, N = args.requests, args.numel
    A, B, ops = workload(rank, R, N)
    a, b = A.cuda(), B.cuda()
    out = torch.empty_like(a)
    a_rows, b_rows, o_rows = list(a.unbind(0)), list(b.unbind(0)), list(out.unbind(0))
    subs = [g.submit_add if int(o) == 0 else g.submit_mul for o in ops]
    torch.cuda.synchronize()

    g.init(capacity=8192, threads_per_block=256)
    if args.worker_mode == "drain":
        g.set_idle_quiesce_ms(0)

    def step():
        for i in range(R):
            subs[i](a_rows[i], b_rows[i], o_rows[i])
        return g.flush(sync=True)

    def barrier():
        if dist is not None:
            g.quiesce()
            torch.cuda.synchronize()
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        g.quiesce()  # the collective needs SMs that a running worker holds
        return rank_max(dist, x, "cuda")

    for _ in range(max(3, args.warmup)):
        step()
    ref = torch.where(ops[:, None] == 0, A + B, A * B)
    correct = bool(torch.equal(out.cpu(), ref))

    # ---- value: whole job, inputs resident in HBM ----
    g.quiesce()
    torch.cuda.synchronize()
    barrier()
    clocks = Clocks(dev)
    clocks.start()
    n_launch0 = g.launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    seqs = [step() for _ in range(args.steps)]
    e1.record()
    e1.synchronize()
    clk = clocks.stop()
    launches = g.launches() - n_launch0
    elapsed_ms = max_over_ranks(e0.elapsed_time(e1))
    value = job_rate(R * args.steps, world, elapsed_ms)
    dev_ns = []
    for s in seqs:
        try:
            t0, t1 = g.flush_times(s)
            dev_ns.append(t1 - t0)
        except Exception:
            pass
    flush_dev_ms = statistics.median(dev_ns) / 1e6 if dev_ns else None
    peak, peak_kind = peaks()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded U(-1,1))",
        "config": {"workload": WORKLOAD, "requests": R, "numel": N, "worker_mode": args.worker_mode,
                   "l2": "inputs larger than L2 (201 MB per step)", "parallelism": f"dp{world} (independent request streams)"},
        "gpu_launches": launches, "clocks": clk, "correct": correct,
        "persistent_flush_device_ms": flush_dev_ms,
        "persistent_flush_hbm_gbs": (R * N * BYTES_PER_ELEM / (flush_dev_ms * 1e-3) / 1e9) if flush_dev_ms else None,
    }

    if not args.no_extras:
        # ---- roofline: drain mode (the worker exits when its flush is done), each launch
        # bracketed by the runtime's CUDA events on the worker's own stream.  Primary: launches
        # that each carry 8 steps of requests (the same inputs, 8 separate outputs, so no
        # request waits for another) -- the kernel at work, with the ~45 us of launch, start
        # and exit spread over 8 steps.  Also reported: one step per launch. ----
        g.set_idle_quiesce_ms(0)
        g.quiesce()
        g.launch_times()
        g.set_launch_timing(True)
        rclocks = Clocks(dev)
        rclocks.start()
        multi = 8
        outs8 = [torch.empty_like(a) for _ in range(multi)]
        rows8 = [list(o.unbind(0)) for o in outs8]
        nl = max(4, args.steps // 4)
        for k in range(nl + 1):
            for m in range(multi):
                om = rows8[m]
                for i in range(R):
                    subs[i](a_rows[i], b_rows[i], om[i])
            g.flush(sync=True)
        g.quiesce()
        torch.cuda.synchronize()
        durs8 = g.launch_times()[1:]
        for k in range(nl + 1):
            for i in range(R):
                subs[i](a_rows[i], b_rows[i], o_rows[i])
            g.flush(sync=True)
        g.quiesce()
        torch.cuda.synchronize()
        durs1 = g.launch_times()[1:]
        rclk = rclocks.stop()
        g.set_launch_timing(False)
        g.set_idle_quiesce_ms(200 if args.worker_mode == "persistent" else 0)
        ok8 = all(bool(torch.equal(o, out)) for o in outs8)
        del outs8, rows8
        alg = R * N * BYTES_PER_ELEM
        kms = sum(durs8) / nl  # per launch (a launch may also take in a later flush)
        k1 = sum(durs1) / nl
        achieved = multi * alg / (kms * 1e-3) / 1e9
        traffic1 = profiled_traffic()
        line["roofline"] = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                            "frac": achieved / peak,
                            "traffic": traffic1 * multi if traffic1 else None, "peak_kind": peak_kind,
                            "kernel": "gpuos_batch_worker", "launch_ms": kms, "launches": len(durs8),
                            "algorithmic_bytes_per_launch": multi * alg, "correct": ok8,
                            "what": f"one launch per {multi} steps of 4096 tiles of 4096 fp32 (read a, b; write out), "
                                    "drain mode, CUDA events on the worker stream around each launch",
                            "one_step_per_launch": {"launch_ms": k1, "achieved": alg / (k1 * 1e-3) / 1e9,
                                                    "frac": alg / (k1 * 1e-3) / 1e9 / peak,
                                                    "traffic": traffic1},
                            "clocks": rclk}

        # ---- the same bytes through one library kernel: torch.add over the whole 4096x4096
        # step in one launch (2 reads : 1 write, like the worker's step) ----
        g.quiesce()
        torch.cuda.synchronize()
        for _ in range(3):
            torch.add(a, b, out=out)
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        kreps = 20
        k0.record()
        for _ in range(kreps):
            torch.add(a, b, out=out)
        k1.record()
        k1.synchronize()
        lib_gbs = R * N * BYTES_PER_ELEM / (k0.elapsed_time(k1) / kreps * 1e-3) / 1e9
        line["roofline"]["same_traffic_library_kernel"] = {
            "what": "torch.add(a, b, out=out) over the step's 4096x4096 fp32 in one launch, CUDA events",
            "achieved": lib_gbs, "frac": lib_gbs / peak, "worker_over_library": achieved / lib_gbs}
        for i in range(R):  # restore the step's results for the checks below
            subs[i](a_rows[i], b_rows[i], o_rows[i])
        g.flush(sync=True)

        # ---- e2e: host buffers, H2D + D2H inside every step, through the public API.  Each
        # step is split into chunks of requests (4 by default; 2, 4, 8, 16 measured 1.44, 1.43,
        # 1.35, 1.22 M ops/s: every chunk costs host waits): chunk c is flushed as soon as its H2D copy has
        # landed and its D2H copy is queued once its flush ticket has completed, so the two copy
        # directions and the worker overlap.  Two sets of device buffers alternate between
        # steps, so the H2D copies of step s+1 are queued right behind those of step s (into the
        # set step s-1 used, which is complete) and the copy engine never waits for the host ----
        hA, hB = A.pin_memory(), B.pin_memory()
        hO = torch.empty_like(hA).pin_memory()
        sets = [(a, b, out, a_rows, b_rows, o_rows)]
        a2, b2, out2 = torch.empty_like(a), torch.empty_like(b), torch.empty_like(out)
        sets.append((a2, b2, out2, list(a2.unbind(0)), list(b2.unbind(0)), list(out2.unbind(0))))
        g.quiesce()
        barrier()
        cur = torch.cuda.current_stream()
        cs, ds = torch.cuda.Stream(), torch.cuda.Stream()
        nchunk = max(1, args.e2e_chunks)
        bounds = [(c * R // nchunk, (c + 1) * R // nchunk) for c in range(nchunk)]
        out_done = [[None] * nchunk for _ in range(2)]

        def queue_h2d(k):
            da, db = sets[k][0], sets[k][1]
            evs = []
            with torch.cuda.stream(cs):
                for lo, hi in bounds:
                    da[lo:hi].copy_(hA[lo:hi], non_blocking=True)
                    db[lo:hi].copy_(hB[lo:hi], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(cs)
                    evs.append(ev)
            return evs

        def queue_d2h(k, c):
            lo, hi = bounds[c]
            with torch.cuda.stream(ds):
                hO[lo:hi].copy_(sets[k][2][lo:hi], non_blocking=True)
                out_done[k][c] = torch.cuda.Event()
                out_done[k][c].record(ds)

        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(cur)
        cs.wait_stream(cur)
        ds.wait_stream(cur)
        landed_next = queue_h2d(0)
        for step in range(args.steps):
            k = step % 2
            landed = landed_next
            if step + 1 < args.steps:
                landed_next = queue_h2d(1 - k)  # the other set: its last step has completed
            _, _, _, ar, br, orow = sets[k]
            seqs = []
            for c, (lo, hi) in enumerate(bounds):
                for i in range(lo, hi):
                    subs[i](ar[i], br[i], orow[i])
                landed[c].synchronize()
                if out_done[k][c] is not None:
                    out_done[k][c].synchronize()  # the D2H of this set's rows two steps ago has run
                seqs.append(g.flush())
                if c:
                    g.wait(seqs[c - 1])
                    queue_d2h(k, c - 1)
            g.wait(seqs[-1])
            queue_d2h(k, nchunk - 1)
        cur.wait_stream(ds)
        cur.wait_stream(cs)
        f1.record(cur)
        f1.synchronize()
        e2e_ms = max_over_ranks(f0.elapsed_time(f1))
        line["e2e"] = {"value": job_rate(R * args.steps, world, e2e_ms), "unit": UNIT,
                       "h2d_bytes_per_step": 2 * R * N * 4, "d2h_bytes_per_step": R * N * 4,
                       "correct": bool(torch.equal(hO, ref)),
                       "how": f"{nchunk} chunks per step; H2D, worker and D2H overlap across chunks; two device "
                              "buffer sets alternate so the next step's H2D queues behind this one's"}

        # ---- the e2e step's copies alone (no requests, no worker): the same pinned H2D of a and
        # b and D2H of out, both directions on their own streams -- the ceiling e2e can reach on
        # this host's PCIe links ----
        torch.cuda.synchronize()
        barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(cur)
        cs.wait_stream(cur)
        ds.wait_stream(cur)
        for step in range(args.steps):
            k = step % 2
            with torch.cuda.stream(cs):
                sets[k][0].copy_(hA, non_blocking=True)
                sets[k][1].copy_(hB, non_blocking=True)
            with torch.cuda.stream(ds):
                hO.copy_(sets[1 - k][2], non_blocking=True)
        cur.wait_stream(cs)
        cur.wait_stream(ds)
        c1.record(cur)
        c1.synchronize()
        copy_ms = max_over_ranks(c0.elapsed_time(c1))
        line["e2e"]["copy_only_ceiling"] = {
            "value": job_rate(R * args.steps, world, copy_ms), "unit": UNIT,
            "e2e_over_ceiling": line["e2e"]["value"] / job_rate(R * args.steps, world, copy_ms),
            "what": "the e2e step's H2D (a, b) and D2H (out) copies alone, H2D and D2H on separate streams, "
                    "max over ranks"}

        # ---- latency: single 4096-element requests, sync flush each ----
        g.set_idle_quiesce_ms(200)
        lat = []
        x1, y1, z1 = a_rows[0], b_rows[0], o_rows[0]
        for k in range(args.latency_samples + 50):
            t0 = time.perf_counter_ns()
            g.submit_add(x1, y1, z1)
            g.flush(sync=True)
            t1 = time.perf_counter_ns()
            if k >= 50:
                lat.append((t1 - t0) / 1e3)
        lat.sort()
        line["latency_us"] = {"p50": lat[len(lat) // 2], "p99": lat[int(len(lat) * 0.99)],
                              "load": "one 4096-element request per sync flush, back to back"}
        line["latency_us"]["at_load"] = open_loop_latency(g, x1, y1, z1, 1e6 / lat[len(lat) // 2],
                                                          args.latency_samples)

        # ---- the same step through the bulk submitter (one submit_many call per step) ----
        g.set_idle_quiesce_ms(200 if args.worker_mode == "persistent" else 0)
        codes = [g.EW_ADD if int(o) == 0 else g.EW_MUL for o in ops]
        for _ in range(3):
            g.submit_many(codes, a_rows, b_rows, o_rows)
            g.flush(sync=True)
        m0, m1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        m0.record()
        for _ in range(args.steps):
            g.submit_many(codes, a_rows, b_rows, o_rows)
            g.flush(sync=True)
        m1.record()
        m1.synchronize()
        bulk_ok = bool(torch.equal(out.cpu(), ref))
        line["bulk_submit"] = {"value": job_rate(R * args.steps, world, max_over_ranks(m0.elapsed_time(m1))),
                               "unit": UNIT, "correct": bulk_ok,
                               "what": "the same steps with one submit_many call per step instead of "
                                       f"{R} submit_add/submit_mul calls (inputs in HBM)"}

        # ---- baseline (b): GPU per-op torch eager ----
        g.quiesce()
        torch.cuda.synchronize()
        ops_l = ops.tolist()
        for _ in range(2):
            for i in range(R):
                (torch.add if ops_l[i] == 0 else torch.mul)(a_rows[i], b_rows[i], out=o_rows[i])
        h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ke = max(3, args.steps // 2)
        h0.record()
        for _ in range(ke):
            for i in range(R):
                (torch.add if ops_l[i] == 0 else torch.mul)(a_rows[i], b_rows[i], out=o_rows[i])
        h1.record()
        h1.synchronize()
        eager = R * ke / (h0.elapsed_time(h1) / 1e3)
        line["baseline_gpu_eager"] = {"value": eager * world, "unit": UNIT,
                                      "what": "same requests as individual torch.add/mul(out=) launches"}
        line["speedup_vs_gpu_eager"] = value / (eager * world)

        # ---- CPU path (rank 0; with several GPUs a shorter window, the other ranks waiting at
        # the closing barrier) ----
        if rank == 0:
            if host_cpus:
                os.sched_setaffinity(0, host_cpus)  # the CPU path gets every host core again
            threads = cpu_threads()
            cpu = CpuPath(A.clone(), B.clone(), torch.empty_like(A), ops_l, threads)
            secs = args.cpu_seconds if world == 1 else min(args.cpu_seconds, 4.0)
            steps, dt = time_cpu_path(cpu, args.warmup, args.steps, secs)
            cpu.close()
            line["cpu_baseline"] = {"value": R * steps / dt, "unit": UNIT, "cores": threads, "kind": "port",
                                    "sample": f"{steps} passes x {R} requests in {dt:.1f} s after >= 3 s of "
                                              f"warm-up (PyTorch CPU eager), rank 0"
                                              + ("" if world == 1 else f" while the other {world - 1} ranks wait")}
    g.shutdown()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
