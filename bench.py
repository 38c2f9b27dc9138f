"""Benchmark of the int8_convrot linear (rotate+quant -> fused INT8 GEMM + dequant).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl tilegen|reference]

Workload (one step): the qkv_proj linear of a 14B-class video DiT block at
M=4096 tokens per GPU: x fp16 [4096, 5120] ~ N(0,1) with 1 % outlier channels
x30, W int8 [15360, 5120] (a N(0,0.02) weight quantised by the same kernel),
group 256, output fp16 [4096, 15360].  Synthetic, seeded data.

Metric: linear time in microseconds (lower is better).  With N ranks each rank
runs its own 4096-row linear (rows shard with no collective), so the job
processes N linears per step and ``value`` = max-over-ranks time / (N * steps):
microseconds per 4096-row linear for the whole job.  L2 is flushed before every
timed step (a 256 MiB write, then a 256 MiB read of another buffer so that the
write's dirty lines are written back before the step); each step is timed with
CUDA events on the launching stream.

The JSON line also carries: the roofline of the dominant kernel (the GEMM,
tensor-bound) and of the quantiser (HBM-bound), the cuBLAS bf16 F.linear time
of the same shape and the speedup over it, an end-to-end number through the
reference's plugin call (``tilegen.comfyui.backend.int8_linear``) with host
buffers, the CPU baseline (the reference's own CPU path on the host cores,
whole steps), sampled SM clocks, and (N=1) the four DiT shapes and the
quantiser sweep.

``--impl reference`` times the reference's own CPU path of the same linear
(its eager rotate+quant on ``x.float()`` and its chunked GEMM on torch's CPU
``_int_mm``, from the package installed in ``baseline/_ref``) on all host
threads, one whole 4096-row linear per step; rank 0 only.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

M_PER_RANK = 4096
GROUP = 256
SHAPE = ("qkv_proj", 5120, 15360)
NOMINAL_INT8_TOPS = 4500.0
PUBLISHED_QKV_US = 10550.0  # RTX 2080 Ti, tilegen FHT int8_convrot qkv_proj, README.md:9
METRIC = "int8_convrot linear us (M=4096) & speedup vs bf16 cuBLAS; quantizer HBM GB/s"
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of each
# kernel in this bench's timed loop, from one ncu capture of the current kernels
# on a B200 (the files named below).  The quantiser's 21 MB of codes are still in
# L2 when it ends, so its traffic is below its algorithmic bytes; the GEMM's
# equals A + B + the part of the output already written back.
GEMM_TRAFFIC_BYTES = 100_430_592 + 95_247_872
QUANT_TRAFFIC_BYTES = 41_977_344 + 174_592
GEMM_TRAFFIC_SOURCE = "profiles/gemm_i8_dequant_pair_qkv.md"
QUANT_TRAFFIC_SOURCE = "profiles/rotquant_short_m4096_k5120.md"


def _peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def _workload_desc():
    name, k, n = SHAPE
    return (f"{name} int8_convrot linear: x fp16 [{M_PER_RANK},{k}] N(0,1) with 1% outlier channels x30, "
            f"W int8 [{n},{k}] per-channel fp32 scales, group {GROUP}, out fp16 [{M_PER_RANK},{n}]")


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock and clock-event reasons during a with-block (the timed region).

    A separate process reads NVML in a tight loop (wall-clock stamped), so the
    samples do not depend on this process's interpreter lock, which the timed
    loop holds while it enqueues; the samples stamped inside the with-block are
    kept.  Falls back to ``nvidia-smi -lms 100`` when NVML is unavailable."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    # NVML clocks-event reason bits (nvml.h): SW power cap, HW slowdown, SW thermal, HW thermal.
    NVML_REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
                    0x40: "hw_thermal_slowdown"}

    POLL = ("import sys, time, pynvml\n"
            "pynvml.nvmlInit()\n"
            "h = pynvml.nvmlDeviceGetHandleByIndex(int(sys.argv[1]))\n"
            "print('max', pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM), flush=True)\n"
            "while True:\n"
            "    t = time.time()\n"
            "    m = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)\n"
            "    b = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)\n"
            "    print(f'{t:.6f} {m} {b}', flush=True)\n"
            "    time.sleep(0.0002)\n")

    def __init__(self, gpu_index: int):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
        if 0 <= gpu_index < len(vis) and vis[gpu_index].strip().isdigit():
            gpu_index = int(vis[gpu_index])
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.kind = None
        self.t0 = self.t1 = 0.0

    def _lines(self):
        try:
            with open(self.path) as f:
                return f.read().splitlines()
        except OSError:
            return []

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".txt")
        os.close(fd)
        try:
            self.proc = subprocess.Popen([sys.executable, "-c", self.POLL, str(self.gpu)],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            self.kind = "nvml"
            deadline = time.time() + 20
            while len(self._lines()) < 2 and time.time() < deadline and self.proc.poll() is None:
                time.sleep(0.01)
            if len(self._lines()) < 2:
                raise RuntimeError("NVML poller did not start")
        except Exception:
            if self.proc is not None:
                self.proc.kill()
            self.kind = "nvidia-smi"
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                     "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
                time.sleep(0.3)
            except Exception:
                self.proc = None
        self.t0 = time.time()
        return self

    def __exit__(self, *a):
        self.t1 = time.time()
        time.sleep(0.005)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except Exception:
                self.proc.kill()

    def summary(self):
        lines = self._lines()
        if self.path and os.path.exists(self.path):
            os.unlink(self.path)
        if self.kind == "nvml":
            smax, rows = None, []
            for ln in lines:
                parts = ln.split()
                try:
                    if parts[0] == "max":
                        smax = float(parts[1])
                    else:
                        rows.append((float(parts[0]), float(parts[1]), int(parts[2])))
                except (IndexError, ValueError):
                    continue
            inside = [r for r in rows if self.t0 <= r[0] <= self.t1]
            used = inside or [r for r in rows if r[0] < self.t0][-1:] + [r for r in rows if r[0] > self.t1][:1]
            if not used:
                return {"sm_mhz": None, "sm_max_mhz": smax, "reasons": ["unsampled"]}
            reasons = sorted({nm for _, _, bits in used for b, nm in self.NVML_REASONS.items() if bits & b})
            return {"sm_mhz": statistics.median(m for _, m, _ in used), "sm_max_mhz": smax,
                    "samples": len(inside), "region_ms": round((self.t1 - self.t0) * 1e3, 2),
                    "source": "NVML, polled by a separate process during the timed region"
                              + ("" if inside else " (none inside: the samples just before and after)"),
                    "reasons": reasons}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": smax, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "samples": len(sm),
                "source": "nvidia-smi", "reasons": sorted(reasons)}


# ------------------------------------------------------------------ helpers
def _setup_dist(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        if args.impl == "tilegen":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
    return world, rank, local


def _reference_cpu():
    """The reference's own CPU path of the linear (its eager rotate+quant on the
    fp32-upcast activations, tilegen/kernels/int8_convrot.py:289-302,
    and its chunked GEMM + dequant on torch's CPU ``_int_mm``,
    tilegen/quant/int8_ops.py:22-70; the weight quantised offline by its
    quantize_convrot_weight, weight.py:14-39).

    Imported from the reference package installed in ``baseline/_ref`` (loaded
    under the name ``tilegen_ref``, since ``tilegen`` here is this repository's
    alias package): kind "reference".  Without that install, this repository's
    torch restatement of the same functions on CPU tensors (the eager path and
    ``_int_mm`` chunks of ``tilegen_b200``): kind "port".
    """
    import importlib
    import importlib.util

    root = os.path.join(HERE, "baseline", "_ref", "tilegen")
    if os.path.isfile(os.path.join(root, "__init__.py")):
        if "tilegen_ref" not in sys.modules:
            spec = importlib.util.spec_from_file_location("tilegen_ref", os.path.join(root, "__init__.py"),
                                                          submodule_search_locations=[root])
            mod = importlib.util.module_from_spec(spec)
            sys.modules["tilegen_ref"] = mod
            spec.loader.exec_module(mod)
        conv = importlib.import_module("tilegen_ref.kernels.int8_convrot")
        ops_ = importlib.import_module("tilegen_ref.quant.int8_ops")
        weight = importlib.import_module("tilegen_ref.quant.weight")
        return ("reference", conv._eager_quantize, ops_.int8_matmul_dequant_chunked,
                weight.quantize_convrot_weight, "baseline/_ref (the reference package, unmodified)")
    from tilegen_b200.kernels.int8_convrot import _eager_quantize
    from tilegen_b200.quant.int8_ops import int8_matmul_dequant_chunked
    from tilegen_b200.quant.weight import quantize_convrot_weight

    return ("port", _eager_quantize, int8_matmul_dequant_chunked, quantize_convrot_weight,
            "tilegen_b200's torch restatement on CPU tensors (baseline/_ref not installed)")


class CpuLinear:
    """The whole 4096-row linear on the host cores through the reference's CPU path
    (``_reference_cpu``), all host threads; the weight is quantised once at set-up
    (offline in the reference too)."""

    def __init__(self, k: int, n: int):
        import torch

        from tilegen_b200.synthetic import gaussian_weight, outlier_activations

        self.kind, self.quant, self.gemm, wquant, self.source = _reference_cpu()
        torch.set_num_threads(os.cpu_count() or 1)
        self.threads = torch.get_num_threads()
        self.x = outlier_activations(M_PER_RANK, k, seed=0, dtype=torch.float16)
        self.wq, self.ws = wquant(gaussian_weight(n, k, seed=1000), GROUP)

    def step(self) -> float:
        """Seconds for one linear: rotate+quant of x.float(), then GEMM + dequant to fp16."""
        import torch

        t0 = time.perf_counter()
        xq, xs = self.quant(self.x.float(), GROUP)
        self.gemm(xq, xs, self.wq, self.ws, None, torch.float16)
        return time.perf_counter() - t0

    def sample(self) -> str:
        return (f"whole {M_PER_RANK}-row steps of the workload: {self.source}: _eager_quantize(x.float(), {GROUP}) "
                f"then int8_matmul_dequant_chunked (CPU torch._int_mm, 256 MiB chunks) to fp16")


def _cpu_baseline(k, n, budget_s=15.0):
    """Mean seconds per linear over whole steps run for about ``budget_s`` (at least 2)."""
    cpu = CpuLinear(k, n)
    cpu.step()  # warm-up: thread pool, allocator
    times, t_end = [], time.perf_counter() + budget_s
    while len(times) < 2 or time.perf_counter() < t_end:
        times.append(cpu.step())
    return statistics.mean(times), cpu, len(times)


def _config(world: int) -> dict:
    """The workload dict both arms print."""
    name, k, n = SHAPE
    return {"workload": _workload_desc(), "M_per_gpu": M_PER_RANK, "K": k, "N": n, "group": GROUP,
            "parallelism": f"rows x {world} (no collective)",
            "l2": "flushed before every timed GPU step: 256 MiB write, then a 256 MiB read of another "
                  "buffer so the write's dirty lines are written back before the step"}


# ------------------------------------------------------------------ reference arm
def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    name, k, n = SHAPE
    cpu = CpuLinear(k, n)
    for _ in range(args.warmup):
        cpu.step()
    per_step = [cpu.step() * 1e6 for _ in range(args.steps)]
    value = statistics.mean(per_step)
    line = {
        "metric": METRIC,
        "value": round(value, 1), "unit": "us", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(value / 1e3, 3), "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic", "impl": "reference",
        "config": _config(world),
        "cpu_baseline": {"value": round(value, 1), "unit": "us", "cores": cpu.threads, "kind": cpu.kind,
                         "sample": cpu.sample()},
        "e2e": {"value": round(value, 1), "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ tilegen arm
class L2Flush:
    """Flush before a timed step: write a 256 MiB buffer (evicting every input from the
    126 MB L2), then read a second 256 MiB buffer so that the write's dirty lines are
    written back now, not during the timed step (where they would cost a short kernel
    up to ~13 us of HBM write-back that belongs to no workload)."""

    def __init__(self, dev):
        import torch

        self.w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        self.r = torch.ones(64 << 20, dtype=torch.float32, device=dev)
        self.sink = torch.empty(1, dtype=torch.float32, device=dev)

    def zero_(self):
        import torch

        self.w.zero_()
        torch.amax(self.r, dim=0, keepdim=True, out=self.sink)


def _time_steps(fn, steps, flush, stream, marks=1):
    """Run ``fn(events)`` ``steps`` times, flushing L2 before each; per-step event times (ms)."""
    import torch

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(marks + 1)] for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        fn(evs[i])
    torch.cuda.synchronize()
    return [[evs[i][j].elapsed_time(evs[i][j + 1]) for j in range(marks)] for i in range(steps)]


def _bf16_linear_us(x16, w_bf16, steps, flush, stream):
    import torch
    import torch.nn.functional as F

    xb = x16.to(torch.bfloat16)

    def f(e):
        e[0].record(stream)
        F.linear(xb, w_bf16)
        e[1].record(stream)

    for _ in range(3):
        f([torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)])
    t = _time_steps(f, steps, flush, stream)
    return statistics.mean(r[0] for r in t) * 1e3


def _int_mm_tops(dev):
    """cuBLASLt int8 GEMM throughput (torch._int_mm, 8192^3, best of 10) on this GPU."""
    import torch

    a = torch.randint(-128, 128, (8192, 8192), dtype=torch.int8, device=dev)
    b = torch.randint(-128, 128, (8192, 8192), dtype=torch.int8, device=dev)
    for _ in range(3):
        torch._int_mm(a, b.t())
    best = float("inf")
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b.t())
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e))
    return 2 * 8192 ** 3 / (best * 1e-3) / 1e12


def _shape_table(dev, flush, stream, iters=100):
    """The four DiT projections at M = 4096 (fp16): the quantiser and the GEMM each timed
    alone, the whole linear, and bf16 cuBLAS; medians of ``iters`` L2-flushed steps of
    each, the three kinds of step interleaved so that all see the same clock and power
    state (seconds of sustained load pull the clock below its maximum)."""
    import torch
    import torch.nn.functional as F

    from tilegen_b200 import ops
    from tilegen_b200.synthetic import DIT_SHAPES, dit_activations, gaussian_weight

    rows = []
    for name, k, n in DIT_SHAPES:
        x = dit_activations(name, M_PER_RANK, seed=0, dtype=torch.float16, device=dev)
        w = gaussian_weight(n, k, seed=1, dtype=torch.bfloat16, device=dev)
        wq, ws = ops.rotate_quant(w, GROUP)
        xb = x.to(torch.bfloat16)

        def split(e):
            e[0].record(stream)
            xq, xs = ops.rotate_quant(x, GROUP)
            e[1].record(stream)
            ops.int8_gemm_dequant(xq, xs, wq, ws, None, torch.float16)
            e[2].record(stream)

        def whole(e):
            e[0].record(stream)
            xq, xs = ops.rotate_quant(x, GROUP)
            ops.int8_gemm_dequant(xq, xs, wq, ws, None, torch.float16)
            e[1].record(stream)

        def bf16(e):
            e[0].record(stream)
            F.linear(xb, w)
            e[1].record(stream)

        kinds = ((split, 3), (whole, 2), (bf16, 2))
        for fn, marks in kinds:
            for _ in range(3):
                fn([torch.cuda.Event(enable_timing=True) for _ in range(marks)])
        evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(marks)] for _ in range(iters)]
               for _, marks in kinds]
        for i in range(iters):
            for j, (fn, _) in enumerate(kinds):
                flush.zero_()
                fn(evs[j][i])
        torch.cuda.synchronize()
        tq = statistics.median(e[0].elapsed_time(e[1]) for e in evs[0]) * 1e3
        tg = statistics.median(e[1].elapsed_time(e[2]) for e in evs[0]) * 1e3
        tl = statistics.median(e[0].elapsed_time(e[1]) for e in evs[1]) * 1e3
        tb = statistics.median(e[0].elapsed_time(e[1]) for e in evs[2]) * 1e3
        qbytes = M_PER_RANK * k * 3 + 4 * M_PER_RANK
        rows.append({"shape": name, "K": k, "N": n, "int8_linear_us": round(tl, 2), "quant_us": round(tq, 2),
                     "gemm_us": round(tg, 2), "bf16_cublas_us": round(tb, 2), "speedup_vs_bf16": round(tb / tl, 3),
                     "quant_gbs": round(qbytes / (tq * 1e-6) / 1e9, 1),
                     "gemm_tops": round(2 * M_PER_RANK * n * k / (tg * 1e-6) / 1e12, 1)})
        del x, xb, w, wq, ws
    return rows


def _stream_us(fn_for, bufs, stream, reps=5):
    """Per-launch microseconds of ``fn_for(buf)`` run back to back over ``bufs`` (whose
    total is larger than L2, so every launch reads its input from HBM), between two
    events; median over ``reps`` passes."""
    import torch

    for b in bufs:
        fn_for(b)
    out = []
    for _ in range(reps):
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for b in bufs:
            fn_for(b)
        e.record(stream)
        torch.cuda.synchronize()
        out.append(a.elapsed_time(e) * 1e3 / len(bufs))
    return statistics.median(out)


def _quant_sweep(dev, flush, stream, iters=10):
    """Standalone rotate+quant over group x K x M x dtype (inputs N(0,1), 1 % outlier
    channels x30): per entry [group, K, M, dtype, us, GB/s, fraction of HBM peak,
    us_stream, fraction_stream].  ``us`` is one launch between two events after an L2
    flush, which includes the fixed cost of an event-timed launch; ``us_stream`` (M =
    4096) is the per-launch time of launches back to back (through the C ABI, outputs
    allocated beforehand) over enough input buffers that together exceed twice the L2,
    so each launch still reads its input from HBM."""
    import torch

    from tilegen_b200 import _lib, ops
    from tilegen_b200.synthetic import outlier_activations

    hbm = _peaks()[0]["hbm_gbs"]
    rows = []
    for group in (64, 128, 256):
        if group not in (4, 16, 64, 256):
            rows.append([group, "unsupported: a ConvRot group is a power of four (H_G = kron of H4)"])
            continue
        for k in (1536, 3072, 5120, 13824):
            for m in (1, 64, 1024, 4096, 65536):
                for dt in (torch.float16, torch.bfloat16):
                    x = outlier_activations(m, k, seed=0, dtype=dt, device=dev)

                    def f(e):
                        e[0].record(stream)
                        ops.rotate_quant(x, group)
                        e[1].record(stream)

                    for _ in range(2):
                        f([torch.cuda.Event(enable_timing=True) for _ in range(2)])
                    us = statistics.median(r[0] for r in _time_steps(f, iters, flush, stream)) * 1e3
                    byts = m * k * 3 + 4 * m
                    gbs = byts / (us * 1e-6) / 1e9
                    row = [group, k, m, "fp16" if dt == torch.float16 else "bf16", round(us, 2),
                           round(gbs, 1), round(gbs / hbm, 4), None, None]
                    if m == 4096:
                        # Straight through the C ABI with outputs allocated up front,
                        # so the host issues launches faster than the GPU runs them.
                        nbuf = max(2, -(-(256 << 20) // (m * k * 2)))
                        bufs = [x] + [outlier_activations(m, k, seed=j + 1, dtype=dt, device=dev)
                                      for j in range(nbuf - 1)]
                        outs = [(torch.empty((m, k), dtype=torch.int8, device=dev),
                                 torch.empty((m,), dtype=torch.float32, device=dev)) for _ in bufs]
                        L = _lib.lib()
                        code = _lib.TG_DT_F16 if dt == torch.float16 else _lib.TG_DT_BF16
                        calls = [(b.data_ptr(), o[0].data_ptr(), o[1].data_ptr()) for b, o in zip(bufs, outs)]

                        def launch(c):
                            _lib.check("tg_quantize_act", L.tg_quantize_act(
                                c[0], code, m, k, group, _lib.TG_ACT_NONE, c[1], c[2], stream.cuda_stream))

                        us_s = _stream_us(launch, calls, stream)
                        row[7] = round(us_s, 2)
                        row[8] = round(byts / (us_s * 1e-6) / 1e9 / hbm, 4)
                        del bufs, outs
                    rows.append(row)
                    del x
    return rows


def _input_act_table(dev, flush, stream, iters=20):
    """ffn_down with its input activation (tilegen/comfyui/backend.py:201-204) at
    M = 4096: gelu_tanh fused into the quantiser vs applied as its own op first,
    for the quantiser alone and the whole linear (bf16 comparator: gelu then
    cuBLAS); and the rotation-free row-wise quantiser (backend.py:230-232)."""
    import torch
    import torch.nn.functional as F

    from tilegen_b200 import ops
    from tilegen_b200.synthetic import gaussian_weight, outlier_activations

    hbm = _peaks()[0]["hbm_gbs"]
    m, k, n = M_PER_RANK, 13824, 5120

    def timed(body):
        def f(e):
            e[0].record(stream)
            body()
            e[1].record(stream)

        for _ in range(3):
            f([torch.cuda.Event(enable_timing=True) for _ in range(2)])
        return round(statistics.mean(r[0] for r in _time_steps(f, iters, flush, stream)) * 1e3, 2)

    act_rows = []
    w = gaussian_weight(n, k, seed=1, dtype=torch.bfloat16, device=dev)
    wq, ws = ops.rotate_quant(w, GROUP)
    for dt in (torch.float16, torch.bfloat16):
        x = outlier_activations(m, k, seed=0, dtype=dt, device=dev)  # pre-activation
        wb = w.to(dt)
        row = {"dtype": "fp16" if dt == torch.float16 else "bf16", "act": "gelu_tanh", "M": m, "K": k, "N": n}
        row["quant_fused_us"] = timed(lambda: ops.quantize_act(x, GROUP, "gelu_tanh"))
        row["quant_unfused_us"] = timed(lambda: ops.rotate_quant(F.gelu(x, approximate="tanh"), GROUP))
        row["linear_fused_us"] = timed(
            lambda: ops.int8_gemm_dequant(*ops.quantize_act(x, GROUP, "gelu_tanh"), wq, ws, None, dt))
        row["linear_unfused_us"] = timed(
            lambda: ops.int8_gemm_dequant(*ops.rotate_quant(F.gelu(x, approximate="tanh"), GROUP), wq, ws, None, dt))
        row["bf16_gelu_cublas_us"] = timed(lambda: F.linear(F.gelu(x, approximate="tanh"), wb))
        row["speedup_vs_bf16"] = round(row["bf16_gelu_cublas_us"] / row["linear_fused_us"], 3)
        act_rows.append(row)
        del x, wb
    del w, wq, ws

    rw_rows = []
    for kk, mm in ((5120, 4096), (13824, 4096), (5120, 65536), (13824, 32768)):
        for dt in (torch.float16, torch.bfloat16):
            x = outlier_activations(mm, kk, seed=0, dtype=dt, device=dev)
            us = timed(lambda: ops.quantize_act(x, 1, None))
            gbs = (mm * kk * 3 + 4 * mm) / (us * 1e-6) / 1e9
            rw_rows.append([kk, mm, "fp16" if dt == torch.float16 else "bf16", us, round(gbs, 1),
                            round(gbs / hbm, 4)])
            del x
    return act_rows, rw_rows


def _ln_mod_table(dev, flush, stream, iters=20):
    """The DiT block's LayerNorm + adaLN modulation in front of qkv_proj at M = 4096
    (two samples of 2048 tokens, one modulation vector each): fused into the
    quantiser (``ops.quantize_ln_mod``) vs torch's ``F.layer_norm`` and the two
    elementwise ops, then the quantiser; the quantisation alone and the whole
    linear both ways, and the bf16 comparator (torch's ops, then cuBLAS)."""
    import torch
    import torch.nn.functional as F

    from tilegen_b200 import ops
    from tilegen_b200.synthetic import dit_modulation, gaussian_weight, residual_stream

    m, k, n = M_PER_RANK, 5120, 15360

    def timed(body):
        def f(e):
            e[0].record(stream)
            body()
            e[1].record(stream)

        for _ in range(3):
            f([torch.cuda.Event(enable_timing=True) for _ in range(2)])
        return round(statistics.median(r[0] for r in _time_steps(f, iters, flush, stream)) * 1e3, 2)

    rows = []
    w = gaussian_weight(n, k, seed=1, dtype=torch.bfloat16, device=dev)
    wq, ws = ops.rotate_quant(w, GROUP)
    for dt in (torch.float16, torch.bfloat16):
        x = residual_stream(m, k, seed=0, dtype=dt, device=dev)
        sc, sh = dit_modulation(2, k, seed=1, dtype=dt, device=dev)
        x3, sc3, sh3 = x.view(2, m // 2, k), sc.view(2, 1, k), sh.view(2, 1, k)
        wb = w.to(dt)

        def norm_mod():  # the DiT block's own form: per-sample vectors broadcast over tokens
            return (F.layer_norm(x3, (k,), eps=1e-6) * (1 + sc3) + sh3).view(m, k)

        row = {"dtype": "fp16" if dt == torch.float16 else "bf16", "M": m, "K": k, "N": n, "vectors": 2}
        row["quant_fused_us"] = timed(lambda: ops.quantize_ln_mod(x, GROUP, sc, sh))
        row["quant_unfused_us"] = timed(lambda: ops.rotate_quant(norm_mod(), GROUP))
        row["linear_fused_us"] = timed(
            lambda: ops.int8_gemm_dequant(*ops.quantize_ln_mod(x, GROUP, sc, sh), wq, ws, None, dt))
        row["linear_unfused_us"] = timed(
            lambda: ops.int8_gemm_dequant(*ops.rotate_quant(norm_mod(), GROUP), wq, ws, None, dt))
        row["bf16_norm_mod_cublas_us"] = timed(lambda: F.linear(norm_mod(), wb))
        row["speedup_vs_bf16"] = round(row["bf16_norm_mod_cublas_us"] / row["linear_fused_us"], 3)
        rows.append(row)
        del x, wb
    del w, wq, ws
    return rows


def _event_floor_us(dev, flush, stream, iters=30):
    """A one-element fill kernel timed like a single quantiser launch (between two
    events after an L2 flush): the fixed cost every such measurement carries."""
    import torch

    sink = torch.empty(1, dtype=torch.float32, device=dev)

    def f(e):
        e[0].record(stream)
        sink.zero_()
        e[1].record(stream)

    for _ in range(3):
        f([torch.cuda.Event(enable_timing=True) for _ in range(2)])
    return statistics.median(r[0] for r in _time_steps(f, iters, flush, stream)) * 1e3


def _graph_us(fn, flush, reps=10, iters=7):
    """Microseconds of ``fn`` replayed ``reps`` times from one CUDA graph, L2 flushed
    before each (cold weights, as in a model, and no launch gaps), less the same
    graph of flushes alone; median of ``iters``."""
    import torch

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
        flush.zero_()
    torch.cuda.current_stream().wait_stream(s)
    graphs = []
    for with_fn in (True, False):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(reps):
                flush.zero_()
                if with_fn:
                    fn()
        graphs.append(g)
    out = []
    for _ in range(iters):
        a, b, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        a.record()
        graphs[0].replay()
        b.record()
        graphs[1].replay()
        c.record()
        torch.cuda.synchronize()
        out.append((a.elapsed_time(b) - b.elapsed_time(c)) * 1e3 / reps)
    del graphs
    return statistics.median(out)


def _small_m_table(dev, flush, hbm_gbs):
    """Few-row linears (decode / preview steps): the routed int8 linear (rotate+quant,
    then the GEMV, split-K or tiled kernel that ``ops`` picks) against bf16 cuBLAS,
    both as whole linears replayed from a CUDA graph with L2 flushed before each."""
    import torch
    import torch.nn.functional as F

    from tilegen_b200 import ops
    from tilegen_b200.synthetic import DIT_SHAPES, dit_activations, gaussian_weight

    rows = []
    for name, k, n in DIT_SHAPES:
        w = gaussian_weight(n, k, seed=1, dtype=torch.bfloat16, device=dev)
        wq, ws = ops.rotate_quant(w, GROUP)
        for m in (1, 4, 16, 64, 128):
            x = dit_activations(name, m, seed=0, dtype=torch.float16, device=dev)
            xb = x.to(torch.bfloat16)
            kern = "gemv" if ops.gemv_route(m, n, k) else ("splitk" if ops.splitk_route(m, n, k) else "tiled")
            t8 = _graph_us(lambda: ops.int8_gemm_dequant(*ops.rotate_quant(x, GROUP), wq, ws, None, torch.float16),
                           flush)
            tb = _graph_us(lambda: F.linear(xb, w), flush)
            rows.append([name, m, kern, round(t8, 2), round(tb, 2), round(tb / t8, 3),
                         round(n * k / (t8 * 1e-6) / 1e9 / hbm_gbs, 3)])
        del w, wq, ws
    return rows


def _dit_block_bf16(dev, flush, stream, world, rank, tokens=65520, iters=10):
    """The DiT projection set on bf16 activations, `tokens` rows sharded over the ranks:
    per shape the max-over-ranks int8 linear and bf16 cuBLAS times and aggregate tokens/s."""
    import torch
    import torch.distributed as dist

    from tilegen_b200 import ops
    from tilegen_b200.sharding import shard_bounds
    from tilegen_b200.synthetic import DIT_SHAPES, dit_activations, gaussian_weight

    lo, hi = shard_bounds(tokens, world, rank)
    m = hi - lo
    rows = []
    for name, k, n in DIT_SHAPES:
        x = dit_activations(name, m, seed=rank, dtype=torch.bfloat16, device=dev)
        w = gaussian_weight(n, k, seed=1, dtype=torch.bfloat16, device=dev)
        wq, ws = ops.rotate_quant(w, GROUP)

        def lin(e):
            e[0].record(stream)
            xq, xs = ops.rotate_quant(x, GROUP)
            ops.int8_gemm_dequant(xq, xs, wq, ws, None, torch.bfloat16)
            e[1].record(stream)

        for _ in range(2):
            lin([torch.cuda.Event(enable_timing=True) for _ in range(2)])
        tl = statistics.mean(r[0] for r in _time_steps(lin, iters, flush, stream)) * 1e3
        tb = _bf16_linear_us(x, w, iters, flush, stream)
        t = torch.tensor([tl, tb], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tl, tb = float(t[0]), float(t[1])
        rows.append({"shape": name, "K": k, "N": n, "rows_per_gpu": m, "int8_linear_us": round(tl, 1),
                     "bf16_cublas_us": round(tb, 1), "speedup_vs_bf16": round(tb / tl, 3),
                     "tokens_per_s": round(tokens / (tl * 1e-6), 1)})
        del x, w, wq, ws
    return rows


def _gather_table(dev, flush, stream, world, rank, tokens=65520, iters=10):
    """N > 1 only: the optional all-gather of a row-sharded output (tilegen_b200.sharding.
    gather_rows, NCCL over NVLink), outside the hot path.  o_proj's fp16 output of
    `tokens` rows sharded over the ranks: the gather alone; then the gather and the next
    layer (ffn_up on the local rows) back to back vs with the gather in flight while the
    next layer runs.  Max over ranks of CUDA-event times."""
    import torch
    import torch.distributed as dist

    from tilegen_b200 import ops
    from tilegen_b200.sharding import gather_rows, shard_bounds
    from tilegen_b200.synthetic import gaussian_weight

    lo, hi = shard_bounds(tokens, world, rank)
    m = hi - lo
    y = (torch.randn(m, 5120, generator=torch.Generator(device=dev).manual_seed(rank), device=dev)
         .to(torch.float16))
    w = gaussian_weight(13824, 5120, seed=1, dtype=torch.float16, device=dev)
    wq, ws = ops.rotate_quant(w, GROUP)
    del w

    def nxt():
        return ops.int8_gemm_dequant(*ops.rotate_quant(y, GROUP), wq, ws, None, torch.float16)

    def gather_only(e):
        e[0].record(stream)
        gather_rows(y, tokens)
        e[1].record(stream)

    def serial(e):
        e[0].record(stream)
        gather_rows(y, tokens)
        nxt()
        e[1].record(stream)

    # The persistent kernels normally take every SM; a collective in flight holds
    # some, which would keep part of their grid waiting until it ends.  While a
    # gather runs, the next layer leaves it SMs: NCCL's all-gather kernels (on
    # B200 with NCCL 2.28 they hold about 32 SMs at 2 GPUs and 64 at 8), or 2 for
    # the copy-engine gather's one-element all-reduce.
    sms = torch.cuda.get_device_properties(dev).multi_processor_count

    def overlapped_with(reserve):
        def f(e):
            e[0].record(stream)
            pending = gather_rows(y, tokens, async_op=True)
            with ops.sm_budget(sms - reserve if reserve else 0):
                nxt()
            pending.wait()
            e[1].record(stream)
        return f

    overlapped = overlapped_with(0)

    def next_only(e):
        e[0].record(stream)
        nxt()
        e[1].record(stream)

    # The same gather by copy engines over NVLink (PeerRowGather): this rank's rows
    # are written into its mapped buffer once per buffer (a GEMM would write them
    # there directly), then each step pulls the peers' blocks.
    from tilegen_b200.sharding import PeerRowGather

    try:
        pg = PeerRowGather(tokens, 5120, torch.float16, dev)  # raises on every rank together
    except RuntimeError as e:
        pg, pg_error = None, str(e)[:200]
    if pg is not None:
        for _ in range(2):
            pg.local().copy_(y)
            pg.start().wait()

    def ce_only(e):
        e[0].record(stream)
        pg.start().wait()
        e[1].record(stream)

    def ce_serial(e):
        e[0].record(stream)
        pg.start().wait()
        nxt()
        e[1].record(stream)

    def ce_overlapped(e):
        e[0].record(stream)
        pending = pg.start()
        with ops.sm_budget(sms - 2):
            nxt()
        pending.wait()
        e[1].record(stream)

    res = []
    fns = (gather_only, next_only, serial, overlapped, overlapped_with(32), overlapped_with(64)) + \
        ((ce_only, ce_serial, ce_overlapped) if pg else ())
    for fn in fns:
        for _ in range(3):
            fn([torch.cuda.Event(enable_timing=True) for _ in range(2)])
        res.append(statistics.median(r[0] for r in _time_steps(fn, iters, flush, stream)) * 1e3)
    torch.cuda.synchronize()
    same = torch.tensor([0.0], device=dev, dtype=torch.float64)
    if pg is not None:
        y_ce = pg.start().wait().clone()
        y_nccl = gather_rows(y, tokens)
        same.fill_(float(torch.equal(y_ce, y_nccl)))
        pg.close()
    t = torch.tensor(res, device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    g, nx, se, ov, ov32, ov64 = (float(v) for v in t[:6])
    per = -(-tokens // world)
    moved = (world - 1) * per * 5120 * 2  # bytes each rank receives
    out = {"tokens": tokens, "N": 5120, "dtype": "fp16", "gather_us": round(g, 1),
           "gather_bus_gbs": round(moved / (g * 1e-6) / 1e9, 1), "next_layer": "ffn_up on the local rows",
           "next_layer_us": round(nx, 1), "gather_then_next_us": round(se, 1),
           "gather_overlapped_with_next_us": round(ov, 1),
           "gather_overlapped_next_on_fewer_sms_us": {"32 SMs left to NCCL": round(ov32, 1),
                                                     "64 SMs left to NCCL": round(ov64, 1)},
           "gather_overlapped_best_us": round(min(ov, ov32, ov64), 1)}
    if pg is None:
        out["copy_engine"] = {"error": pg_error}
        return out
    ce, ces, ceo = (float(v) for v in t[6:])
    out["copy_engine"] = {"gather_us": round(ce, 1), "gather_bus_gbs": round(moved / (ce * 1e-6) / 1e9, 1),
                          "gather_then_next_us": round(ces, 1),
                          "gather_overlapped_with_next_us": round(ceo, 1),
                          "overlap_note": "the next layer on all SMs but 2 (ops.sm_budget)",
                          "equal_to_nccl_gather": bool(same.item() == 1.0),
                          "path": "tilegen_b200.sharding.PeerRowGather: a one-element NCCL all-reduce as the "
                                  "ready signal, then one cudaMemcpyAsync per peer from its mapped buffer, "
                                  "each on its own stream (copy engines over NVLink, no SMs)"}
    return out


def run_tilegen(args):
    import torch
    import torch.distributed as dist

    world, rank, local = _setup_dist(args)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from tilegen.kernels.int8_convrot import quantize_convrot
    from tilegen.quant.int8_ops import int8_matmul_dequant_chunked
    from tilegen_b200 import _lib, ops
    from tilegen_b200.synthetic import gaussian_weight, outlier_activations

    peaks, peak_kind = _peaks()
    name, k, n = SHAPE
    m = M_PER_RANK
    x = outlier_activations(m, k, seed=rank, dtype=torch.float16, device=dev)
    w = gaussian_weight(n, k, seed=1000, dtype=torch.bfloat16, device=dev)
    wq, ws = ops.rotate_quant(w, GROUP)
    flush = L2Flush(dev)
    stream = torch.cuda.current_stream()

    # One step = the whole linear (quantiser, then the GEMM launched as its
    # programmatic dependent, so its prologue overlaps the quantiser's tail).
    def step(e):
        e[0].record(stream)
        xq, xs = ops.rotate_quant(x, GROUP)
        ops.int8_gemm_dequant(xq, xs, wq, ws, None, torch.float16)
        e[1].record(stream)

    # The same with an event between the kernels: per-kernel durations for the
    # rooflines (no overlap across the middle event).
    def split_step(e):
        e[0].record(stream)
        xq, xs = ops.rotate_quant(x, GROUP)
        e[1].record(stream)
        ops.int8_gemm_dequant(xq, xs, wq, ws, None, torch.float16)
        e[2].record(stream)

    for _ in range(max(3, args.warmup)):
        step([torch.cuda.Event(enable_timing=True) for _ in range(2)])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    with ClockSampler(local) as clk:
        t = _time_steps(step, args.steps, flush, stream, marks=1)
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    if world > 1:
        dist.barrier()
    clocks = clk.summary()
    total_ms = sum(r[0] for r in t)
    ts = _time_steps(split_step, max(5, min(args.steps, 50)), flush, stream, marks=2)
    tq = [r[0] for r in ts]
    tg = [r[1] for r in ts]
    tot = torch.tensor([total_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    max_total_ms = float(tot.item())
    value_us = max_total_ms * 1e3 / (world * args.steps)

    if args.quick:
        if world > 1:
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"quick": True, "value_us": round(value_us, 3), "quant_us": round(statistics.mean(tq) * 1e3, 2),
                              "gemm_us": round(statistics.mean(tg) * 1e3, 2), "clocks": clocks}), flush=True)
        return

    # ---- end to end with host buffers, copies timed ----
    # Headline: the reference-facing plugin call, tilegen.comfyui.backend.int8_linear
    # (what comfy_kitchen's registry dispatches to), between a pinned host->device
    # copy of x and a device->host copy of the output, one stream.  Also: the
    # same through the quantiser and GEMM API calls, and this repository's
    # host-buffer linear (tilegen_b200.streaming.int8_linear_host: row chunks with
    # H2D / kernels / D2H overlapped on three streams, replayed as one CUDA graph).
    from tilegen.comfyui import backend as plugin
    from tilegen_b200.streaming import int8_linear_host

    x_host = x.cpu().pin_memory()
    out_host = torch.empty((m, n), dtype=torch.float16).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_plugin_step(e):
        e[0].record(stream)
        x_dev.copy_(x_host, non_blocking=True)
        y = plugin.int8_linear(x_dev, wq, ws, None, torch.float16, convrot=True, convrot_groupsize=GROUP)
        out_host.copy_(y, non_blocking=True)
        e[1].record(stream)

    def e2e_step(e):
        e[0].record(stream)
        int8_linear_host(x_host, wq, ws, None, torch.float16, out=out_host, group_size=GROUP, graph=True)
        e[1].record(stream)

    def e2e_serial_step(e):
        e[0].record(stream)
        x_dev.copy_(x_host, non_blocking=True)
        xq, xs = quantize_convrot(x_dev, GROUP, backend="fht")
        y = int8_matmul_dequant_chunked(xq, xs, wq, ws, None, torch.float16)
        out_host.copy_(y, non_blocking=True)
        e[1].record(stream)

    def e2e_time(fn):
        for _ in range(3):
            fn([torch.cuda.Event(enable_timing=True) for _ in range(2)])
        if world > 1:
            dist.barrier()
        te = _time_steps(fn, max(3, min(args.steps, 50)), flush, stream)
        tot = torch.tensor([sum(r[0] for r in te)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(tot, op=dist.ReduceOp.MAX)
        return float(tot.item()) * 1e3 / (world * len(te))

    e2e_plugin_us = e2e_time(e2e_plugin_step)
    plugin_out = out_host.clone()
    e2e_us = e2e_time(e2e_step)
    e2e_serial_us = e2e_time(e2e_serial_step)
    ref_out = out_host.clone()
    e2e_step([torch.cuda.Event(enable_timing=True) for _ in range(2)])
    torch.cuda.synchronize()
    e2e_bitexact = bool(torch.equal(out_host.view(torch.int16), ref_out.view(torch.int16))
                        and torch.equal(plugin_out.view(torch.int16), ref_out.view(torch.int16)))

    # ---- comparators ----
    bf16_us = _bf16_linear_us(x, w, max(5, min(args.steps, 50)), flush, stream)
    int8_lib_tops = _int_mm_tops(dev)
    status = _lib.device_status(local)

    shapes = cpu = sweep = act_table = small_m = ln_table = None
    event_floor = _event_floor_us(dev, flush, stream)
    if world == 1:
        shapes = _shape_table(dev, flush, stream)
        small_m = _small_m_table(dev, flush, peaks["hbm_gbs"])
        sweep = _quant_sweep(dev, flush, stream)
        act_table = _input_act_table(dev, flush, stream)
        ln_table = _ln_mod_table(dev, flush, stream)
    # Last: seconds of sustained load that leave the GPU at its power cap.
    if world > 1:
        dist.barrier()
    block = _dit_block_bf16(dev, flush, stream, world, rank)
    gather = _gather_table(dev, flush, stream, world, rank) if world > 1 else None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu_s, cl, nsteps = _cpu_baseline(k, n)
        cpu = {"value": round(cpu_s * 1e6, 1), "unit": "us", "cores": cl.threads, "kind": cl.kind,
               "sample": f"{nsteps} " + cl.sample()}

    if world > 1:
        if rank == 0:
            pass
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    gemm_ms = statistics.mean(tg)
    quant_ms = statistics.mean(tq)
    gemm_tops = 2 * m * n * k / (gemm_ms * 1e-3) / 1e12
    quant_bytes = m * k * 2 + m * k + 4 * m
    quant_gbs = quant_bytes / (quant_ms * 1e-3) / 1e9
    int8_peak = 2.0 * peaks["bf16_tflops"]
    lin_us = value_us if world == 1 else (quant_ms + gemm_ms) * 1e3
    line = {
        "metric": METRIC,
        "value": round(value_us, 3), "unit": "us", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": round(max_total_ms / args.steps, 5),
        "higher_is_better": False, "scaling": "weak",
        "vs_baseline": round(value_us / PUBLISHED_QKV_US, 5),
        "vs_baseline_ref": "tilegen FHT int8_convrot qkv_proj on RTX 2080 Ti, 10.55 ms (README.md:9)",
        "dtype": "int8", "data": "synthetic",
        "config": _config(world),
        "speedup_vs_bf16_cublas": round(bf16_us / lin_us, 3), "bf16_cublas_us": round(bf16_us, 2),
        "quant_us": round(quant_ms * 1e3, 2), "gemm_us": round(gemm_ms * 1e3, 2),
        "kernel_split_note": "quant_us/gemm_us: each kernel timed alone (event between them); value: both back to back",
        "roofline": {"bound": "tensor", "kernel": "gemm_i8_dequant_kernel", "achieved": round(gemm_tops, 1),
                     "peak": round(int8_peak, 1), "unit": "TOP/s", "frac": round(gemm_tops / int8_peak, 4),
                     "peak_source": f"2 x {peak_kind} bf16 cuBLAS burst (dense int8 = 2 x dense bf16)",
                     "traffic": GEMM_TRAFFIC_BYTES, "traffic_source": GEMM_TRAFFIC_SOURCE,
                     "algorithmic_ops_per_launch": 2 * m * n * k,
                     "vs_cublaslt_int8_tops": round(int8_lib_tops, 1),
                     "vs_nominal_int8": round(gemm_tops / NOMINAL_INT8_TOPS, 4)},
        "quant_roofline": {"bound": "hbm", "kernel": "rotquant_kernel", "achieved": round(quant_gbs, 1),
                           "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(quant_gbs / peaks["hbm_gbs"], 4),
                           "peak_source": peak_kind, "algorithmic_bytes_per_launch": quant_bytes,
                           "traffic": QUANT_TRAFFIC_BYTES, "traffic_source": QUANT_TRAFFIC_SOURCE,
                           "timing": "one launch between two events after an L2 flush (quant_us)",
                           "event_floor_us": round(event_floor, 2)},
        "e2e": {"value": round(e2e_plugin_us, 2), "unit": "us", "h2d_bytes_per_step": x.numel() * 2,
                "d2h_bytes_per_step": m * n * 2,
                "path": "one stream: pinned host x -> device, tilegen.comfyui.backend.int8_linear(convrot=True) "
                        "(the reference's plugin call), output -> pinned host",
                "api_calls_us": round(e2e_serial_us, 2),
                "api_calls_path": "one stream: H2D of x, tilegen.kernels.quantize_convrot, "
                                  "tilegen.quant.int8_matmul_dequant_chunked, D2H of the output",
                "host_linear_us": round(e2e_us, 2),
                "host_linear_path": "pinned host x -> tilegen_b200.streaming.int8_linear_host(graph=True) (chunks "
                                    "of 256, 512, then 1024 rows: H2D, rotate+quant + GEMM, D2H on three streams, "
                                    "replayed as one CUDA graph) -> pinned host out",
                "bit_identical_across_paths": e2e_bitexact},
        "gpu_launches": 2 * args.steps,  # rotquant_kernel + gemm_i8_dequant_kernel per step (timed region)
        "clocks": clocks,
        "device_status": status,
        "wall_s_timed_region": round(wall, 3),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if shapes is not None:
        line["dit_shapes"] = shapes
    line["dit_block_bf16"] = {"tokens": 65520, "rows_sharded_over": world, "shapes": block}
    if sweep is not None:
        for r in sweep:
            if r[:4] == [GROUP, k, m, "fp16"] and r[7] is not None:
                line["quant_roofline"]["back_to_back"] = {
                    "us": r[7], "frac": r[8],
                    "timing": "launches back to back over inputs that together exceed twice the L2 (quant_sweep "
                              "us_stream)"}
        line["quant_sweep"] = {"columns": ["group", "K", "M", "dtype", "us", "GB/s", "frac_of_hbm", "us_stream",
                                           "frac_of_hbm_stream"], "rows": sweep}
    if gather is not None:
        line["gather_rows"] = gather
    if small_m is not None:
        line["small_m_linears"] = {"columns": ["shape", "M", "kernel", "int8_linear_us", "bf16_cublas_us",
                                               "speedup_vs_bf16", "weight_stream_frac_of_hbm"], "rows": small_m,
                                   "timing": "whole linears (rotate+quant + GEMM; bf16: F.linear) replayed 10 at a "
                                             "time from a CUDA graph, L2 flushed before each, flush time subtracted"}
    if ln_table is not None:
        line["norm_modulation_qkv"] = ln_table
    if act_table is not None:
        line["input_act_ffn_down"] = act_table[0]
        line["rowwise_quant"] = {"columns": ["K", "M", "dtype", "us", "GB/s", "frac_of_hbm"], "rows": act_table[1]}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("tilegen", "reference"), default="tilegen")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline sample")
    ap.add_argument("--quick", action="store_true",
                    help="only the timed loop (no e2e, comparators, shape table or CPU baseline); for profiling")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_tilegen(args)


if __name__ == "__main__":
    main()
