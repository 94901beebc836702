#!/usr/bin/env python3
"""Benchmark of the B200 matrix-multiply hot path (one JSON line on rank 0).

Headline workload (BASELINE metric "FP16 GEMM TFLOP/s (4096^3) & GEMV HBM GB/s
(4096x14336); % of B200 peak"):

* step  = one FP16 GEMM C[4096,4096] = A[4096,4096] B[4096,4096] on tcgen05
  (engine_cuda_matmul_f16), A, B ~ N(0,1), FP32 accumulate.  Operands rotate over
  a pool of sets larger than the 126 MB L2, so every step starts cold.
  ``value`` = whole-job TFLOP/s over the K timed steps (sum over ranks of the work
  / max over ranks of the CUDA-event time).
* ``gemv`` = the decode GEMV y[4096] = W[4096,14336] x (engine_cuda_gemv_f16_nk),
  W ~ N(0,0.02), x ~ N(0,1), over a rotating pool of weight matrices (448 MiB),
  reported in HBM GB/s of algorithmic bytes.
* ``e2e`` = the GEMM metric through the C ABI with pinned HOST buffers: each step
  copies A and B host->device, runs the GEMM and reads C back.
* ``cpu_baseline`` = the reference engine's own cpu::matmul (oracle/_ref) on a
  bounded row sample of the same GEMM, all host cores, rank 0 at N=1 only.

``--impl reference`` times the reference's CPU implementation alone (the
reference has no GPU path for this configuration) and prints its line.
``--workload tp-decode|tp-prefill`` runs the Llama-3-8B-shaped tensor-parallel
projection layer set instead (see bare-metal-llm-engine_b200/tp.py);
``--workload tp-comm`` (torchrun, >= 2 GPUs) times the row-split projection with
its all-reduce: NVLink fused vs NVLink / NCCL after the projection.
``--workload kernel --case NAME`` runs one configuration alone for a few
launches (the ncu summaries in profiles/ are captured on it).
"""
from __future__ import annotations

import argparse
import ctypes
import importlib.util
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
PKG_DIR = ROOT / "bare-metal-llm-engine_b200"
METRIC = "FP16 GEMM TFLOP/s (4096³) & GEMV HBM GB/s (4096×14336); % of B200 peak"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_pkg():
    if "bmle_b200" in sys.modules:
        return sys.modules["bmle_b200"]
    spec = importlib.util.spec_from_file_location(
        "bmle_b200", PKG_DIR / "__init__.py", submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["bmle_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def traffic_for(kernel: str):
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    v = d.get(kernel)
    return None if v is None else float(v.get("bytes_per_launch", v) if isinstance(v, dict) else v)


# --------------------------------------------------------------- clock sampling

_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
            0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
            0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
            0x100: "display_clock_setting"}


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML during the timed region."""

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self.period = period_s
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = device_index
            if vis:
                try:
                    idx = int(vis.split(",")[device_index])
                except ValueError:
                    idx = device_index
            self._h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: report no clocks rather than fail
            self._h = None

    def _sample(self):
        nv = self._nv
        mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
        try:
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        except AttributeError:
            r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
        self.samples.append(mhz)
        self.reasons |= int(r) & ~0x1  # idle is not a slowdown

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(self.period)

    def __enter__(self):
        if self._h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        if self._h is not None:
            self._stop.set()
            self._t.join()
            try:
                self._sample()
            except Exception:
                pass

    def median(self):
        """Median SM MHz of the samples (None without NVML or samples)."""
        return statistics.median(self.samples) if (self._h is not None and self.samples) else None

    def summary(self):
        if self._h is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"]}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": [n for b, n in _REASONS.items() if self.reasons & b]}


# --------------------------------------------------------------- CPU baseline

def _oracle():
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    import oracle

    return oracle


def cpu_gemm_sample(A32, B32, rows: int, nthreads: int):
    """Times the reference's cpu::matmul (oracle/_ref) -- else the oracle port --
    on `rows` rows of the GEMM.  Returns (seconds, kind)."""
    orc = _oracle()
    sub = np.ascontiguousarray(A32[:rows])
    M, K = sub.shape
    N = B32.shape[1]
    C = np.empty((M, N), np.float32)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    if orc.ref_available():
        t0 = time.perf_counter()
        orc.ref_lib().ref_matmul(p(sub), p(B32), p(C), M, N, K, nthreads)
        return time.perf_counter() - t0, "reference"
    t0 = time.perf_counter()
    orc.lib().orc_matmul_mt(p(sub), p(B32), p(C), M, N, K, nthreads)
    return time.perf_counter() - t0, "port"


def cpu_gemm_throughput(target_s: float, nthreads: int, n: int = 4096):
    rng = np.random.default_rng(20260826)
    A32 = rng.standard_normal((max(nthreads * 64, 64), n)).astype(np.float16).astype(np.float32)
    B32 = rng.standard_normal((n, n)).astype(np.float16).astype(np.float32)
    rows = nthreads
    t, kind = cpu_gemm_sample(A32, B32, rows, nthreads)
    while t < target_s * 0.5 and rows < A32.shape[0]:
        rows = min(A32.shape[0], int(rows * max(2.0, target_s / max(t, 1e-3))))
        rows = max(nthreads, rows - rows % nthreads)
        t, kind = cpu_gemm_sample(A32, B32, rows, nthreads)
    flops = 2.0 * rows * n * n
    return flops / t / 1e12, kind, rows, t


def environment(with_gpu: bool) -> dict:
    """Provenance of a bench line: the library build (build_info.json, written by
    build.py), the host, and with_gpu the device and driver."""
    import platform

    env = {"python": platform.python_version(), "host_cores": os.cpu_count()}
    try:
        with open("/proc/cpuinfo") as f:
            env["host_cpu"] = next((ln.split(":", 1)[1].strip() for ln in f
                                    if ln.startswith("model name")), platform.processor())
    except OSError:
        env["host_cpu"] = platform.processor()
    bi = PKG_DIR / "build_info.json"
    env["build"] = json.loads(bi.read_text()) if bi.exists() else None
    if with_gpu:
        import torch

        p = torch.cuda.get_device_properties(torch.cuda.current_device())
        env.update(device=p.name, sm_count=p.multi_processor_count,
                   compute_capability=f"{p.major}.{p.minor}",
                   memory_gib=round(p.total_memory / 2 ** 30, 1), torch=torch.__version__)
        try:
            import pynvml

            pynvml.nvmlInit()
            v = pynvml.nvmlSystemGetDriverVersion()
            env["driver"] = v.decode() if isinstance(v, bytes) else v
        except Exception:
            env["driver"] = None
    return env


def headline_config(world: int) -> dict:
    """The workload both arms quote, identical on both (how the reference arm ran
    it is a separate top-level key of its line)."""
    return {"workload": "FP16 GEMM C[4096,4096] = A[4096,4096] B[4096,4096] (FP32 accumulate) "
                        "+ decode GEMV W[4096,14336] x",
            "M": 4096, "N": 4096, "K": 4096, "parallelism": f"replicas x{world}",
            "l2": "rotating operand pools larger than the 126 MB L2 "
                  "(4 x 96 MiB GEMM sets, 4 x 112 MiB GEMV weights)"}


def cpu_single_thread(cpu_seconds: float) -> dict:
    """The reference's own framing (one thread) beside the all-cores figure: the
    same GEMM on a smaller row sample, about a quarter of the all-cores time."""
    v, kind, rows, t = cpu_gemm_throughput(max(1.0, min(5.0, cpu_seconds / 4)), 1)
    return {"value": v, "unit": "TFLOP/s", "cores": 1, "kind": kind,
            "sample": f"{rows} of 4096 output rows of the 4096^3 GEMM, {t:.1f} s"}


# --------------------------------------------------------------- distributed

def dist_setup(gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# --------------------------------------------------------------- reference arm

def run_reference(args):
    world, rank, _ = dist_setup(args.gpus)
    if rank != 0:
        return 0
    orc = _oracle()
    nthreads = orc.ncores()
    n = 4096
    rng = np.random.default_rng(20260826)
    A32 = rng.standard_normal((nthreads * 8, n)).astype(np.float16).astype(np.float32)
    B32 = rng.standard_normal((n, n)).astype(np.float16).astype(np.float32)
    # size one step to ~0.5 s of CPU work
    rows = nthreads
    t, kind = cpu_gemm_sample(A32, B32, rows, nthreads)
    while t < 0.25 and rows < A32.shape[0]:
        rows = min(A32.shape[0], rows * 2)
        t, kind = cpu_gemm_sample(A32, B32, rows, nthreads)
    for _ in range(args.warmup):
        cpu_gemm_sample(A32, B32, rows, nthreads)
    times = []
    for _ in range(args.steps):
        dt, kind = cpu_gemm_sample(A32, B32, rows, nthreads)
        times.append(dt)
    total = sum(times)
    flops = 2.0 * rows * n * n * args.steps
    value = flops / total / 1e12
    sample = (f"{rows} of 4096 output rows of the 4096^3 GEMM per step "
              f"({'engine::cpu::matmul' if kind == 'reference' else 'oracle port'}, "
              f"FP16 inputs widened to float)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (fp64 accumulate)", "data": "synthetic",
        "config": headline_config(world),
        "implementation": "the reference's CPU code (engine::cpu::matmul), a row sample of the "
                          "GEMM per step",
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": nthreads, "kind": kind,
                         "sample": sample, "single_thread": cpu_single_thread(4.0)},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "environment": environment(with_gpu=False),
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------- headline (ours)

def time_launches(torch, fn, sets, steps, warmup, stream, per_launch=True):
    """Runs fn(set) warmup + steps times on rotating sets; returns per-launch and
    total ms.  per_launch=False records only the two events around the steps, so
    the launches run back to back as a caller issues them (a programmatic
    dependent launch starts its set-up while the previous kernel drains; an event
    recorded between two launches would serialise them); the per-launch list is
    then empty."""
    for i in range(warmup):
        fn(sets[i % len(sets)])
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps if per_launch else 0)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(steps):
        if per_launch:
            ev[i][0].record(stream)
        fn(sets[i % len(sets)])
        if per_launch:
            ev[i][1].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    per = [a.elapsed_time(b) for a, b in ev]
    return per, t0.elapsed_time(t1)


def time_graph(torch, fn, sets, steps, warmup, reps=5, stats=False, min_ms=0.0):
    """Captures `steps` launches (rotating operand sets) in one CUDA graph and
    times at least `reps` replays -- more, until `min_ms` of device time has
    passed, so a clock sampler sees the kernel under load -- with CUDA events on
    the replay stream; returns the median ms per launch, or with stats=True
    {"median", "q1", "q3"} over the replays.  Launch-bound kernels (~5-25 us)
    are timed without host enqueue gaps."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for i in range(warmup):
            fn(sets[i % len(sets)], side.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for i in range(steps):
            fn(sets[i % len(sets)], side.cuda_stream)
    g.replay()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    per = []
    while len(per) < max(reps, 1) or sum(per) * steps < min_ms:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(s)
        g.replay()
        e1.record(s)
        torch.cuda.synchronize()
        per.append(e0.elapsed_time(e1) / steps)
        if len(per) >= 400:
            break
    del g
    med = statistics.median(per)
    if not stats:
        return med
    q = statistics.quantiles(per, n=4) if len(per) > 1 else [med, med, med]
    return {"median": med, "q1": q[0], "q3": q[2]}


def secondary_configs(torch, pkg, dev, g, world, args, local=0):
    """The other BASELINE configurations, one entry each: CUDA-graph timing over
    operand pools larger than L2, the median SM clock sampled while each one
    runs ("mhz") and, for the HBM-bound lines, the time in clock cycles
    ("kcyc" = us x MHz / 1000), which separates a slower clock from a slower
    kernel."""
    out = {}

    def timed(name, fn, sets, steps, warmup, byt=None, flops=None, extra=None):
        with ClockSampler(local, period_s=0.001) as clk:
            ms = time_graph(torch, fn, sets, steps, warmup, min_ms=30.0)
        d = {"us": ms * 1e3, "mhz": clk.median()}
        if byt is not None:
            d["gbs"] = byt / (ms * 1e-3) / 1e9
            if d["mhz"]:
                d["kcyc"] = ms * 1e3 * d["mhz"] / 1e3
        if flops is not None:
            d["tflops"] = flops / (ms * 1e-3) / 1e12
        if extra:
            d.update(extra)
        out[name] = d

    # Config 2: the other two decode GEMV shapes (rotating pools > L2), first in
    # the sequence, beside the headline shape measured just before
    for (N, K, nsets) in ((4096, 4096, 6), (14336, 4096, 4)):
        sets = [((torch.randn(N, K, device=dev, generator=g) * 0.02).half(),
                 torch.randn(K, device=dev, generator=g).half(),
                 torch.empty(N, device=dev, dtype=torch.float16)) for _ in range(nsets)]
        fn = lambda s, st, N=N, K=K: pkg.cuda.gemv_f16_nk(  # noqa: E731
            s[0].data_ptr(), s[1].data_ptr(), 0, s[2].data_ptr(), N, K, st)
        timed(f"gemv_{N}x{K}", fn, sets, 60, 5, byt=2.0 * (N * K + K + N))
        del sets
    # Config 3: fused RMSNorm -> QKV, W[6144,4096], B in {1, 16}
    N, K = 6144, 4096
    pool = [(torch.randn(16, K, device=dev, generator=g).half(),
             (1 + 0.1 * torch.randn(K, device=dev, generator=g)).half(),
             (torch.randn(N, K, device=dev, generator=g) * 0.02).half(),
             torch.empty(16, N, device=dev, dtype=torch.float16)) for _ in range(5)]
    for B in (1, 16):
        fn = lambda s, st, B=B: pkg.cuda.rmsnorm_linear_f16(  # noqa: E731
            s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), 0, s[3].data_ptr(), B, N, K, 1e-5, st)
        timed(f"rmsnorm_qkv_b{B}", fn, pool, 100, 5, byt=2.0 * (N * K + B * K + K + B * N))
    del pool
    # Block-quantised decode GEMV (GGUF Q8_0 / Q4_0, the engine's declared formats),
    # 4096x14336, in the streamed layout; random payload bytes and scales (timing
    # only: the same bytes and work as real quantised weights).
    N, K = 4096, 14336
    for qtype, name, pay, nsets in ((8, "q8_0", K, 4), (4, "q4_0", K // 2, 6)):
        sets = [(torch.randint(0, 256, (N, pay), device=dev, generator=g, dtype=torch.uint8),
                 (torch.rand(N, K // 32, device=dev, generator=g) * 1e-3).half(),
                 torch.randn(K, device=dev, generator=g).half(),
                 torch.empty(N, device=dev, dtype=torch.float16)) for _ in range(nsets)]
        fn = lambda s, st, qt=qtype: pkg.cuda.gemv_q_nk(  # noqa: E731
            qt, s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), 0, s[3].data_ptr(), N, K, st)
        byt = N * pay + 2.0 * (N * K // 32) + 2.0 * (K + N)
        timed(f"gemv_{name}_{N}x{K}", fn, sets, 60, 5, byt=byt, extra={"bytes_per_launch": byt})
        del sets
    torch.cuda.empty_cache()
    # Config 1: the reference's FP32 register-tiled matmul at 512^3 (48 rotating
    # 3 MiB sets = 144 MiB > L2): a latency-bound launch, so it runs with the
    # other short lines, before the long tensor-core work lowers the clock.
    n = 512
    sets = [(torch.rand(n, n, device=dev, generator=g) * 2 - 1,
             torch.rand(n, n, device=dev, generator=g) * 2 - 1,
             torch.empty(n, n, device=dev)) for _ in range(48)]
    fn = lambda s, st: pkg.cuda.matmul_register_tiled(  # noqa: E731
        s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), n, n, n, st)
    timed("matmul_f32_512", fn, sets, 96, 5, flops=2.0 * n ** 3)
    del sets
    # Attention (the engine's attention_prefill / attention_decode launchers),
    # ahead of the long prefill GEMMs, whose power draw lowers the clock after them;
    # Llama-3-8B heads (32 query, 8 KV, d = 128): causal prefill at S = 2048
    # (FLOPs of the causal half: 2 * S^2 * d * heads), and decode of one token
    # over 4096 and 16384 cached keys (bytes: K and V once).
    H, Hk, d = 32, 8, 128
    S = 2048
    sets = [(torch.randn(S, H, d, device=dev, generator=g).half(),
             torch.randn(Hk, S, d, device=dev, generator=g).half(),
             torch.randn(Hk, S, d, device=dev, generator=g).half(),
             torch.empty(S, H, d, device=dev, dtype=torch.float16)) for _ in range(2)]
    fn = lambda s, st: pkg.cuda.attention_prefill(  # noqa: E731
        s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), s[3].data_ptr(), S, S, H, Hk, d, S * d,
        d ** -0.5, 0, True, 0, st)
    timed("attn_prefill_s2048", fn, sets, 20, 3, flops=2.0 * S * S * d * H)
    del sets
    for kv, nsets in ((4096, 10), (16384, 3)):
        sets = [(torch.randn(H, d, device=dev, generator=g).half(),
                 torch.randn(Hk, kv, d, device=dev, generator=g).half(),
                 torch.randn(Hk, kv, d, device=dev, generator=g).half(),
                 torch.empty(H, d, device=dev, dtype=torch.float16)) for _ in range(nsets)]
        fn = lambda s, st, kv=kv: pkg.cuda.attention_decode(  # noqa: E731
            s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), s[3].data_ptr(), kv, H, Hk, d,
            kv * d, d ** -0.5, 0, st)
        timed(f"attn_decode_{kv}", fn, sets, 60, 5, byt=2.0 * 2 * Hk * kv * d)
        del sets
    torch.cuda.empty_cache()
    # Config 4b: X[S,4096] W[14336,4096]^T
    N, K = 14336, 4096
    Ws = [(torch.randn(N, K, device=dev, generator=g) * 0.02).half() for _ in range(2)]
    for S in (512, 2048, 4096):
        X = torch.randn(S, K, device=dev, generator=g).half()
        Y = torch.empty(S, N, device=dev, dtype=torch.float16)
        sets = [(X, W, Y) for W in Ws]
        fn = lambda s, st, S=S: pkg.cuda.linear_f16(  # noqa: E731
            s[0].data_ptr(), s[1].data_ptr(), 0, s[2].data_ptr(), S, N, K, st)
        timed(f"prefill_s{S}", fn, sets, 10 if S >= 2048 else 20, 3, flops=2.0 * S * N * K)
        del X, Y, sets
    del Ws
    torch.cuda.empty_cache()
    # The 14336x4096 GEMV again, right after the prefill GEMMs: the same kernel
    # and weights as the entry at the top of the sequence, so any difference in
    # "us" or "kcyc" is the GPU's state after long tensor-core work.
    N, K = 14336, 4096
    sets = [((torch.randn(N, K, device=dev, generator=g) * 0.02).half(),
             torch.randn(K, device=dev, generator=g).half(),
             torch.empty(N, device=dev, dtype=torch.float16)) for _ in range(4)]
    fn = lambda s, st: pkg.cuda.gemv_f16_nk(  # noqa: E731
        s[0].data_ptr(), s[1].data_ptr(), 0, s[2].data_ptr(), N, K, st)
    timed("gemv_14336x4096_after_prefill", fn, sets, 60, 5, byt=2.0 * (N * K + K + N))
    del sets
    # Config 4a in BF16
    n = 4096
    sets = [(torch.randn(n, n, device=dev, generator=g).bfloat16(),
             torch.randn(n, n, device=dev, generator=g).bfloat16(),
             torch.empty(n, n, device=dev, dtype=torch.bfloat16)) for _ in range(4)]
    fn = lambda s, st: pkg.cuda.matmul_bf16(  # noqa: E731
        s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), n, n, n, st)
    timed("matmul_bf16_4096", fn, sets, 20, 3, flops=2.0 * n ** 3)
    del sets
    # The reference's own headline size for the FP32 register-tiled matmul, 4096^3
    # (2 rotating sets of 192 MiB > L2)
    n = 4096
    sets = [(torch.rand(n, n, device=dev, generator=g) * 2 - 1,
             torch.rand(n, n, device=dev, generator=g) * 2 - 1,
             torch.empty(n, n, device=dev)) for _ in range(2)]
    fn = lambda s, st: pkg.cuda.matmul_register_tiled(  # noqa: E731
        s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), n, n, n, st)
    timed("matmul_f32_4096", fn, sets, 4, 3, flops=2.0 * n ** 3)
    del sets
    torch.cuda.empty_cache()
    return with_fractions(out)


def old_kernel_baseline(torch, pkg, dev, g):
    """The reference's own sm_89-design CUDA kernels, compiled unmodified for
    sm_100a (oracle/_ref/libref_cuda.so), timed beside this library's drop-in on
    the same GPU, inputs and timing (CUDA graph, operand pools larger than L2):
    config 1 (FP32 matmul_register_tiled 512^3, and the reference's own 4096^3
    headline size), the legacy [K,N] gemv_fp16 at 4096x4096 and 4096x14336, and
    the FP32 rmsnorm_linear dispatcher at one row.  A baseline leg only: nothing
    of it is in the product path.  None when the library was not built."""
    orc = _oracle()
    if not orc.ref_cuda_available():
        return None
    ref = orc.ref_cuda_lib()
    out = {}

    def pair(name, ours, theirs, sets, steps, flops=None, byt=None, graph=True):
        if graph:
            ms_o = time_graph(torch, ours, sets, steps, 3, min_ms=20.0)
            ms_r = time_graph(torch, theirs, sets, steps, 3, min_ms=20.0)
        else:  # back-to-back eager launches on one stream (the reference's pool
            # allocator queries events, which a stream capture forbids)
            st = torch.cuda.current_stream()
            ms_o = time_launches(torch, lambda x: ours(x, st.cuda_stream), sets, steps, 3, st)[1] / steps
            ms_r = time_launches(torch, lambda x: theirs(x, st.cuda_stream), sets, steps, 3, st)[1] / steps
        d = {"ours_us": ms_o * 1e3, "ref_us": ms_r * 1e3, "speedup": ms_r / ms_o,
             "timing": "cuda graph" if graph else "eager launches"}
        if flops:
            d["ours_tflops"] = flops / (ms_o * 1e-3) / 1e12
            d["ref_tflops"] = flops / (ms_r * 1e-3) / 1e12
        if byt:
            d["ours_gbs"] = byt / (ms_o * 1e-3) / 1e9
            d["ref_gbs"] = byt / (ms_r * 1e-3) / 1e9
        out[name] = d

    def chk(rc):
        if rc != 0:
            raise RuntimeError("reference CUDA launcher failed")

    for n, nsets, steps in ((512, 48, 96), (4096, 2, 4)):
        sets = [(torch.rand(n, n, device=dev, generator=g) * 2 - 1,
                 torch.rand(n, n, device=dev, generator=g) * 2 - 1,
                 torch.empty(n, n, device=dev)) for _ in range(nsets)]
        pair(f"matmul_register_tiled_f32_{n}",
             lambda s, st, n=n: pkg.cuda.matmul_register_tiled(
                 s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), n, n, n, st),
             lambda s, st, n=n: chk(ref.refcuda_matmul_register_tiled(
                 s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), n, n, n, st)),
             sets, steps, flops=2.0 * n ** 3)
        del sets
    for (N, K, nsets) in ((4096, 4096, 6), (4096, 14336, 4)):  # legacy A[K,N]
        sets = [((torch.randn(K, N, device=dev, generator=g) * 0.02).half(),
                 torch.randn(K, device=dev, generator=g).half(),
                 torch.empty(N, device=dev, dtype=torch.float16)) for _ in range(nsets)]
        pair(f"gemv_fp16_kn_{K}x{N}",
             lambda s, st, N=N, K=K: pkg.cuda.gemv_fp16(
                 s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), N, K, st),
             lambda s, st, N=N, K=K: chk(ref.refcuda_gemv_fp16(
                 s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), N, K, st)),
             sets, 40, byt=2.0 * (N * K + K + N))
        del sets
    N = K = 4096  # FP32 rmsnorm_linear, one row (the reference dispatches rmsnorm + gemv)
    sets = [(torch.randn(1, K, device=dev, generator=g), 1 + 0.1 * torch.randn(K, device=dev, generator=g),
             torch.randn(K, N, device=dev, generator=g) * 0.02,
             torch.empty(1, N, device=dev)) for _ in range(3)]
    pair("rmsnorm_linear_f32_1x4096x4096",
         lambda s, st: pkg.cuda.rmsnorm_linear(s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(),
                                               s[3].data_ptr(), 1, N, K, 1e-5, st),
         lambda s, st: chk(ref.refcuda_rmsnorm_linear(s[0].data_ptr(), s[1].data_ptr(),
                                                      s[2].data_ptr(), s[3].data_ptr(), 1, N, K,
                                                      1e-5, st)),
         sets, 40, byt=4.0 * (N * K + 2 * K + N), graph=False)
    del sets
    torch.cuda.empty_cache()
    out["note"] = ("the reference's kernels/*.cu compiled unmodified for sm_100a; same inputs "
                   "and timing for both; speedup = ref_us / ours_us")
    return out


def _sig(x, n: int = 4):
    """x rounded to n significant digits (floats only)."""
    if isinstance(x, bool) or not isinstance(x, float) or x == 0.0 or x != x:
        return x
    return float(f"{x:.{n}g}")


def compact(d):
    """A nested result with every float rounded to 4 significant digits, so the
    JSON line stays short enough for a log tail to hold its last blocks."""
    if d is None:
        return None
    if isinstance(d, dict):
        return {k: compact(v) for k, v in d.items()}
    if isinstance(d, (list, tuple)):
        return [compact(v) for v in d]
    return _sig(d)


# FP32 SIMT peak for the CUDA-core GEMMs: 148 SMs x 128 FMA/clk x 2 FLOP x 1.965 GHz
# (nominal; the measured peaks cover only copy bandwidth and bf16 tensor GEMM).
FP32_SIMT_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12


def with_fractions(out: dict) -> dict:
    """Adds each line's roofline fraction: HBM lines against the measured copy
    bandwidth, tensor lines against the measured bf16 dense burst peak, FP32
    CUDA-core lines against the nominal FP32 SIMT peak."""
    pk, kind = peaks()
    for name, d in out.items():
        if "gbs" in d:
            d["frac"] = d["gbs"] / pk["hbm_gbs"]
        elif name.startswith("matmul_f32"):
            d["frac"] = d["tflops"] / FP32_SIMT_TFLOPS
        elif "tflops" in d:
            d["frac"] = d["tflops"] / pk["bf16_tflops"]
    out["peaks"] = {"gbs": f"{kind} HBM copy {pk['hbm_gbs']}",
                    "tflops": f"{kind} bf16 dense burst {pk['bf16_tflops']}",
                    "matmul_f32": f"nominal FP32 SIMT {FP32_SIMT_TFLOPS:.1f}"}
    return out


def e2e_pipelined(torch, pkg, dev, n: int, steps: int, warmup: int, world: int):
    """The headline GEMM end to end through the C ABI with pinned HOST buffers:
    every step copies its A and B host->device, runs engine_cuda_matmul_f16 and
    reads C back.  Steps are pipelined over three streams and two device buffer
    sets -- the H2D copies of step i+1 and the D2H copy of step i-1 run on the two
    copy engines while step i computes -- with events ordering each buffer's
    reuse.  Returns (ms for `steps` steps, max over ranks, H2D and D2H bytes per
    step)."""
    g = torch.Generator().manual_seed(1)
    hA = torch.randn(n, n, generator=g).half().pin_memory()
    hB = torch.randn(n, n, generator=g).half().pin_memory()
    hC = [torch.empty(n, n, dtype=torch.float16).pin_memory() for _ in range(2)]
    dA = [torch.empty(n, n, device=dev, dtype=torch.float16) for _ in range(2)]
    dB = [torch.empty_like(dA[0]) for _ in range(2)]
    dC = [torch.empty_like(dA[0]) for _ in range(2)]
    comp = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev = lambda: torch.cuda.Event()  # noqa: E731

    def run(k: int):
        loaded = [None, None]      # H2D of the step that last used buffer set j finished
        computed = [None, None]    # its GEMM finished (A, B free again)
        read = [None, None]        # its D2H finished (C free again)
        for i in range(k):
            j = i & 1
            with torch.cuda.stream(h2d):
                if computed[j] is not None:
                    h2d.wait_event(computed[j])
                dA[j].copy_(hA, non_blocking=True)
                dB[j].copy_(hB, non_blocking=True)
                loaded[j] = ev()
                loaded[j].record(h2d)
            comp.wait_event(loaded[j])
            if read[j] is not None:
                comp.wait_event(read[j])
            pkg.cuda.matmul_f16(dA[j].data_ptr(), dB[j].data_ptr(), dC[j].data_ptr(), n, n, n,
                                comp.cuda_stream)
            computed[j] = ev()
            computed[j].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(computed[j])
                hC[j].copy_(dC[j], non_blocking=True)
                read[j] = ev()
                read[j].record(d2h)
        for r in read:
            if r is not None:
                comp.wait_event(r)

    run(warmup)
    torch.cuda.synchronize()
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    run(steps)
    e1.record(comp)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    return ms, 2 * n * n * 2, n * n * 2


def sustained_gemm(torch, gemm, sets, seconds: float, stream, local: int):
    """Back-to-back launches for about `seconds` of device time (under the
    power cap); returns (ms per launch, launches, clock summary)."""
    per, _ = time_launches(torch, gemm, sets, 20, 3, stream)
    count = max(50, int(seconds * 1e3 / max(statistics.mean(per), 1e-3)))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local, period_s=0.01) as clk:
        e0.record(stream)
        for i in range(count):
            gemm(sets[i % len(sets)])
        e1.record(stream)
        torch.cuda.synchronize()
    return e0.elapsed_time(e1) / count, count, clk.summary()


def run_headline(args):
    import torch

    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    pkg = load_pkg()
    pk, pk_kind = peaks()
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    n = 4096
    g = torch.Generator(device=dev).manual_seed(20260826 + rank)

    # ---- GEMM 4096^3 on a rotating pool (4 x 96 MiB > 126 MB L2)
    nsets = 4
    sets = []
    for _ in range(nsets):
        A = torch.randn(n, n, device=dev, generator=g).half()
        B = torch.randn(n, n, device=dev, generator=g).half()
        C = torch.empty(n, n, device=dev, dtype=torch.float16)
        sets.append((A, B, C))
    gemm = lambda s: pkg.cuda.matmul_f16(s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(),  # noqa: E731
                                         n, n, n, sp)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local, period_s=0.001) as clk:
        _, total_ms = time_launches(torch, gemm, sets, args.steps, args.warmup, stream,
                                    per_launch=False)
    barrier(world)
    flops = 2.0 * n * n * n
    total_ms_max = max_over_ranks(total_ms, world)
    value = world * flops * args.steps / (total_ms_max * 1e-3) / 1e12

    # ---- roofline: a dedicated loop of >= 400 launches (per-launch CUDA events,
    # clocks sampled), independent of --steps; then the same GEMM as one CUDA
    # graph of back-to-back launches beside cuBLAS (torch.mm, not the product
    # path) on the same operands, and ~1.5 s of launches under the power cap.
    rsteps = max(400, args.steps)
    with ClockSampler(local, period_s=0.002) as rclk:
        _, rtotal = time_launches(torch, gemm, sets, rsteps, 3, stream, per_launch=False)
    gemm_kernel_ms = rtotal / rsteps  # average launch duration, back to back
    achieved = flops / (gemm_kernel_ms * 1e-3) / 1e12
    # The same launches one at a time, each between its own two events (no
    # overlap with its neighbours): mean, median and IQR of a lone launch.
    rper, _ = time_launches(torch, gemm, sets, rsteps, 3, stream)
    peak_t = pk["bf16_tflops"]
    ours_graph = time_graph(torch, lambda s, st: pkg.cuda.matmul_f16(  # noqa: E731
        s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), n, n, n, st), sets, 40, 3, reps=7)
    cublas_graph = time_graph(torch, lambda s, st: torch.mm(s[0], s[1], out=s[2]),  # noqa: E731
                              sets, 40, 3, reps=7)

    # ---- decode GEMV y = W[4096,14336] x over 4 rotating weight matrices (448 MiB)
    Nv, Kv = 4096, 14336
    wsets = []
    for _ in range(4):
        W = (torch.randn(Nv, Kv, device=dev, generator=g) * 0.02).half()
        x = torch.randn(Kv, device=dev, generator=g).half()
        y = torch.empty(Nv, device=dev, dtype=torch.float16)
        wsets.append((W, x, y))
    gemv = lambda s, st: pkg.cuda.gemv_f16_nk(s[0].data_ptr(), s[1].data_ptr(), 0,  # noqa: E731
                                              s[2].data_ptr(), Nv, Kv, st)
    gsteps = max(args.steps, 50)
    barrier(world)
    with ClockSampler(local, period_s=0.001) as gclk:
        gst = time_graph(torch, gemv, wsets, gsteps, max(args.warmup, 3), reps=7, stats=True,
                         min_ms=40.0)
    gemv_kernel_ms = max_over_ranks(gst["median"], world)
    gbytes = 2.0 * (Nv * Kv + Kv + Nv)
    gemv_gbs = gbytes / (gemv_kernel_ms * 1e-3) / 1e9
    gemv_job = world * gemv_gbs
    del wsets
    torch.cuda.empty_cache()

    secondary = (secondary_configs(torch, pkg, dev, g, world, args, local)
                 if not args.skip_secondary else None)

    # ---- the headline GEMM for 1.5 s at the power cap (the sustained roofline
    # denominator).  Last of the timed device work above: the SM clock stays
    # lowered for a while after it, which would slow the HBM-bound lines.
    sus_ms, sus_count, sus_clk = sustained_gemm(torch, gemm, sets, 1.5, stream, local)
    sus_tf = flops / (sus_ms * 1e-3) / 1e12
    del sets
    torch.cuda.empty_cache()

    # ---- e2e through the C ABI with pinned host buffers (copies pipelined)
    esteps = max(3, min(args.steps, 50))
    e2e_ms, h2d_b, d2h_b = e2e_pipelined(torch, pkg, dev, n, esteps, max(args.warmup, 3), world)
    e2e_value = world * flops * esteps / (e2e_ms * 1e-3) / 1e12
    torch.cuda.empty_cache()

    # ---- the reference's own CUDA kernels on this GPU (baseline leg, rank 0 of N=1)
    old = None
    if world == 1 and not args.skip_secondary:
        old = old_kernel_baseline(torch, pkg, dev, g)

    # ---- tensor-parallel layer set at t = world (every rank)
    tpb = None
    if not args.skip_tp:
        from bmle_b200 import tp as _tp

        tpb = _tp.bench_tp_block(args.steps, min(args.warmup, 3), pk["hbm_gbs"],
                                 pk["bf16_tflops_sustained"],
                                 f"{pk_kind} HBM copy (decode) / {pk_kind} bf16 sustained (prefill)")

    # ---- CPU baseline (rank 0, N=1 only)
    cpu = None
    if world == 1 and not args.skip_cpu:
        orc = _oracle()
        nth = orc.ncores()
        v, kind, rows, t = cpu_gemm_throughput(args.cpu_seconds, nth)
        cpu = {"value": v, "unit": "TFLOP/s", "cores": nth, "kind": kind,
               "sample": f"{rows} of 4096 output rows of the 4096^3 GEMM "
                         f"({'engine::cpu::matmul' if kind == 'reference' else 'oracle port'}, "
                         f"FP16 inputs widened to float), {t:.1f} s",
               "single_thread": cpu_single_thread(args.cpu_seconds)}

    traffic = traffic_for("gemm_tc_4096")
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic: seeded N(0,1) FP16 operands (torch Philox), W ~ N(0,0.02)",
        "config": headline_config(world),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_t, "unit": "TFLOP/s",
                     "frac": achieved / peak_t, "traffic": traffic,
                     "peak_kind": f"{pk_kind} bf16 dense burst",
                     "kernel": "gemm_tc2_kernel<256> 4096^3 (2-SM tcgen05, 256x256 tiles, stream-K tail)",
                     "kernel_ms": gemm_kernel_ms, "launches": rsteps,
                     "timing": "CUDA events around the launches, issued back to back; "
                               "kernel_ms = elapsed / launches",
                     "isolated_launch_ms": {
                         "mean": statistics.mean(rper), "median": statistics.median(rper),
                         "iqr": (lambda q: [q[0], q[2]])(statistics.quantiles(rper, n=4)),
                         "timing": "an event pair around each launch (serialises it)"},
                     "clocks": rclk.summary(),
                     "graph_kernel_ms": ours_graph,
                     "cublas_ref_graph_ms": cublas_graph,
                     "sustained": {"kernel_ms": sus_ms, "launches": sus_count,
                                   "achieved": sus_tf, "peak": pk["bf16_tflops_sustained"],
                                   "frac": sus_tf / pk["bf16_tflops_sustained"],
                                   "peak_kind": f"{pk_kind} bf16 dense sustained",
                                   "clocks": sus_clk}},
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d_b,
                "d2h_bytes_per_step": d2h_b,
                "pipeline": "H2D of step i+1 and D2H of step i-1 overlap step i's GEMM "
                            "(three streams, two buffer sets)"},
        "cpu_baseline": cpu,
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
        "environment": environment(with_gpu=True),
        "other_configs": compact(secondary),
        "old_kernel_baseline": compact(old),
        "tp": compact(tpb),
        "gemv": {"value": gemv_gbs, "unit": "GB/s", "frac": gemv_gbs / pk["hbm_gbs"],
                 "peak": pk["hbm_gbs"], "peak_kind": f"{pk_kind} HBM copy",
                 "kernel_us": gemv_kernel_ms * 1e3, "job_gbs": gemv_job,
                 "kernel_us_iqr": [gst["q1"] * 1e3, gst["q3"] * 1e3],
                 "bytes_per_launch": gbytes, "traffic": traffic_for("gemv_nk_4096x14336"),
                 "mhz": gclk.median(),
                 "timing": "CUDA graph of back-to-back launches, 4 x 112 MiB rotating weights"},
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return 0


KERNEL_CASES = ("gemm4096", "gemv_4096x14336", "rmsnorm_qkv_b1", "rmsnorm_qkv_b16",
                "matmul_f32_512", "matmul_f32_4096", "prefill_s2048", "gate_up_swiglu_b1",
                "tp_down_b1_world1", "tp_allreduce_b32_world1", "gemv_q8_0_4096x14336",
                "gemv_q4_0_4096x14336", "gemv_fp16_kn_4096", "attn_prefill_s2048",
                "attn_decode_4096", "attn_decode_1000", "kv_cache_write_b32")


def run_kernel_case(args) -> int:
    """--workload kernel --case NAME: one BASELINE configuration alone, `warmup`
    then `steps` launches on the current stream (no graphs), for profiling a
    single kernel with few launches before it.  Prints the mean per-launch time."""
    import torch

    pkg = load_pkg()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(20260826)
    st = torch.cuda.current_stream().cuda_stream
    c = args.case
    if c == "gemm4096":
        n = 4096
        sets = [tuple(torch.randn(n, n, device=dev, generator=g).half() for _ in range(2)) +
                (torch.empty(n, n, device=dev, dtype=torch.float16),) for _ in range(2)]
        fn = lambda s: pkg.cuda.matmul_f16(s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), n, n, n, st)  # noqa: E731
    elif c == "gemv_4096x14336":
        N, K = 4096, 14336
        sets = [((torch.randn(N, K, device=dev, generator=g) * 0.02).half(),
                 torch.randn(K, device=dev, generator=g).half(),
                 torch.empty(N, device=dev, dtype=torch.float16)) for _ in range(2)]
        fn = lambda s: pkg.cuda.gemv_f16_nk(s[0].data_ptr(), s[1].data_ptr(), 0, s[2].data_ptr(), N, K, st)  # noqa: E731
    elif c in ("rmsnorm_qkv_b1", "rmsnorm_qkv_b16"):
        N, K = 6144, 4096
        B = 1 if c.endswith("b1") else 16
        sets = [(torch.randn(B, K, device=dev, generator=g).half(),
                 (1 + 0.1 * torch.randn(K, device=dev, generator=g)).half(),
                 (torch.randn(N, K, device=dev, generator=g) * 0.02).half(),
                 torch.empty(B, N, device=dev, dtype=torch.float16)) for _ in range(3)]
        fn = lambda s: pkg.cuda.rmsnorm_linear_f16(s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), 0,  # noqa: E731
                                                   s[3].data_ptr(), B, N, K, 1e-5, st)
    elif c == "matmul_f32_512":
        n = 512
        sets = [(torch.rand(n, n, device=dev, generator=g) * 2 - 1,
                 torch.rand(n, n, device=dev, generator=g) * 2 - 1,
                 torch.empty(n, n, device=dev)) for _ in range(48)]
        fn = lambda s: pkg.cuda.matmul_register_tiled(s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), n, n, n, st)  # noqa: E731
    elif c == "gate_up_swiglu_b1":  # Llama-3-8B gate/up (2 x 14336 rows) + SwiGLU, batch 1
        F, K = 14336, 4096
        sets = [(torch.randn(1, K, device=dev, generator=g).half(),
                 (1 + 0.1 * torch.randn(K, device=dev, generator=g)).half(),
                 (torch.randn(2 * F, K, device=dev, generator=g) * 0.02).half(),
                 torch.empty(1, F, device=dev, dtype=torch.float16)) for _ in range(2)]
        fn = lambda s: pkg.cuda.rmsnorm_linear_swiglu_f16(s[0].data_ptr(), s[1].data_ptr(),  # noqa: E731
                                                          s[2].data_ptr(), s[3].data_ptr(), 1, F, K,
                                                          1e-5, st)
    elif c == "tp_down_b1_world1":  # the fused row-split down projection + all-reduce, one rank
        N, K = 4096, 14336
        comm = pkg.tp.NvlinkComm(0, 1, N)
        sets = [(torch.randn(1, K, device=dev, generator=g).half(),
                 (torch.randn(N, K, device=dev, generator=g) * 0.02).half(),
                 torch.randn(1, N, device=dev, generator=g).half(),
                 torch.empty(1, N, device=dev, dtype=torch.float16)) for _ in range(4)]
        fn = lambda s: pkg.cuda.tp_linear_allreduce_f16(comm.handle, s[0].data_ptr(), s[1].data_ptr(),  # noqa: E731
                                                        s[2].data_ptr(), s[3].data_ptr(), 1, N, K, st)
    elif c == "matmul_f32_4096":  # the reference's FP32 headline size
        n = 4096
        sets = [(torch.rand(n, n, device=dev, generator=g) * 2 - 1,
                 torch.rand(n, n, device=dev, generator=g) * 2 - 1,
                 torch.empty(n, n, device=dev)) for _ in range(2)]
        fn = lambda s: pkg.cuda.matmul_register_tiled(s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), n, n, n, st)  # noqa: E731
    elif c == "tp_allreduce_b32_world1":  # the communicator's all-reduce, 32 x 4096, one rank
        comm = pkg.tp.NvlinkComm(0, 1, 32 * 4096)
        sets = [(torch.randn(32 * 4096, device=dev, generator=g).half(),
                 torch.empty(32 * 4096, device=dev, dtype=torch.float16)) for _ in range(2)]
        fn = lambda s: pkg.cuda.tp_allreduce_f16(comm.handle, s[0].data_ptr(), 0, s[1].data_ptr(),  # noqa: E731
                                                 32 * 4096, st)
    elif c == "gemv_fp16_kn_4096":  # the legacy gemv_fp16, A[K, N] 4096 x 4096
        N = K = 4096
        sets = [((torch.randn(K, N, device=dev, generator=g) * 0.02).half(),
                 torch.randn(K, device=dev, generator=g).half(),
                 torch.empty(N, device=dev, dtype=torch.float16)) for _ in range(6)]
        fn = lambda s: pkg.cuda.gemv_fp16(s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), N, K, st)  # noqa: E731
    elif c == "attn_prefill_s2048":  # Llama-3-8B heads, causal, S = 2048 (tcgen05)
        S, H, Hk, d = 2048, 32, 8, 128
        sets = [(torch.randn(S, H, d, device=dev, generator=g).half(),
                 torch.randn(Hk, S, d, device=dev, generator=g).half(),
                 torch.randn(Hk, S, d, device=dev, generator=g).half(),
                 torch.empty(S, H, d, device=dev, dtype=torch.float16)) for _ in range(2)]
        fn = lambda s: pkg.cuda.attention_prefill(s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(),  # noqa: E731
                                                  s[3].data_ptr(), S, S, H, Hk, d, S * d, d ** -0.5,
                                                  0, True, 0, st)
    elif c == "attn_decode_1000":  # 1000 keys: the splits merge inside a thread-block cluster
        kv, H, Hk, d = 1000, 32, 8, 128
        sets = [(torch.randn(H, d, device=dev, generator=g).half(),
                 torch.randn(Hk, kv, d, device=dev, generator=g).half(),
                 torch.randn(Hk, kv, d, device=dev, generator=g).half(),
                 torch.empty(H, d, device=dev, dtype=torch.float16)) for _ in range(16)]
        fn = lambda s: pkg.cuda.attention_decode(s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(),  # noqa: E731
                                                 s[3].data_ptr(), kv, H, Hk, d, kv * d, d ** -0.5, 0,
                                                 st)
    elif c == "kv_cache_write_b32":  # decode of 32 sequences: K / V of a Q/K/V output into the caches
        B, Hk, d, L, qkv_cols = 32, 8, 128, 1024, 6144
        sets = [(torch.randn(B, qkv_cols, device=dev, generator=g).half(),
                 torch.zeros(B * Hk, L, d, device=dev, dtype=torch.float16),
                 torch.zeros(B * Hk, L, d, device=dev, dtype=torch.float16)) for _ in range(2)]
        fn = lambda s: pkg.cuda.kv_cache_write_rows(  # noqa: E731
            s[0].data_ptr() + 2 * 4096, s[0].data_ptr() + 2 * 5120, qkv_cols, s[1].data_ptr(),
            s[2].data_ptr(), B, 1, Hk, d, L - 1, L, st)
    elif c == "attn_decode_4096":  # one token over 4096 keys, Llama-3-8B heads
        kv, H, Hk, d = 4096, 32, 8, 128
        sets = [(torch.randn(H, d, device=dev, generator=g).half(),
                 torch.randn(Hk, kv, d, device=dev, generator=g).half(),
                 torch.randn(Hk, kv, d, device=dev, generator=g).half(),
                 torch.empty(H, d, device=dev, dtype=torch.float16)) for _ in range(8)]
        fn = lambda s: pkg.cuda.attention_decode(s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(),  # noqa: E731
                                                 s[3].data_ptr(), kv, H, Hk, d, kv * d, d ** -0.5, 0,
                                                 st)
    elif c.startswith("gemv_q"):  # block-quantised decode GEMV, streamed layout (timing only)
        N, K = 4096, 14336
        qt = 8 if c.startswith("gemv_q8") else 4
        pay = K if qt == 8 else K // 2
        sets = [(torch.randint(0, 256, (N, pay), device=dev, generator=g, dtype=torch.uint8),
                 (torch.rand(N, K // 32, device=dev, generator=g) * 1e-3).half(),
                 torch.randn(K, device=dev, generator=g).half(),
                 torch.empty(N, device=dev, dtype=torch.float16)) for _ in range(2)]
        fn = lambda s: pkg.cuda.gemv_q_nk(qt, s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), 0,  # noqa: E731
                                          s[3].data_ptr(), N, K, st)
    else:  # prefill_s2048
        S, N, K = 2048, 14336, 4096
        sets = [(torch.randn(S, K, device=dev, generator=g).half(),
                 (torch.randn(N, K, device=dev, generator=g) * 0.02).half(),
                 torch.empty(S, N, device=dev, dtype=torch.float16)) for _ in range(2)]
        fn = lambda s: pkg.cuda.linear_f16(s[0].data_ptr(), s[1].data_ptr(), 0, s[2].data_ptr(), S, N, K, st)  # noqa: E731
    stream = torch.cuda.current_stream()
    per, total = time_launches(torch, fn, sets, args.steps, args.warmup, stream)
    print(json.dumps({"workload": "kernel", "case": c, "steps": args.steps, "warmup": args.warmup,
                      "us_per_launch": 1e3 * statistics.mean(per),
                      "timing": "CUDA events per launch, rotating operand sets"}), flush=True)
    return 0


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["headline", "tp-decode", "tp-prefill", "tp-comm", "kernel"],
                    default="headline")
    ap.add_argument("--case", choices=KERNEL_CASES, default="gemm4096",
                    help="--workload kernel: the configuration to run alone")
    ap.add_argument("--batch", type=int, default=1, help="tp-decode batch (1 or 32)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-secondary", action="store_true")
    ap.add_argument("--skip-tp", action="store_true",
                    help="leave out the tensor-parallel layer-set block of the headline line")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "kernel":
        return run_kernel_case(args)
    if args.workload != "headline":
        tp = importlib.import_module("bmle_b200.tp") if "bmle_b200" in sys.modules else None
        load_pkg()
        from bmle_b200 import tp  # noqa: F811

        if args.workload == "tp-comm":
            return tp.bench_collectives(args)
        return tp.bench_main(args, METRIC)
    return run_headline(args)


if __name__ == "__main__":
    sys.exit(main())
