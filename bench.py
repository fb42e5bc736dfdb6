"""Benchmark of the B200 BF16 GEMM — BASELINE metric: BF16 GEMM TFLOPS at
M=N=K=4096 and its fraction of the B200 dense BF16 peak; 1/2/4/8-GPU scaling.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step = one GEMM C = A @ B (A [4096,4096], B [4096,4096] row-major = the
BASELINE config, U(-1,1) bf16) on each GPU.  With N GPUs (torchrun, one rank
per GPU) A is [4096*N, 4096], one 4096-row panel per rank; every step rank 0
broadcasts B to all ranks over NCCL and each rank multiplies its panel, C
stays sharded: per-GPU work is fixed as N grows ("weak" scaling) and the
broadcast is inside every step.

Timing: CUDA events on the launching stream, W warm-up steps, then exactly K
timed steps bracketed by barrier + synchronize, max over ranks.  Inputs
rotate over 4 buffer sets (4 x 96 MiB > 126 MB L2) so no step finds its
operands in L2.  Clocks are sampled through NVML during the timed region.

The line also carries:
  e2e        the step through the public API with host (pinned) buffers:
             host->device copies of the step's inputs, the GEMM and the
             device->host copy of C inside the timed region;
  rowshard   BASELINE config 5 (131072x8192x8192 split over the N ranks, B
             broadcast, C sharded; strong scaling), with the 1-GPU time of
             the same job measured in the same run at N>1;
  parity     (N>1) the sharded result on sampled rows against an fp32 CPU
             product, and the fused all-gather GEMM against GEMM + NCCL
             all-gather, bit for bit on every rank;
  configs    (N=1) BASELINE configs 2-4, ours and cuBLAS in the same loop;
  cpu_baseline  (N=1) the reference arithmetic on the host cores.

`--impl reference` times the reference's arithmetic on the host cores (the
reference has no CPU implementation of its own; this is the oracle port in
oracle/gemm_oracle.c) on a bounded row sample of the same workload, on every
host thread the process may use.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "cuda-kernels_b200"))
sys.path.insert(0, REPO)

METRIC = "bf16_gemm_tflops_4096"
M_PER_RANK = 4096
N_DIM = 4096
K_DIM = 4096
ROTATE = 4
FLOPS_PER_STEP = 2.0 * M_PER_RANK * N_DIM * K_DIM


def _peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"burst": float(d["bf16_tflops"]), "sustained": float(d["bf16_tflops_sustained"]),
                "hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"burst": 1590.0, "sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


def _traffic():
    """Per-launch DRAM bytes of the GEMM kernel from the committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", "gemm_bf16_4096_traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return None


class ClockSampler:
    """Samples SM clock, power and clock-event reasons of one GPU via NVML."""

    def __init__(self, pci_bus_id: str, period_s: float = 0.02):
        self.period = period_s
        self.samples = []
        self._stop = threading.Event()
        self._thr = None
        self.error = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(pci_bus_id.encode() if isinstance(pci_bus_id, str) else pci_bus_id)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # NVML missing: report, do not fail the bench
            self.nv = None
            self.error = repr(e)
            self.max_mhz = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                pw = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                self.samples.append((mhz, reasons, pw))
            except Exception as e:
                self.error = repr(e)
                return
            time.sleep(self.period)

    def start(self):
        if self.nv is not None:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()

    def stop(self):
        if self._thr is not None:
            self._stop.set()
            self._thr.join()

    def summary(self):
        if self.nv is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": len(self.samples),
                    "error": self.error}
        nv = self.nv
        names = {
            "hw_slowdown": nv.nvmlClocksThrottleReasonHwSlowdown,
            "hw_thermal_slowdown": nv.nvmlClocksThrottleReasonHwThermalSlowdown,
            "sw_thermal_slowdown": nv.nvmlClocksThrottleReasonSwThermalSlowdown,
            "sw_power_cap": nv.nvmlClocksThrottleReasonSwPowerCap,
            "hw_power_brake_slowdown": nv.nvmlClocksThrottleReasonHwPowerBrakeSlowdown,
        }
        seen = sorted({n for _, r, _ in self.samples for n, bit in names.items() if r & bit})
        return {"sm_mhz": statistics.median(s[0] for s in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": seen, "samples": len(self.samples),
                "power_w_median": round(statistics.median(s[2] for s in self.samples), 1)}


def _dist_setup():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def host_threads() -> int:
    """Host threads the CPU legs use: every core this process may run on.  Set
    explicitly (not inherited from OMP_NUM_THREADS, which torchrun sets to 1),
    so the CPU figures do not change with the number of GPU ranks."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:  # not Linux
        return os.cpu_count() or 1


def cpu_baseline(target_s: float = 10.0, rows: int = 512):
    """The oracle (CPU restatement of the reference arithmetic) on the host
    cores, on row panels of the same workload, repeated for ~target_s."""
    import numpy as np
    from oracle import oracle as o
    threads = host_threads()
    rng = np.random.default_rng(0)
    a = o.f32_to_bf16(rng.uniform(-1, 1, (rows, K_DIM)).astype(np.float32))
    b = o.f32_to_bf16(rng.uniform(-1, 1, (K_DIM, N_DIM)).astype(np.float32))
    o.gemm_f32acc(a[:8], b, 1, threads)  # warm
    t0 = time.perf_counter()
    n = 0
    while True:
        o.gemm_bf16(a, b, 1, threads)
        n += 1
        if time.perf_counter() - t0 >= target_s:
            break
    dt = time.perf_counter() - t0
    tflops = 2.0 * rows * N_DIM * K_DIM * n / dt / 1e12
    return {"value": round(tflops, 5), "unit": "TFLOPS", "cores": threads, "kind": "port",
            "sample": f"{n} x A[{rows},{K_DIM}] @ B[{K_DIM},{N_DIM}] row panels of the 4096^3 GEMM "
                      f"(oracle/gemm_oracle.c, fp32 accumulate, {threads} threads, {dt:.1f} s)"}


def attention_cpu_baseline(target_s: float = 3.0, seq: int = 2048):
    """The attention oracle (exact fp64 attention in numpy, oracle/oracle.py) on the
    host cores: one head of the causal benchmark shape, repeated for ~target_s."""
    import numpy as np
    from oracle import oracle as o
    rng = np.random.default_rng(2)
    q, k, v = (o.f32_to_bf16(rng.standard_normal((1, seq, 1, 128)).astype(np.float32)) for _ in range(3))
    try:
        from threadpoolctl import threadpool_info
        cores = max([int(i.get("num_threads", 1)) for i in threadpool_info()] or [1])
    except Exception:  # noqa: BLE001 - the thread count is informational
        cores = os.cpu_count() or 1
    t0 = time.perf_counter()
    n = 0
    while True:
        o.attention(q, k, v, True)
        n += 1
        if time.perf_counter() - t0 >= target_s:
            break
    dt = time.perf_counter() - t0
    tflops = 2.0 * 2.0 * seq * seq * 128 / 2.0 * n / dt / 1e12
    return {"value": round(tflops, 5), "unit": "TFLOPS", "cores": cores, "kind": "port",
            "sample": f"{n} x causal attention batch 1, seq {seq}, 1 head, head_dim 128 "
                      f"(oracle.attention, fp64 numpy, {dt:.1f} s)"}


def run_reference(args, world, rank):
    """--impl reference: the reference arithmetic on the host cores (oracle port),
    on every host thread this process may use, whatever the number of ranks."""
    if rank != 0:
        return 0
    import numpy as np
    from oracle import oracle as o
    threads = host_threads()
    rows = args.ref_rows
    rng = np.random.default_rng(1)
    a = o.f32_to_bf16(rng.uniform(-1, 1, (rows, K_DIM)).astype(np.float32))
    b = o.f32_to_bf16(rng.uniform(-1, 1, (K_DIM, N_DIM)).astype(np.float32))
    for _ in range(args.warmup):
        o.gemm_bf16(a, b, 1, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        o.gemm_bf16(a, b, 1, threads)
    dt = time.perf_counter() - t0
    tflops = 2.0 * rows * N_DIM * K_DIM * args.steps / dt / 1e12
    sample = (f"each step: A[{rows},{K_DIM}] row panel of the 4096^3 GEMM @ B[{K_DIM},{N_DIM}] "
              f"on {threads} host threads (the reference has no CPU path; oracle port)")
    line = {"metric": METRIC, "value": round(tflops, 5), "unit": "TFLOPS",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt * 1e3 / args.steps, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": _config(args.layout, world),
            "impl": "reference",
            "cpu_baseline": {"value": round(tflops, 5), "unit": "TFLOPS", "cores": threads,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(tflops, 5), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def sweep_configs():
    """Single-GPU BASELINE configs 1-4 (config 5 is the multi-GPU row-sharded job)."""
    out = []
    for n in (1024, 2048, 4096, 8192, 16384):
        out.append(("square", n, n, n, "uniform"))
    for m in (16, 64, 128):
        for (n, k) in ((4096, 4096), (14336, 4096), (4096, 14336)):
            out.append(("skinny", m, n, k, "normal"))
    for m in (8192, 8191, 5000):
        for (n, k) in ((4096, 4096), (6144, 4096), (28672, 4096), (4096, 14336), (128256, 4096)):
            out.append(("projection", m, n, k, "normal"))
    return out


def time_config(M, N, K, layout, dist_kind, b200_gemm, target_ms=250.0, warmup=10, with_cublas=True, use_graph=True,
                with_split=True):
    """Device-time one GEMM shape back to back over rotating buffer sets larger than L2."""
    import math
    import torch
    dev = torch.device("cuda", torch.cuda.current_device())
    set_bytes = 2 * (M * K + K * N + M * N)
    R = max(2, math.ceil(400e6 / set_bytes))
    g = torch.Generator(device=dev).manual_seed(M * 31 + N * 7 + K)

    def gen(shape, std=1.0):
        if dist_kind == "uniform":
            return (torch.rand(shape, generator=g, device=dev) * 2 - 1).to(torch.bfloat16)
        return (torch.randn(shape, generator=g, device=dev) * std).to(torch.bfloat16)

    b_shape = (K, N) if layout == "kn" else (N, K)
    A = [gen((M, K)) for _ in range(R)]
    B = [gen(b_shape, 1.0 if dist_kind == "uniform" else K ** -0.5) for _ in range(R)]
    C = [torch.empty((M, N), dtype=torch.bfloat16, device=dev) for _ in range(R)]

    def ours(i):
        b200_gemm.gemm(A[i % R], B[i % R], b_layout=layout, out=C[i % R])

    def ours_splitk(i):
        b200_gemm.gemm(A[i % R], B[i % R], b_layout=layout, out=C[i % R], split_k=True)

    def cublas(i):
        torch.matmul(A[i % R], B[i % R] if layout == "kn" else B[i % R].t(), out=C[i % R])

    res = {}
    variants = [("b200", ours), ("cublas", cublas)]
    if with_split and b200_gemm.ops.workspace_bytes(M, N, K, layout) > 0:
        variants.insert(1, ("b200_split_k", ours_splitk))
    for name, fn in variants:
        if name == "cublas" and not with_cublas:
            continue
        for i in range(warmup):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(3):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        est = max(e0.elapsed_time(e1) / 3, 1e-3)
        if use_graph and est < 1.0:
            # Short GEMMs: replay a captured batch so that host launch cost is
            # not timed (both implementations are measured the same way).
            per = R * max(1, int(2.0 / (est * R)))
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                fn(0)
                torch.cuda.synchronize()
                with torch.cuda.graph(graph, stream=s):
                    for i in range(per):
                        fn(i)
            torch.cuda.synchronize()
            graph.replay()
            torch.cuda.synchronize()
            reps = max(3, int(target_ms / (est * per)))
            e0.record()
            for _ in range(reps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            res[name] = e0.elapsed_time(e1) / (reps * per)
            del graph
            continue
        steps = max(5, int(target_ms / est))
        e0.record()
        for i in range(steps):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        res[name] = e0.elapsed_time(e1) / steps
    b200_gemm.check_status()
    del A, B, C
    torch.cuda.empty_cache()
    return res


def _time_variants(fns, target_ms=250.0, warmup=10, use_graph=True):
    """Device time per call of each fn(i) (i picks the rotating buffer set), back to back;
    graph replay for calls under 1 ms so host launch cost is not timed."""
    import torch
    res = {}
    for name, fn in fns.items():
        for i in range(warmup):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(3):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        est = max(e0.elapsed_time(e1) / 3, 1e-3)
        if use_graph and est < 1.0:
            per = max(8, int(2.0 / est))
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                fn(0)
                torch.cuda.synchronize()
                with torch.cuda.graph(graph, stream=s):
                    for i in range(per):
                        fn(i)
            torch.cuda.synchronize()
            graph.replay()
            torch.cuda.synchronize()
            reps = max(3, int(target_ms / (est * per)))
            e0.record()
            for _ in range(reps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            res[name] = e0.elapsed_time(e1) / (reps * per)
            del graph
            continue
        steps = max(5, int(target_ms / est))
        e0.record()
        for i in range(steps):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        res[name] = e0.elapsed_time(e1) / steps
    return res


def run_epilogue(args) -> int:
    """--epilogue: the fused epilogue (b200_gemm_bf16_ex) against the same result
    computed unfused (plain GEMM, then bias and residual adds as separate
    passes over C), and cuBLAS's own fused bias (torch.addmm) + residual add.
    One JSON line per shape; device time per call, rotating inputs > L2."""
    import math
    import torch
    torch.cuda.set_device(0)
    import b200_gemm
    dev = torch.device("cuda", 0)
    shapes = [(4096, 4096, 4096), (8192, 4096, 4096), (128, 14336, 4096), (16, 4096, 4096)]
    for (M, N, K) in shapes:
        set_bytes = 2 * (M * K + K * N + 2 * M * N)
        R = max(2, math.ceil(400e6 / set_bytes))
        g = torch.Generator(device=dev).manual_seed(M + N + K)
        A = [torch.randn((M, K), generator=g, device=dev).bfloat16() for _ in range(R)]
        B = [(torch.randn((K, N), generator=g, device=dev) * K ** -0.5).bfloat16() for _ in range(R)]
        Res = [torch.randn((M, N), generator=g, device=dev).bfloat16() for _ in range(R)]
        C = [torch.empty((M, N), dtype=torch.bfloat16, device=dev) for _ in range(R)]
        C32 = torch.empty((M, N), dtype=torch.float32, device=dev)
        bias = torch.randn((N,), generator=g, device=dev).bfloat16()
        fns = {
            "plain": lambda i: b200_gemm.gemm(A[i % R], B[i % R], b_layout="kn", out=C[i % R]),
            "fused_bias_residual": lambda i: b200_gemm.gemm(A[i % R], B[i % R], b_layout="kn", out=C[i % R],
                                                            beta=1.0, c=Res[i % R], bias=bias),
            "unfused_bias_residual": lambda i: (b200_gemm.gemm(A[i % R], B[i % R], b_layout="kn", out=C[i % R]),
                                                C[i % R].add_(bias), C[i % R].add_(Res[i % R])),
            "fused_f32_out": lambda i: b200_gemm.gemm(A[i % R], B[i % R], b_layout="kn", out=C32,
                                                      out_dtype=torch.float32),
            "cublas_addmm_bias_plus_residual": lambda i: (torch.addmm(bias, A[i % R], B[i % R], out=C[i % R]),
                                                          C[i % R].add_(Res[i % R])),
        }
        t = _time_variants(fns, target_ms=args.target_ms)
        b200_gemm.check_status()
        flops = 2.0 * M * N * K
        line = {"what": "fused_epilogue", "config": {"M": M, "N": N, "K": K, "b_layout": "kn", "data": "normal"},
                "us": {k: round(v * 1e3, 2) for k, v in t.items()},
                "tflops": {k: round(flops / (v / 1e3) / 1e12, 1) for k, v in t.items()},
                "fused_vs_unfused": round(t["unfused_bias_residual"] / t["fused_bias_residual"], 3),
                "fused_vs_cublas_addmm": round(t["cublas_addmm_bias_plus_residual"] / t["fused_bias_residual"], 3)}
        print(json.dumps(line), flush=True)
        del A, B, Res, C, C32
        torch.cuda.empty_cache()
    return 0


def run_fp32(args) -> int:
    """--fp32: the reference's fp32_matmul operator (M=N=K=4096, A and B fp32 row-major,
    fp32_matmul/README.md:4-8): ours (three-way bf16 split on the tensor cores,
    split kernels included in the time) against cuBLAS fp32 (torch.matmul, TF32 off)."""
    import math
    import torch
    torch.cuda.set_device(0)
    import b200_gemm
    dev = torch.device("cuda", 0)
    for (M, N, K) in [(4096, 4096, 4096), (8192, 8192, 8192), (128, 4096, 4096)]:
        R = max(2, math.ceil(400e6 / (4 * (M * K + K * N + M * N))))
        g = torch.Generator(device=dev).manual_seed(M + N + K)
        A = [torch.randn((M, K), generator=g, device=dev) for _ in range(R)]
        B = [torch.randn((K, N), generator=g, device=dev) for _ in range(R)]
        C = [torch.empty((M, N), device=dev) for _ in range(R)]
        torch.backends.cuda.matmul.allow_tf32 = False
        fns = {"b200_f32": lambda i: b200_gemm.gemm_f32(A[i % R], B[i % R], out=C[i % R]),
               "cublas_f32": lambda i: torch.matmul(A[i % R], B[i % R], out=C[i % R])}
        t = _time_variants(fns, target_ms=args.target_ms)
        b200_gemm.check_status()
        flops = 2.0 * M * N * K
        print(json.dumps({"what": "fp32_gemm", "config": {"M": M, "N": N, "K": K, "b_layout": "kn",
                                                           "data": "normal", "dtype": "f32"},
                          "ms": {k: round(v, 4) for k, v in t.items()},
                          "tflops": {k: round(flops / (v / 1e3) / 1e12, 1) for k, v in t.items()},
                          "vs_cublas": round(t["cublas_f32"] / t["b200_f32"], 3)}), flush=True)
        del A, B, C
        torch.cuda.empty_cache()
    return 0


def run_attention(args) -> int:
    """--attention: the reference's flash_attn benchmark (flash_attn/main.py:28-56,
    README.md:9): causal bf16 attention, (batch, seq, heads, head_dim) = (1, S, 32, 128),
    S = 512 ... 8192, plus the full (non-causal) mask at 4096 and 8192; ours against torch
    SDPA and the flash-attn package on the same GPU.  TFLOPS counted as the reference does:
    2 * 2 * B * H * S^2 * D, halved for the causal mask."""
    import torch
    import torch.nn.functional as F
    torch.cuda.set_device(0)
    import b200_gemm
    dev = torch.device("cuda", 0)
    try:
        from flash_attn import flash_attn_func
    except Exception:  # noqa: BLE001 - the comparison is optional
        flash_attn_func = None
    peaks = _peaks()
    cpu = None if args.no_cpu_baseline else attention_cpu_baseline()
    cases = [(S, True) for S in (512, 1024, 2048, 4096, 8192)] + [(4096, False), (8192, False)]
    for S, causal in cases:
        g = torch.Generator(device=dev).manual_seed(S)
        q, k, v = (torch.randn((1, S, 32, 128), generator=g, device=dev).bfloat16() for _ in range(3))
        qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        out = torch.empty_like(q)
        fns = {"b200": lambda i: b200_gemm.flash_attn(q, k, v, causal=causal, out=out),
               "torch_sdpa": lambda i: F.scaled_dot_product_attention(qt, kt, vt, is_causal=causal)}
        if flash_attn_func is not None:
            fns["flash_attn_pkg"] = lambda i: flash_attn_func(q, k, v, causal=causal)
        t = _time_variants(fns, target_ms=args.target_ms)
        b200_gemm.check_status()
        flops = 2.0 * 2.0 * 32 * S * S * 128 / (2.0 if causal else 1.0)
        tf = {k_: round(flops / (v_ / 1e3) / 1e12, 1) for k_, v_ in t.items()}
        print(json.dumps({"what": "flash_attention_" + ("causal" if causal else "full"),
                          "config": {"batch": 1, "seq_len": S, "heads": 32, "head_dim": 128, "dtype": "bf16"},
                          "ms": {k_: round(v_, 4) for k_, v_ in t.items()}, "tflops": tf,
                          # each size is timed in a ~0.25 s loop: the sustained (power-capped) peak applies
                          "roofline": {"bound": "tensor", "achieved": tf["b200"], "peak": peaks["sustained"],
                                       "unit": "TFLOP/s", "frac": round(tf["b200"] / peaks["sustained"], 3),
                                       "peak_source": peaks["source"]},
                          "cpu_baseline": cpu}),
              flush=True)
    return 0


def run_sweep(args) -> int:
    """--sweep: one JSON line per single-GPU BASELINE config (b200 and cuBLAS, same loop)."""
    import torch
    torch.cuda.set_device(0)
    import b200_gemm
    peaks = _peaks()
    for family, M, N, K, dist_kind in sweep_configs():
        for layout in (("kn", "nk") if (family == "square" and M == 4096) or family == "skinny" else ("kn",)):
            t = time_config(M, N, K, layout, dist_kind, b200_gemm, with_cublas=not args.no_cublas,
                            use_graph=not args.no_graph)
            flops = 2.0 * M * N * K
            nbytes = 2.0 * (M * K + K * N + M * N)
            tf = flops / (t["b200"] / 1e3) / 1e12
            gbs = nbytes / (t["b200"] / 1e3) / 1e9
            hbm_bound = nbytes / (peaks["hbm_gbs"] * 1e9) > flops / (peaks["burst"] * 1e12)
            line = {"config": {"family": family, "M": M, "N": N, "K": K, "b_layout": layout, "data": dist_kind},
                    "ms": round(t["b200"], 5), "tflops": round(tf, 1), "gbs": round(gbs, 1),
                    "bound": "hbm" if hbm_bound else "tensor",
                    "frac": round(gbs / peaks["hbm_gbs"] if hbm_bound else tf / peaks["burst"], 4),
                    "peak_source": peaks["source"], "timing": "graph replay" if (not args.no_graph and t["b200"] < 1.0) else "direct launches"}
            if "b200_split_k" in t:
                line["split_k_tail_ms"] = round(t["b200_split_k"], 5)
                line["split_k_tail_tflops"] = round(flops / (t["b200_split_k"] / 1e3) / 1e12, 1)
            if "cublas" in t:
                line["cublas_ms"] = round(t["cublas"], 5)
                line["speedup_vs_cublas"] = round(t["cublas"] / t["b200"], 3)
            print(json.dumps(line), flush=True)
    return 0


def run_rowshard(args) -> int:
    """--rowshard: BASELINE config 5, M=131072, N=K=8192 split into row panels
    over the ranks (strong scaling).  Each step: B (stored [N,K]) broadcast
    from rank 0 over NCCL, whole or in --chunks column chunks overlapped with
    the GEMM, + the GEMM of every panel; device time, max over ranks.  Also
    reports the GEMM alone and the optional C all-gather, timed separately."""
    import torch
    import torch.distributed as dist
    world, rank, local = _dist_setup()
    import b200_gemm
    from b200_gemm.dist import row_sharded_gemm, shard_rows
    M, N, K = args.rowshard_m, 8192, 8192
    dev = torch.device("cuda", torch.cuda.current_device())
    s, e = shard_rows(M, world, rank)
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    a = (torch.rand((e - s, K), generator=g, device=dev) * 2 - 1).to(torch.bfloat16)
    b = (torch.rand((N, K), generator=g, device=dev) * 2 - 1).to(torch.bfloat16)
    c = torch.empty((e - s, N), dtype=torch.bfloat16, device=dev)

    def step(bcast):
        row_sharded_gemm(a, b, M=M, b_layout="nk", chunks=args.chunks, out=c, broadcast=bcast)

    # Warm up to the power-capped steady state (>= 1.5 s of GEMMs) and time at
    # least ~1 s, so every N is measured in the same clock regime.
    res = {}
    for name, bcast in (("gemm_only", False), ("broadcast_plus_gemm", world > 1)):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step(bcast)
        e1.record()
        torch.cuda.synchronize()
        # All ranks must issue the same number of collectives: agree on the
        # step time (max over ranks) before deriving the step counts from it.
        one = max(_max_over_ranks(e0.elapsed_time(e1), world), 1e-3)
        # (--steps is ignored here: each mode runs for about one second.)
        warm = max(args.warmup, int(1500.0 / one) + 1)
        steps = max(3, int(1000.0 / one) + 1)
        for _ in range(warm):
            step(bcast)
        torch.cuda.synchronize()
        _barrier(world)
        e0.record()
        for _ in range(steps):
            step(bcast)
        e1.record()
        torch.cuda.synchronize()
        _barrier(world)
        res[name] = _max_over_ranks(e0.elapsed_time(e1) / steps, world)
    b200_gemm.check_status()
    # Optional C all-gather (every rank ends with the whole [M, N] C), timed
    # separately as the BASELINE asks; then the whole step with the gather:
    # broadcast + GEMM + NCCL all-gather, against broadcast + the GEMM with the
    # all-gather fused into its epilogue (b200_gemm_bf16_allgather).
    gather_ms = unfused_ms = fused_ms = None
    if world > 1:
        from b200_gemm.dist import GatheredC, gather_rows, row_sharded_gemm_gather
        full = gather_rows(c, M)
        torch.cuda.synchronize()
        _barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        e0.record()
        for _ in range(reps):
            full = gather_rows(c, M)
        e1.record()
        torch.cuda.synchronize()
        _barrier(world)
        gather_ms = _max_over_ranks(e0.elapsed_time(e1) / reps, world)
        del full
        gbuf = GatheredC(M, N)

        def unfused():
            step(True)
            return gather_rows(c, M)

        def fused():
            return row_sharded_gemm_gather(a, b, gathered=gbuf, M=M, b_layout="nk")

        times = {}
        for name, fn in (("unfused", unfused), ("fused", fused)):
            fn()
            torch.cuda.synchronize()
            _barrier(world)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            one = max(_max_over_ranks(e0.elapsed_time(e1), world), 1e-3)
            n_warm, n = int(500.0 / one) + 1, int(1000.0 / one) + 2
            for _ in range(n_warm):
                fn()
            torch.cuda.synchronize()
            _barrier(world)
            e0.record()
            for _ in range(n):
                fn()
            e1.record()
            torch.cuda.synchronize()
            _barrier(world)
            times[name] = _max_over_ranks(e0.elapsed_time(e1) / n, world)
        unfused_ms, fused_ms = times["unfused"], times["fused"]
        b200_gemm.check_status()
        gbuf.close()
    flops = 2.0 * M * N * K
    if rank == 0:
        print(json.dumps({
            "metric": "bf16_gemm_tflops_rowshard_131072x8192x8192", "n_gpus": world, "steps": steps,
            "value": round(flops / (res["broadcast_plus_gemm"] / 1e3) / 1e12, 2), "unit": "TFLOPS",
            "ms_per_step": round(res["broadcast_plus_gemm"], 4), "gemm_only_ms": round(res["gemm_only"], 4),
            "gemm_only_tflops": round(flops / (res["gemm_only"] / 1e3) / 1e12, 2), "scaling": "strong",
            "c_allgather_ms": round(gather_ms, 3) if gather_ms is not None else None,
            "step_with_allgather_ms": {"gemm_then_nccl_allgather": round(unfused_ms, 4) if unfused_ms else None,
                                       "gemm_with_fused_allgather": round(fused_ms, 4) if fused_ms else None},
            "config": {"M": M, "N": N, "K": K, "b_layout": "nk", "chunks": args.chunks,
                       "panel_rows": e - s, "timing": "device, max over ranks"}}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_shape(args) -> int:
    """--shape M,N,K: time one GEMM shape (ours, and cuBLAS unless --no-cublas); one JSON line."""
    import torch
    torch.cuda.set_device(0)
    import b200_gemm
    M, N, K = (int(x) for x in args.shape.split(","))
    t = time_config(M, N, K, args.layout, args.dist, b200_gemm, target_ms=args.target_ms,
                    with_cublas=not args.no_cublas, use_graph=not args.no_graph)
    flops = 2.0 * M * N * K
    nbytes = 2.0 * (M * K + K * N + M * N)
    line = {"config": {"M": M, "N": N, "K": K, "b_layout": args.layout, "data": args.dist},
            "ms": round(t["b200"], 5), "tflops": round(flops / (t["b200"] / 1e3) / 1e12, 1),
            "gbs": round(nbytes / (t["b200"] / 1e3) / 1e9, 1)}
    if "cublas" in t:
        line["cublas_ms"] = round(t["cublas"], 5)
    print(json.dumps(line), flush=True)
    return 0


def _config(layout, world):
    return {"workload": "bf16 gemm M=N=K=4096 per GPU, A[M,K] x B[K,N] row-major, U(-1,1), fp32 accumulate, "
                        "bf16 out; N>1: one 4096-row A panel per rank, B broadcast from rank 0 every step "
                        "(copy engines over NVLink, overlapped with the previous step's GEMM), C sharded",
            "M_per_gpu": M_PER_RANK, "N": N_DIM, "K": K_DIM, "b_layout": layout,
            "parallelism": f"row-sharded x{world}" if world > 1 else "single",
            "l2": f"inputs larger than L2: rotating {ROTATE} A/B/C sets ({ROTATE * 96} MiB > 126 MB L2)"}


class _Steps:
    """The headline job's steps.  N=1: one GEMM per step.  N>1: step s
    multiplies this rank's A panel by rank 0's B of step s, delivered by
    PeerBroadcast (copy engines over NVLink): while the GEMM of step s runs,
    the B of steps s+1 and s+2 are already moving (three receive slots; at 8
    GPUs one exchange takes longer than one GEMM).  Step numbers count up
    across warm-up and timed steps (the exchange's flags compare them)."""

    def __init__(self, b200_gemm, A, B, C, layout, world, rank, stream):
        self.g, self.A, self.B, self.C, self.layout = b200_gemm, A, B, C, layout
        self.world, self.rank, self.stream = world, rank, stream
        self.s = 0
        self.pb = None
        if world > 1:
            from b200_gemm.dist import PeerBroadcast
            nbytes = B[0].numel() * B[0].element_size()
            self.pb = PeerBroadcast(nbytes)
            self.ahead = self.pb.SLOTS - 1  # steps issued ahead of the one being multiplied
            self.slot_views = [None] * self.pb.SLOTS
            if rank != 0:
                self.slot_views = [self.pb.data(k).view(torch_bf16()).view(B[0].shape) for k in range(self.pb.SLOTS)]
            for k in range(self.ahead):
                self.pb.issue(k, B[k % ROTATE] if rank == 0 else None)

    def b_of(self, s):
        return self.B[s % ROTATE] if (self.world == 1 or self.rank == 0) else self.slot_views[s % self.pb.SLOTS]

    def __call__(self):
        s = self.s
        self.s += 1
        j = s % ROTATE
        if self.pb is None:
            self.g.gemm(self.A[j], self.B[j], b_layout=self.layout, out=self.C[j])
            return
        t = s + self.ahead
        self.pb.issue(t, self.B[t % ROTATE] if self.rank == 0 else None)
        # waits for this step's B and releases its slot inside the GEMM kernel
        self.pb.gemm(s, self.A[j], tuple(self.B[0].shape), out=self.C[j], b_layout=self.layout,
                     src=self.B[j] if self.rank == 0 else None, stream=self.stream)

    def exchange_only(self):
        """One step of the B exchange alone (no GEMM): its cost on its own."""
        s = self.s
        self.s += 1
        t = s + self.ahead
        self.pb.issue(t, self.B[t % ROTATE] if self.rank == 0 else None)
        self.pb.wait(s, self.stream)
        self.pb.release(s, self.stream)

    def close(self):
        if self.pb is not None:
            self.pb.close()


def torch_bf16():
    import torch
    return torch.bfloat16


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--layout", default="kn", choices=["kn", "nk"])
    ap.add_argument("--e2e-steps", type=int, default=30)
    ap.add_argument("--cublas-steps", type=int, default=-1,
                    help="cuBLAS comparison loop length (default: same as --steps, so both run under the same "
                         "power state; 0: skip)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-rows", type=int, default=256)
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the per-config lines (BASELINE configs 2-4 at N=1, the row-sharded job at every N)")
    ap.add_argument("--sweep", action="store_true", help="time every single-GPU BASELINE config (one line each)")
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="sweep: time direct launches instead of graph replay")
    ap.add_argument("--shape", default=None, help="time one shape M,N,K (one JSON line)")
    ap.add_argument("--dist", default="normal", choices=["normal", "uniform"])
    ap.add_argument("--target-ms", type=float, default=250.0)
    ap.add_argument("--rowshard", action="store_true", help="BASELINE config 5: row-sharded 131072x8192x8192")
    ap.add_argument("--epilogue", action="store_true", help="fused epilogue vs unfused and vs cuBLAS addmm")
    ap.add_argument("--fp32", action="store_true", help="fp32 GEMM (reference fp32_matmul) vs cuBLAS fp32")
    ap.add_argument("--attention", action="store_true", help="causal flash attention (reference flash_attn)")
    ap.add_argument("--rowshard-m", type=int, default=131072)
    ap.add_argument("--chunks", type=int, default=1, help="--rowshard: column chunks of B broadcast one by one")
    args = ap.parse_args(argv)
    if args.rowshard:
        return run_rowshard(args)
    if args.shape:
        return run_shape(args)
    if args.epilogue:
        return run_epilogue(args)
    if args.fp32:
        return run_fp32(args)
    if args.attention:
        return run_attention(args)
    if args.sweep:
        return run_sweep(args)
    if args.warmup < 3:
        args.warmup = 3
    args.e2e_steps = max(args.e2e_steps, 1)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, world, rank)

    import torch
    import torch.distributed as dist
    world, rank, local = _dist_setup()
    import b200_gemm

    dev = torch.device("cuda", torch.cuda.current_device())
    M, N, K = M_PER_RANK, N_DIM, K_DIM
    layout = args.layout
    g = torch.Generator(device=dev).manual_seed(1234 + rank)

    def rand(shape):
        return (torch.rand(shape, generator=g, device=dev, dtype=torch.float32) * 2 - 1).to(torch.bfloat16)

    b_shape = (K, N) if layout == "kn" else (N, K)
    A = [rand((M, K)) for _ in range(ROTATE)]
    if rank == 0:
        B = [rand(b_shape) for _ in range(ROTATE)]
    else:
        B = [torch.empty(b_shape, dtype=torch.bfloat16, device=dev) for _ in range(ROTATE)]
    C = [torch.empty((M, N), dtype=torch.bfloat16, device=dev) for _ in range(ROTATE)]
    stream = torch.cuda.current_stream(dev)

    # The first collective on a new communicator sets up its connections:
    # warm it outside any timed region, then time the broadcast on its own.
    bcast_ms = None
    if world > 1:
        for t in B:
            dist.broadcast(t, src=0)
        torch.cuda.synchronize()
        _barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        e0.record(stream)
        for r in range(reps):
            for t in B:
                dist.broadcast(t, src=0)
        e1.record(stream)
        torch.cuda.synchronize()
        bcast_ms = _max_over_ranks(e0.elapsed_time(e1) / (reps * ROTATE), world)

    step = _Steps(b200_gemm, A, B, C, layout, world, rank, stream)
    for i in range(args.warmup):
        step()
    torch.cuda.synchronize()
    b200_gemm.check_status()

    props = torch.cuda.get_device_properties(dev)
    sampler = ClockSampler(f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0")
    t_beg, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # A step is exactly one GEMM launch (plus, at N>1, the exchange's stream
    # operations), and consecutive launches overlap through programmatic
    # dependent launch: no event is put on the stream between them (an event
    # record there serialises them, ~3 us a step), so the mean launch
    # duration is taken as the timed region / steps (at N>1 an upper bound
    # that includes the exchange's waits).

    _barrier(world)
    torch.cuda.synchronize()
    sampler.start()
    t_beg.record(stream)
    h0 = time.perf_counter()
    for i in range(args.steps):
        step()
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps  # host time to enqueue one step
    t_end.record(stream)
    torch.cuda.synchronize()
    _barrier(world)
    sampler.stop()
    b200_gemm.check_status()

    total_ms = _max_over_ranks(t_beg.elapsed_time(t_end), world)
    launch_ms = t_beg.elapsed_time(t_end) / args.steps
    launch_ms_max = _max_over_ranks(launch_ms, world)
    host_ms_max = _max_over_ranks(host_ms, world)
    tflops = world * FLOPS_PER_STEP * args.steps / (total_ms / 1e3) / 1e12
    kernel_tflops = FLOPS_PER_STEP / (launch_ms_max / 1e3) / 1e12

    # cuBLAS on the same GPU, same rotation and loop shape (context only; not the product).
    cub_tflops = None
    if rank == 0 and args.cublas_steps != 0:
        n_cub = args.steps if args.cublas_steps < 0 else args.cublas_steps
        for i in range(10):
            torch.matmul(A[i % ROTATE], B[i % ROTATE] if layout == "kn" else B[i % ROTATE].t(), out=C[i % ROTATE])
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        c0.record()
        for i in range(n_cub):
            j = i % ROTATE
            torch.matmul(A[j], B[j] if layout == "kn" else B[j].t(), out=C[j])
        c1.record()
        torch.cuda.synchronize()
        cub_tflops = FLOPS_PER_STEP * n_cub / (c0.elapsed_time(c1) / 1e3) / 1e12

    # ---- N>1: the B exchange checked and timed on its own, and the NCCL
    # alternative (broadcast, then GEMM, on one stream) in the same run ------
    exchange = None
    if world > 1:
        exchange = _exchange_report(step, A, B, C, layout, world, rank, stream, b200_gemm)
    step.close()
    # ---- N>1: parity of the sharded result and of the fused all-gather -------
    parity = _multi_gpu_parity(A[0], B[0], layout, world, rank, b200_gemm) if world > 1 else None
    if parity is not None:
        parity["b_exchange"] = exchange.pop("bitwise_ok")
    del A, B, C
    torch.cuda.empty_cache()

    # ---- end to end through the public API with host buffers ----------------
    e2e = _e2e(args, world, rank, dev, layout, b200_gemm)

    # ---- BASELINE config 5 (row-sharded 131072x8192x8192) at this N ---------
    rowshard = None if args.no_configs else _rowshard_object(args, world, rank, dev, b200_gemm)

    peaks = _peaks()
    long_region = total_ms >= 500.0
    peak = peaks["sustained"] if long_region else peaks["burst"]
    traffic = _traffic()
    line = {
        "metric": METRIC,
        "value": round(tflops, 2),
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": _config(layout, world),
        "pct_of_peak": round(100.0 * tflops / world / peak, 2),
        "roofline": {"bound": "tensor", "achieved": round(kernel_tflops, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(kernel_tflops / peak, 4),
                     "peak_kind": ("sustained" if long_region else "burst") + f" bf16 cuBLAS, {peaks['source']}",
                     "traffic": (traffic or {}).get("bytes_per_launch"),
                     "algorithmic_flops_per_launch": FLOPS_PER_STEP,
                     "avg_launch_ms": round(launch_ms_max, 5),
                     "launch_timing": "timed region / steps: one GEMM launch per step, back to back (max over ranks)"},
        "host_enqueue_ms_per_step": round(host_ms_max, 4),
        "clocks": sampler.summary(),
        "gpu_launches": args.steps,
        "e2e": e2e,
        "cublas_same_loop_tflops": round(cub_tflops, 2) if cub_tflops else None,
        "b_broadcast_ms": round(bcast_ms, 4) if bcast_ms is not None else None,
    }
    if exchange is not None:
        line["b_exchange"] = exchange
    if parity is not None:
        line["parity"] = parity
    if rowshard is not None:
        line["rowshard"] = rowshard
    if rank == 0 and world == 1 and not args.no_configs:
        line["configs"] = _config_lines(b200_gemm, peaks)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def _exchange_report(step, A, B, C, layout, world, rank, stream, b200_gemm):
    """After the timed region at N>1: (1) the B that the last step multiplied
    on every rank equals rank 0's, bit for bit; (2) the exchange alone per
    step; (3) the design it replaces, NCCL broadcast then GEMM on one stream,
    per step; device time, max over ranks."""
    import torch
    import torch.distributed as dist
    last = step.s - 1
    torch.cuda.synchronize()
    ref = B[last % ROTATE].clone() if rank == 0 else torch.empty_like(B[0])
    dist.broadcast(ref, src=0)
    torch.cuda.synchronize()
    ok = torch.tensor([int(torch.equal(step.b_of(last), ref))], device=ref.device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    del ref

    def timed(fn, n=20):
        for _ in range(3):
            fn(0)
        torch.cuda.synchronize()
        _barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(n):
            fn(i)
        e1.record(stream)
        torch.cuda.synchronize()
        _barrier(world)
        return _max_over_ranks(e0.elapsed_time(e1) / n, world)

    ex_ms = timed(lambda i: step.exchange_only())
    torch.cuda.synchronize()

    def nccl_step(i):
        j = i % ROTATE
        dist.broadcast(B[j], src=0)
        b200_gemm.gemm(A[j], B[j], b_layout=layout, out=C[j])
    nccl_ms = timed(nccl_step)
    b200_gemm.check_status()
    return {"bitwise_ok": bool(ok.item()),
            "how": "copy engines (cudaMemcpyAsync into peers' IPC-mapped slots, rank 0 scatters one piece per "
                   "rank and each rank forwards its piece) with stream-ordered flags between GPUs; no SMs",
            "exchange_only_ms": round(ex_ms, 4), "nccl_broadcast_then_gemm_ms": round(nccl_ms, 4),
            "bytes_per_step": B[0].numel() * B[0].element_size()}


def _multi_gpu_parity(a, b, layout, world, rank, b200_gemm):
    """After the timed region at N>1: (1) the row-sharded C of every rank on
    sampled rows against an fp32 CPU product of the same bf16 inputs (the
    north_star bound: |dC| <= 2 bf16 ulp, relative Frobenius <= 1e-3);
    (2) the GEMM with the C all-gather fused in (b200_gemm_bf16_allgather)
    against the plain GEMM followed by NCCL's all-gather, bit for bit on every
    rank.  Both flags are ANDed over the ranks."""
    import torch
    import torch.distributed as dist
    from b200_gemm.dist import GatheredC, row_sharded_gemm_gather
    M_loc, K = a.shape
    N = b.shape[1] if layout == "kn" else b.shape[0]
    M = M_loc * world
    c = b200_gemm.gemm(a, b, b_layout=layout)
    full = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    dist.all_gather_into_tensor(full, c)
    # (1) sampled rows of this rank's panel
    rows = torch.arange(0, M_loc, M_loc // 16, device=a.device)
    a32 = a[rows].float().cpu()
    b32 = (b if layout == "kn" else b.t()).float().cpu()
    ref = a32 @ b32
    got = c[rows].float().cpu()
    rms = float(ref.pow(2).mean().sqrt())
    mag = torch.clamp(ref.abs(), min=rms * 2.0 ** -8)
    ulp = torch.exp2(torch.floor(torch.log2(mag)) - 7)
    ok_elem = bool(((got - ref).abs() <= 2 * ulp).all())
    # Rounding the exact product to bf16 alone costs ~1.6e-3 relative
    # Frobenius error, so the 1e-3 bound compares two bf16-rounded results.
    ref16 = ref.bfloat16().float()
    frob = float((got - ref16).norm() / max(float(ref.norm()), 1e-30))
    ok1 = ok_elem and frob <= 1e-3
    # (2) fused all-gather
    gbuf = GatheredC(M, N)
    fused = row_sharded_gemm_gather(a, b, gathered=gbuf, M=M, b_layout=layout, broadcast=False)
    torch.cuda.synchronize()
    ok2 = bool(torch.equal(fused, full))
    b200_gemm.check_status()
    gbuf.close()
    flags = torch.tensor([int(ok1), int(ok2)], dtype=torch.int32, device=a.device)
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    return {"rowshard": bool(flags[0]), "gather": bool(flags[1]), "rowshard_rel_frob": round(frob, 7),
            "checked": f"rowshard: {len(rows)} rows per rank vs fp32 CPU product (|dC| <= 2 bf16 ulp; relative "
                       f"Frobenius vs the product rounded to bf16 <= 1e-3); gather: all {M}x{N} of C on "
                       f"every rank vs GEMM + NCCL all_gather_into_tensor, bitwise"}


def _rowshard_object(args, world, rank, dev, b200_gemm):
    """BASELINE config 5 at this N: C = A B with A [131072, 8192] split into one
    row panel per rank, B [8192, 8192] (stored [N, K], the reference's layout)
    broadcast from rank 0, C sharded.  gemm_only_ms: the panel GEMMs alone;
    broadcast_plus_gemm_ms: the whole job, B from rank 0 on the copy engines
    in two parts (the GEMM of the first 1024 columns of C starts when their
    rows of B have arrived, the rest of B moves meanwhile,
    dist.row_sharded_gemm_peer); nccl_broadcast_plus_gemm_ms: the same job with
    an NCCL broadcast of B before the GEMM; all device-timed, max over ranks.
    At N>1 rank 0 also runs the whole job alone (the N=1 figure in the same
    run), so the speed-up is measured, not assumed."""
    import torch
    import torch.distributed as dist
    from b200_gemm.dist import PeerBroadcast, row_sharded_gemm, row_sharded_gemm_peer, shard_rows
    Mt, N, K = args.rowshard_m, 8192, 8192
    flops = 2.0 * Mt * N * K
    s, e = shard_rows(Mt, world, rank)
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    a = (torch.rand((e - s, K), generator=g, device=dev) * 2 - 1).to(torch.bfloat16)
    b = (torch.rand((N, K), generator=g, device=dev) * 2 - 1).to(torch.bfloat16)  # [N, K]
    c = torch.empty((e - s, N), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)

    def timed(fn, budget_ms=300.0):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        fn()
        torch.cuda.synchronize()
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        one = max(_max_over_ranks(e0.elapsed_time(e1), world), 1e-3)  # same step count on every rank
        n = max(3, int(budget_ms / one))
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        _barrier(world)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        _barrier(world)
        return _max_over_ranks(e0.elapsed_time(e1) / n, world), n

    gemm_ms, n1 = timed(lambda: row_sharded_gemm(a, b, M=Mt, b_layout="nk", out=c, broadcast=False))
    nccl_ms, n3 = timed(lambda: row_sharded_gemm(a, b, M=Mt, b_layout="nk", out=c, broadcast=world > 1))
    if world > 1:
        pb = PeerBroadcast(b.numel() * b.element_size())
        step = [0]

        def job():
            row_sharded_gemm_peer(a, b, M=Mt, exchange=pb, step=step[0], out=c, first_rows=1024)
            step[0] += 2
        both_ms, n2 = timed(job)
        torch.cuda.synchronize()
        pb.close()
    else:
        both_ms, n2 = nccl_ms, n3
    b200_gemm.check_status()
    del a, c
    out = {"workload": f"BASELINE config 5: A[{Mt},{K}] row panels x B stored [{N},{K}] (C = A B^T), U(-1,1), "
                       f"B broadcast from rank 0 (copy engines, two parts overlapped with the GEMM), C sharded; "
                       f"strong scaling",
           "M": Mt, "N": N, "K": K, "panel_rows": e - s, "steps": [n1, n2, n3],
           "gemm_only_ms": round(gemm_ms, 4), "broadcast_plus_gemm_ms": round(both_ms, 4),
           "nccl_broadcast_plus_gemm_ms": round(nccl_ms, 4),
           "gemm_only_tflops": round(flops / gemm_ms / 1e9, 1),
           "tflops": round(flops / both_ms / 1e9, 1), "timing": "device, max over ranks"}
    if world > 1:
        # The whole job on rank 0 alone, in the same run, for the speed-up.
        t1 = torch.zeros(1, dtype=torch.float64, device=dev)
        if rank == 0:
            ga = torch.Generator(device=dev).manual_seed(78)
            a1 = (torch.rand((Mt, K), generator=ga, device=dev) * 2 - 1).to(torch.bfloat16)
            c1 = torch.empty((Mt, N), dtype=torch.bfloat16, device=dev)
            for _ in range(2):
                b200_gemm.gemm(a1, b, b_layout="nk", out=c1)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = 10
            e0.record(stream)
            for _ in range(reps):
                b200_gemm.gemm(a1, b, b_layout="nk", out=c1)
            e1.record(stream)
            torch.cuda.synchronize()
            t1[0] = e0.elapsed_time(e1) / reps
            del a1, c1
        dist.broadcast(t1, src=0)
        one_gpu_ms = float(t1[0])
        out["one_gpu_ms"] = round(one_gpu_ms, 4)
        out["speedup_vs_one_gpu"] = round(one_gpu_ms / both_ms, 3)
        out["speedup_gemm_only"] = round(one_gpu_ms / gemm_ms, 3)
    del b
    torch.cuda.empty_cache()
    return out


def _config_lines(b200_gemm, peaks):
    """BASELINE configs 2-4 on this GPU (square sweep, skinny M <= 128, projection
    shapes with ragged M), B [K,N]: ours and cuBLAS in the same loop, inputs
    rotating over sets larger than L2, graph replay for GEMMs under 1 ms."""
    out = []
    for family, M, N, K, dist_kind in sweep_configs():
        if family == "square" and M == 4096:
            continue  # the headline above
        t = time_config(M, N, K, "kn", dist_kind, b200_gemm, target_ms=60.0, warmup=5, with_split=False)
        flops = 2.0 * M * N * K
        nbytes = 2.0 * (M * K + K * N + M * N)
        tf = flops / (t["b200"] / 1e3) / 1e12
        gbs = nbytes / (t["b200"] / 1e3) / 1e9
        hbm = family == "skinny"
        out.append({"family": family, "M": M, "N": N, "K": K, "us": round(t["b200"] * 1e3, 2),
                    "tflops": round(tf, 1), "gbs": round(gbs, 1), "bound": "hbm" if hbm else "tensor",
                    "frac": round(gbs / peaks["hbm_gbs"] if hbm else tf / peaks["burst"], 4),
                    "cublas_us": round(t["cublas"] * 1e3, 2) if "cublas" in t else None,
                    "vs_cublas": round(t["cublas"] / t["b200"], 3) if "cublas" in t else None})
    return out


def _e2e(args, world, rank, dev, layout, b200_gemm):
    """Host buffers -> device -> GEMM -> host, every step, through the public API.

    Pipelined like a serving loop: three streams (copy in, compute, copy out)
    and two device buffer sets, so step i+1's host->device copy and step i-1's
    device->host copy overlap step i's GEMM.  Every step still moves its own
    inputs in and its result out inside the timed region.  At N>1 each rank
    uploads its own A panel and a 1/N slice of B (rows of the [K,N] B) from its
    pinned host memory, and the slices are all-gathered over NVLink (NCCL), so
    no single PCIe link carries all of B."""
    import torch
    import torch.distributed as dist
    M, N, K = M_PER_RANK, N_DIM, K_DIM
    b_shape = (K, N) if layout == "kn" else (N, K)
    rows_b = b_shape[0]
    if world > 1 and rows_b % world != 0:
        raise ValueError("B's rows must split evenly over the ranks")
    slice_rows = rows_b // world
    g = torch.Generator().manual_seed(99)
    b_full = (torch.rand(b_shape, generator=g) * 2 - 1).to(torch.bfloat16)
    b_h = b_full[rank * slice_rows:(rank + 1) * slice_rows].clone().pin_memory()
    del b_full
    g = torch.Generator().manual_seed(100 + rank)
    a_h = ((torch.rand((M, K), generator=g) * 2 - 1).to(torch.bfloat16)).pin_memory()
    c_h = [torch.empty((M, N), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    a_d = [torch.empty((M, K), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    b_d = [torch.empty(b_shape, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    c_d = [torch.empty((M, N), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    s_in, s_comp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    for e in ev_comp + ev_out:
        e.record(torch.cuda.current_stream(dev))

    def step(i):
        j = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_comp[j])  # the GEMM that last read a_d[j]/b_d[j] is done
            mine = b_d[j][rank * slice_rows:(rank + 1) * slice_rows]
            mine.copy_(b_h, non_blocking=True)
            if world > 1:
                dist.all_gather_into_tensor(b_d[j], mine)
            a_d[j].copy_(a_h, non_blocking=True)
            ev_in[j].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(ev_in[j])
            s_comp.wait_event(ev_out[j])  # c_d[j] has been copied out
            b200_gemm.gemm(a_d[j], b_d[j], b_layout=layout, out=c_d[j])
            ev_comp[j].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[j])
            c_h[j].copy_(c_d[j], non_blocking=True)
            ev_out[j].record(s_out)

    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    _barrier(world)
    main = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main)
    for s_ in (s_in, s_comp, s_out):
        s_.wait_stream(main)
    for i in range(args.e2e_steps):
        step(i)
    for s_ in (s_in, s_comp, s_out):
        main.wait_stream(s_)
    e1.record(main)
    torch.cuda.synchronize()
    _barrier(world)
    ms = _max_over_ranks(e0.elapsed_time(e1), world)
    tflops = world * FLOPS_PER_STEP * args.e2e_steps / (ms / 1e3) / 1e12
    h2d = a_h.numel() * 2 + b_h.numel() * 2
    return {"value": round(tflops, 3), "unit": "TFLOPS", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": c_h[0].numel() * 2, "bytes_per_step_are": "per rank",
            "h2d_bytes_per_step_all_ranks": h2d * world, "steps": args.e2e_steps,
            "ms_per_step": round(ms / args.e2e_steps, 4),
            "path": "pinned host A panel (+ this rank's 1/N slice of B) -> H2D"
                    + (" -> NCCL all-gather of B" if world > 1 else "")
                    + " -> b200_gemm.gemm (C ABI) -> D2H C, every step; copy-in, GEMM and copy-out on three "
                      "streams with two buffer sets (step i+1 in, i compute, i-1 out overlap)"}


if __name__ == "__main__":
    sys.exit(main())
