"""Benchmark of the PolyTensor hot path on B200 (one JSON line on stdout, rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

Default workload (configs[1] of the baseline): the polynomial matrix product
C_k = sum_{i+j=k} A_i B_j of float32 PolyTensors, M = N = K = 8192, degree 4, planes
N(0,1)/k!.  A "step" is one product over one pair of resident operands; the metric is
coefficient TFLOP/s = 2*M*N*K*(n+1)(n+2)/2 per step (algorithmic work, the split-bf16
tensor-core passes are not counted).  With N > 1 (torchrun) every rank multiplies its own
operands (replicas, weak scaling) and the value is total work / max-over-ranks time.

``--impl reference`` times the reference algorithm on the host CPU instead (the oracle
restatement of src/polytensors/_plain.py:118-128, all host threads, a bounded row sample).
"""

import argparse
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "poly-tensors_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

WORKLOADS = {
    "poly_matmul": dict(M=8192, N=8192, K=8192, degree=4, dtype="float32"),
    "poly_matmul_f64": dict(M=4096, N=4096, K=4096, degree=2, dtype="float64"),
    "poly_matmul_2048": dict(M=2048, N=2048, K=2048, degree=4, dtype="float32"),
}


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return data, "measured"
    return FALLBACK_PEAKS, "fallback"


# ------------------------------------------------------------------------------------
# clocks sampled with nvidia-smi while the timed region runs

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.thread is not None:
                self.thread.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------
# workload: polynomial matrix product

def make_series(shape, n, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(*shape, generator=g, dtype=torch.float32) / math.factorial(k)).to(dtype)
            for k in range(n + 1)]


def matmul_flops(M, N, K, n):
    return 2.0 * M * N * K * (n + 1) * (n + 2) / 2


def cpu_matmul_rate(cfg, threads, target_s=12.0):
    """Reference algorithm (oracle restatement of plain_polynomial_product, matrix=True) on the
    host CPU over a bounded row sample of A.  Returns (TFLOP/s, sample description)."""
    from oracle import polyref

    dtype = getattr(torch, cfg["dtype"])
    torch.set_num_threads(threads)
    M, N, K, n = cfg["M"], cfg["N"], cfg["K"], cfg["degree"]
    B = make_series((K, N), n, 2, dtype)
    rows = 64
    with torch.no_grad():
        while True:
            A = make_series((rows, K), n, 1, dtype)
            t0 = time.perf_counter()
            polyref.poly_matmul(A, B)
            dt = time.perf_counter() - t0
            if dt >= target_s / 4 or rows >= M:
                break
            rows = min(M, rows * max(2, int(target_s / 4 / max(dt, 1e-3))))
    rate = matmul_flops(rows, N, K, n) / dt / 1e12
    return rate, f"{rows} of {M} rows of A, full B ({cfg['dtype']}, degree {n}), {dt:.1f} s"


def run_matmul(args, cfg, rank, world, device):
    from polytensors_b200 import _kernels, _lib

    dtype = getattr(torch, cfg["dtype"])
    M, N, K, n = cfg["M"], cfg["N"], cfg["K"], cfg["degree"]
    flops = matmul_flops(M, N, K, n)
    A_host = [t.pin_memory() for t in make_series((M, K), n, 1 + 10 * rank, dtype)]
    B_host = [t.pin_memory() for t in make_series((K, N), n, 2 + 10 * rank, dtype)]
    A = [t.to(device) for t in A_host]
    B = [t.to(device) for t in B_host]
    esz = A[0].element_size()
    in_bytes = (n + 1) * (M * K + K * N) * esz
    out_bytes = (n + 1) * M * N * esz
    stream = torch.cuda.current_stream(device)
    lib = _lib.load()

    def step():
        return _kernels.poly_matmul(A, B)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    barrier(world)
    _lib.profile_query("poly_gemm")
    _lib.profile_enable(True)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clocks:
        torch.cuda.synchronize(device)
        barrier(world)
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        torch.cuda.synchronize(device)
        barrier(world)
    _lib.profile_enable(False)
    ms = start.elapsed_time(end) / args.steps
    kernel_ms, launches = _lib.profile_query("poly_gemm")
    ms_max = max_over_ranks(ms, world, device)

    # end to end: pinned host operands -> device -> product -> host, every step
    outs_host = [torch.empty((M, N), dtype=dtype).pin_memory() for _ in range(n + 1)]

    def e2e_step():
        a = [t.to(device, non_blocking=True) for t in A_host]
        b = [t.to(device, non_blocking=True) for t in B_host]
        c = _kernels.poly_matmul(a, b)
        for dst, src in zip(outs_host, c):
            dst.copy_(src, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize(device)
    barrier(world)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e_end.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end) / args.steps, world, device)

    pk, source = peaks()
    peak = pk["bf16_tflops"]
    achieved = flops / (kernel_ms / launches / 1e3) / 1e12 if launches else None
    result = {
        "metric": f"poly-matmul coeff TFLOP/s ({cfg['dtype']}, M=N=K={M}, degree {n})",
        "value": world * flops / (ms_max / 1e3) / 1e12,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_max,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 (bf16x3 split on tcgen05, fp32 accumulate)" if dtype == torch.float32 else cfg["dtype"],
        "data": "synthetic: planes N(0,1)/k!, seeded",
        "config": {"workload": f"poly_matmul M=N=K={M} degree {n} {cfg['dtype']}", "M": M, "N": N, "K": K,
                   "degree": n, "dtype": cfg["dtype"], "parallelism": f"replicas x{world}",
                   "l2": "inputs larger than L2 (no flush)"},
        "e2e": {"value": world * flops / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": out_bytes,
                "api": "polytensors_b200._kernels.poly_matmul (pk_poly_gemm C ABI)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak if achieved else None, "traffic": None,
                     "peak_source": f"bf16_tflops ({source})",
                     "note": "algorithmic flops; the float32 path issues 3 bf16 MMAs per product, "
                             "so its tensor-pipe ceiling is peak/3" if dtype == torch.float32 else
                             "float64 runs on DMMA; bf16 peak shown for reference"},
        "gpu_launches": 3 * args.steps,
        "kernel_ms_per_launch": kernel_ms / launches if launches else None,
        "clocks": clocks.summary(),
    }
    return result


# ------------------------------------------------------------------------------------

def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return t.item()


def reference_arm(args, cfg):
    threads = os.cpu_count() or 1
    samples = []
    for _ in range(max(1, args.warmup) if args.warmup else 0):
        pass
    desc = ""
    for _ in range(args.steps):
        rate, desc = cpu_matmul_rate(cfg, threads, target_s=8.0)
        samples.append(rate)
    value = statistics.median(samples)
    return {
        "impl": "reference",
        "metric": f"poly-matmul coeff TFLOP/s ({cfg['dtype']}, M=N=K={cfg['M']}, degree {cfg['degree']})",
        "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": cfg["dtype"],
        "data": "synthetic: planes N(0,1)/k!, seeded",
        "config": {"workload": f"poly_matmul M=N=K={cfg['M']} degree {cfg['degree']} {cfg['dtype']}"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="poly_matmul", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="polykern", choices=["polykern", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    cfg = WORKLOADS[args.workload]

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(reference_arm(args, cfg)), flush=True)
        return

    if args.warmup < 3:
        print("note: fewer than 3 warm-up steps", file=sys.stderr)
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)
    result = run_matmul(args, cfg, rank, world, device)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, desc = cpu_matmul_rate(cfg, os.cpu_count() or 1)
        result["cpu_baseline"] = {"value": rate, "unit": "TFLOP/s", "cores": os.cpu_count() or 1,
                                  "kind": "port", "sample": desc}
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
