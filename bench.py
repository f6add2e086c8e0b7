"""Benchmark of the PolyTensor hot path on B200 (one JSON line on stdout, rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

Default workload: configs[4], one SGD step of the 12-layer d768 transformer with PolyTensor
parameters (degree 3, float32) over the global batch of 64 x 1024 tokens.  With N > 1
(torchrun, one rank per GPU) the batch is sharded over the ranks and the gradient series are
averaged by one bucketed NCCL all-reduce per step (strong scaling); value = tokens/s of the
whole job, max-over-ranks device time.  The line also carries, under ``poly_matmul``, the
configs[1] float32 polynomial matrix product (M = N = K = 8192, degree 4; replicas on every
rank) with its own roofline, e2e, row-sampled parity and CPU baseline; and under ``parity`` the
training forward + backward checked against the oracle on a bounded full-width sample.

``--impl reference`` times the reference's CPU path on the host cores instead (the oracle
restatement of the reference's plain-range rules, all host threads, bounded samples).  Other
``--workload`` values (poly_matmul, norm_ce, attention, poly_matmul_sweep, ...) are per-op
measurements of configs[1-3].
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

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one product launch: the 2048^3
# degree-4 capture of the current kernel (522 MB) scaled x64 by the units processed, see
# profiles/tc_poly_gemm_f32_n4_2048_and_8192.md.
_GEMM_TRAFFIC = {(8192, 4, "float32"): 522.0e6 * 64}
# DRAM bytes per algorithmic flop of the training step's product launches: 66.6 GB over 19.42 TFLOP
# in a 2-layer, 1-micro-batch step (profiles/tc_poly_gemm_train_dram.md); the full step's traffic is
# this ratio times its algorithmic product flops.
_TRAIN_GEMM_BYTES_PER_FLOP = 66.6e9 / 19.42e12

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
    """The reference's own plain-range product on the host CPU (its PolyTensor `a @ b` inside
    plain_range(), from the package installed in baseline/_ref) over a bounded row sample of A;
    without the package, the oracle restatement of plain_polynomial_product (matrix=True).
    Returns (TFLOP/s, sample description, kind: "reference" or "port")."""
    from oracle import polyref

    dtype = getattr(torch, cfg["dtype"])
    torch.set_num_threads(threads)
    M, N, K, n = cfg["M"], cfg["N"], cfg["K"], cfg["degree"]
    B = make_series((K, N), n, 2, dtype)
    pt = _reference_package()
    if pt is not None:
        RP = pt.PolyTensor
        Bp = RP(tuple(B))

        def product(A):
            with RP.plain_range():
                return RP(tuple(A)) @ Bp

        kind, what = "reference", "the reference's PolyTensor a @ b in plain_range()"
    else:
        def product(A):
            return polyref.poly_matmul(A, B)

        kind, what = "port", "oracle restatement of plain_polynomial_product"
    rows = 64
    with torch.no_grad():
        product(make_series((8, K), n, 1, dtype))   # untimed: the first call's one-time setup
        while True:
            A = make_series((rows, K), n, 1, dtype)
            t0 = time.perf_counter()
            product(A)
            dt = time.perf_counter() - t0
            if dt >= target_s / 4 or rows >= M:
                break
            rows = min(M, rows * max(2, int(target_s / 4 / max(dt, 1e-3))))
    rate = matmul_flops(rows, N, K, n) / dt / 1e12
    return rate, f"{what}: {rows} of {M} rows of A, full B ({cfg['dtype']}, degree {n}), {dt:.1f} s", kind


def matmul_parity(A_host, B_host, C, rows=64, seed=99):
    """Row-sampled parity of one full-size product: rows of A times the whole of B through the
    float64 oracle on the CPU, against the same rows of the GPU product."""
    from oracle import polyref

    M = A_host[0].shape[0]
    idx = torch.randperm(M, generator=torch.Generator().manual_seed(seed))[:rows].sort().values
    want = polyref.poly_matmul([a[idx].double() for a in A_host], [b.double() for b in B_host])
    got = [c[idx.to(c.device)].cpu() for c in C]
    errs = polyref.plane_errors(got, want)
    return {"max_plane_err": max(errs), "per_plane": errs, "tol": 1e-4 if A_host[0].dtype == torch.float32 else 1e-10,
            "metric": "per coefficient plane max|gpu - oracle| / max|oracle|",
            "against": "oracle restatement of plain_polynomial_product, float64, CPU",
            "sample": f"{rows} random rows of A times the full B (seeded)"}


def run_matmul(args, cfg, rank, world, device, parity=False):
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
        C = step()
    torch.cuda.synchronize(device)
    parity_result = matmul_parity(A_host, B_host, C) if parity else None
    del C
    barrier(world)
    _lib.profile_query("poly_gemm")
    _lib.launch_count(reset=True)
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
    gpu_launches = _lib.launch_count()
    ms = start.elapsed_time(end) / args.steps
    kernel_ms, launches = _lib.profile_query("poly_gemm")
    ms_max = max_over_ranks(ms, world, device)

    # end to end: every step copies its operands from pinned host memory, runs the product
    # through the C ABI and copies the product planes back to pinned host memory.  Steps are
    # pipelined over three streams (copy in / compute / copy out) with double-buffered device
    # operands, so host<->device traffic of neighbouring steps overlaps the tensor work.
    outs_host = [[torch.empty((M, N), dtype=dtype).pin_memory() for _ in range(n + 1)] for _ in range(2)]
    dev_in = [([torch.empty_like(t, device=device) for t in A_host], [torch.empty_like(t, device=device) for t in B_host])
              for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    s_cmp = stream
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    out_ready = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]
    for ev in (*in_free, *out_done):
        ev.record(s_cmp)

    def e2e_steps(count):
        for i in range(count):
            b = i % 2
            a_dev, b_dev = dev_in[b]
            with torch.cuda.stream(s_in):
                s_in.wait_event(in_free[b])
                for dst, src in zip(a_dev + b_dev, A_host + B_host):
                    dst.copy_(src, non_blocking=True)
                in_ready[b].record(s_in)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(in_ready[b])
                s_cmp.wait_event(out_done[b])   # the previous product in this slot has left
                c = _kernels.poly_matmul(a_dev, b_dev)
                in_free[b].record(s_cmp)
                out_ready[b].record(s_cmp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(out_ready[b])
                for dst, src in zip(outs_host[b], c):
                    dst.copy_(src, non_blocking=True)
                    src.record_stream(s_out)
                out_done[b].record(s_out)

    e2e_steps(2)
    torch.cuda.synchronize(device)
    barrier(world)
    t0 = time.perf_counter()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record(s_in)
    s_cmp.wait_event(e_start)
    e2e_steps(args.steps)
    s_in.wait_stream(s_out)
    s_in.wait_stream(s_cmp)
    e_end.record(s_in)
    torch.cuda.synchronize(device)
    e2e_wall = (time.perf_counter() - t0) * 1e3 / args.steps
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
        "config": matmul_config(cfg),
        "parallelism": f"replicas x{world}",
        "e2e": {"value": world * flops / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": out_bytes, "ms_per_step": e2e_ms,
                "wall_ms_per_step": e2e_wall,
                "api": "polytensors_b200._kernels.poly_matmul (pk_poly_gemm C ABI), pinned host buffers, "
                       "copy-in / compute / copy-out streams pipelined across steps"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak if achieved else None,
                     # DRAM bytes of one product launch from an ncu capture of this exact default
                     # configuration (dram__bytes_read.sum + dram__bytes_write.sum)
                     "traffic": _GEMM_TRAFFIC.get((M, n, cfg["dtype"])),
                     "peak_source": f"bf16_tflops ({source})",
                     "note": "algorithmic flops; the float32 path issues 3 bf16 MMAs per product, "
                             "so its tensor-pipe ceiling is peak/3" if dtype == torch.float32 else
                             "float64 runs on DMMA; bf16 peak shown for reference"},
        "gpu_launches": gpu_launches,
        "parity": parity_result,
        "kernel_ms_per_launch": kernel_ms / launches if launches else None,
        "clocks": clocks.summary(),
    }
    return result


# ------------------------------------------------------------------------------------
# secondary workloads (configs[2..4] and the configs[1] sweep); not the driver's default

def _series_poly(shape, n, seed, dtype, device, requires_grad=False):
    from polytensors_b200 import PolyTensor

    planes = [p.to(device) for p in make_series(shape, n, seed, dtype)]
    return PolyTensor(tuple(planes), requires_grad=requires_grad)


def _timed(fn, steps, warmup, device, world):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(device)
    with ClockSampler(device.index) as clocks:
        start.record(stream)
        for _ in range(steps):
            fn()
        end.record(stream)
        torch.cuda.synchronize(device)
    barrier(world)
    return max_over_ranks(start.elapsed_time(end) / steps, world, device), clocks.summary()


def _kernel_rates(names_bytes, steps):
    """Per-kernel achieved GB/s from the library's event timings over ``steps`` steps; names_bytes:
    {name: algorithmic bytes per step} (a step may launch a kernel once, or once per chunk)."""
    from polytensors_b200 import _lib

    out = {}
    for name, nbytes in names_bytes.items():
        ms, launches = _lib.profile_query(name)
        if launches:
            out[name] = {"GB/s": nbytes * steps / (ms / 1e3) / 1e9, "ms_per_step": ms / steps,
                         "launches_per_step": launches / steps, "algorithmic_bytes_per_step": nbytes}
    return out


def run_norm_ce(args, rank, world, device):
    """RMSNorm(w) -> GELU -> linear(32000) -> cross entropy, forward + backward, degree 4."""
    import torch.nn.functional as F
    from polytensors_b200 import PolyTensor, _lib

    n, R, H, V = 4, args.rows, 4096, 32000
    x = _series_poly((R, H), n, 1, torch.float32, device, requires_grad=True)
    g = torch.Generator().manual_seed(2)
    w = PolyTensor(((1 + 0.02 * torch.randn(H, generator=g)).to(device),), degree=n, requires_grad=True)
    W = PolyTensor(((0.02 * torch.randn(V, H, generator=g)).to(device),), degree=n, requires_grad=True)
    target = torch.randint(0, V, (R,), generator=g).to(device)

    fused_head = getattr(args, "fused_head", False)

    def step():
        for t in (x, w, W):
            t.grad = None
        with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
            h = F.gelu(F.rms_norm(x, (H,), w))
            if fused_head:
                # linear + cross entropy over row chunks: the logit planes are never all formed
                loss = PolyTensor.linear_cross_entropy(h, W, target)
            else:
                loss = F.cross_entropy(F.linear(h, W), target)
            loss.backward()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    torch.cuda.reset_peak_memory_stats(device)
    step()
    torch.cuda.synchronize(device)
    peak_gb = torch.cuda.max_memory_allocated(device) / 1e9
    for name in ("rmsnorm_fwd", "rmsnorm_bwd", "cross_entropy_fwd", "cross_entropy_bwd", "poly_gemm", "series_map"):
        _lib.profile_query(name)
    _lib.profile_enable(True)
    ms, clocks = _timed(step, args.steps, 0, device, world)
    _lib.profile_enable(False)
    P = n + 1
    rates = _kernel_rates({"rmsnorm_fwd": 2 * P * R * H * 4, "rmsnorm_bwd": 3 * P * R * H * 4,
                           "cross_entropy_fwd": P * R * V * 4, "cross_entropy_bwd": 2 * P * R * V * 4}, args.steps)
    gms, glaunch = _lib.profile_query("poly_gemm")
    T = (n + 1) * (n + 2) / 2
    # forward + the two backward products (+ the logits recomputed in backward with the fused head)
    gemm_flops = (4 if fused_head else 3) * 2 * R * H * V * T
    mem_bytes = sum(r["algorithmic_bytes_per_step"] for r in rates.values())
    mem_ms = sum(r["ms_per_step"] for r in rates.values())
    pk, source = peaks()
    value = mem_bytes / (mem_ms / 1e3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # 1024 of the 16384 rows (the full batch's softmax-series intermediates would not fit in host
        # memory); about 20 s on 16 host cores
        cpu_rows = 1024
        rate, dt, desc, kind = cpu_norm_ce_rate(cpu_rows, os.cpu_count() or 1)
        cpu = {"value": rate, "unit": "GB/s", "cores": os.cpu_count() or 1, "kind": kind, "sample": desc,
               "ms_per_step_extrapolated": dt * 1e3 * 16384 / cpu_rows}
    return {
        "cpu_baseline": cpu,
        "peak_memory_gb": peak_gb,
        "fused_head": bool(fused_head),
        "metric": "norm/CE kernels GB/s (configs[2]: RMSNorm+GELU+linear(32000)+CE fwd+bwd, degree 4, float32)",
        "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: planes N(0,1)/k!, seeded",
        "config": {"workload": f"norm_gelu_linear_ce rows={R} hidden={H} vocab={V} degree {n}",
                   "l2": "inputs larger than L2"},
        "kernels": rates,
        "linear": {"TFLOP/s": gemm_flops * args.steps / (gms / 1e3) / 1e12 if glaunch else None,
                   "launches_per_step": glaunch / args.steps, "flops_per_step": gemm_flops},
        "roofline": {"bound": "hbm", "achieved": value, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": value / pk["hbm_gbs"], "traffic": None, "peak_source": f"hbm_gbs ({source})"},
        "clocks": clocks,
    }


def cpu_norm_ce_rate(rows, threads):
    """The reference's own plain-range chain for configs[2] on the host CPU at `rows` rows (its
    PolyTensor from baseline/_ref: F.rms_norm -> F.gelu -> F.linear(32000) -> F.cross_entropy, forward
    and backward; without the package, the oracle restatement of those rules).  Returns (GB/s of
    the norm/CE algorithmic bytes scaled to the sample, seconds, description, kind)."""
    import torch.nn.functional as F
    from oracle import polyref

    torch.set_num_threads(threads)
    n, H, V = 4, 4096, 32000
    X = make_series((rows, H), n, 1, torch.float32)
    g = torch.Generator().manual_seed(2)
    W0 = [1 + 0.02 * torch.randn(H, generator=g)] + [torch.zeros(H) for _ in range(n)]
    Wl = [0.02 * torch.randn(V, H, generator=g)] + [torch.zeros(V, H) for _ in range(n)]
    target = torch.randint(0, V, (rows,), generator=g)
    pt = _reference_package()
    if pt is not None:
        RP = pt.PolyTensor

        def run(r):
            x = RP(tuple(t[:r] for t in X), requires_grad=True)
            ws, wl = RP(tuple(W0), requires_grad=True), RP(tuple(Wl), requires_grad=True)
            with RP.plain_range(), RP.retain_wrappers():
                F.cross_entropy(F.linear(F.gelu(F.rms_norm(x, (H,), ws)), wl), target[:r]).backward()

        run(8)   # untimed: the first call's one-time setup
        kind, what = "reference", "the reference's PolyTensor chain"
    else:
        def loss_fn(Xs, ws, wl):
            h = polyref.gelu(polyref.rms_norm(Xs, (H,), ws))
            logits = polyref.cauchy(h, [w.t() for w in wl], lambda a, b: a @ b)
            return polyref.cross_entropy(logits, target)

        def run(r):
            seed = [torch.tensor(1.0)] + [torch.tensor(0.0)] * n
            polyref.series_vjp(loss_fn, [X, W0, Wl], seed)

        kind, what = "port", "oracle restatement"
    t0 = time.perf_counter()
    run(rows)
    dt = time.perf_counter() - t0
    P = n + 1
    nbytes = (2 + 3) * P * rows * H * 4 + 3 * P * rows * V * 4
    return nbytes / dt / 1e9, dt, f"{what}: {rows} of 16384 rows, fwd + backward, float32, {dt:.1f} s", kind


def cpu_attention_rate(L, threads, D=128):
    """The reference's SDPA on a (1, 4, L, D) head slice, causal, degree 3, forward + backward,
    float32, in plain range (its PolyTensor from baseline/_ref, which evaluates its decomposition on
    host tensors; without the package, the oracle restatement).  Returns (coefficient TFLOP/s,
    description, kind)."""
    import torch.nn.functional as F
    from oracle import polyref

    torch.set_num_threads(threads)
    n, shape = 3, (1, 4, L, D)
    Q, Kp, V, G = (make_series(shape, n, s, torch.float32) for s in (1, 2, 3, 4))
    pt = _reference_package()
    if pt is not None:
        RP = pt.PolyTensor

        def run(length):
            q, k, v = (RP(tuple(t[:, :, :length] for t in X), requires_grad=True) for X in (Q, Kp, V))
            with RP.plain_range(), RP.retain_wrappers():
                F.scaled_dot_product_attention(q, k, v, is_causal=True).backward(
                    RP(tuple(t[:, :, :length] for t in G)))

        run(16)   # untimed: the first call's one-time setup
        kind, what = "reference", "the reference's PolyTensor SDPA"
    else:
        def run(length):
            polyref.series_vjp(lambda q, k, v: polyref.attention(q, k, v, is_causal=True), [Q, Kp, V], G)

        kind, what = "port", "oracle restatement"
    t0 = time.perf_counter()
    run(L)
    dt = time.perf_counter() - t0
    return (attention_flops(1, 4, L, D, n) / dt / 1e12,
            f"{what}: (1, 4, {L}, {D}) head slice, fwd + backward, {dt:.1f} s", kind)


def attention_flops(B, H, L, D, n):
    T = (n + 1) * (n + 2) / 2
    pairs = L * (L + 1) / 2
    return 6 * T * 2 * B * H * pairs * D   # forward 2 contractions, backward 4 (no recompute counted)


def run_attention_fwd(args, rank, world, device):
    """Forward only of configs[3] (profiling aid): (args.batch, 32, L, 128), degree 3, causal."""
    import torch.nn.functional as F
    from polytensors_b200 import PolyTensor

    n, B, H, L, D = 3, args.batch, 32, args.seq, 128
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    q, k, v = (_series_poly((B, H, L, D), n, s, dtype, device) for s in (1, 2, 3))

    def step():
        with torch.no_grad(), PolyTensor.plain_range():
            F.scaled_dot_product_attention(q, k, v, is_causal=True)

    ms, clocks = _timed(step, args.steps, args.warmup, device, world)
    flops = attention_flops(B, H, L, D, n) / 3
    return {"metric": "poly-attention forward coeff TFLOP/s", "value": flops / (ms / 1e3) / 1e12, "unit": "TFLOP/s",
            "ms_per_step": ms, "config": {"workload": f"attention_fwd B={B} H=32 L={L} D=128 degree 3 causal {args.dtype}"},
            "clocks": clocks}


def run_attention(args, rank, world, device):
    """causal series attention (8, 32, L, 128), degree 3, forward + backward
    (--batch / --heads / --head-dim change the shape, e.g. configs[4]'s (8, 12, 1024, 64))."""
    import torch.nn.functional as F
    from polytensors_b200 import PolyTensor

    n, B, H, L, D = 3, args.batch, getattr(args, "heads", 32), args.seq, getattr(args, "head_dim", 128)
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    q, k, v = (_series_poly((B, H, L, D), n, s, dtype, device, requires_grad=True) for s in (1, 2, 3))
    G = _series_poly((B, H, L, D), n, 4, dtype, device)

    def step():
        for t in (q, k, v):
            t.grad = None
        with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
            o.backward(G)

    def forward_only():
        with torch.no_grad(), PolyTensor.plain_range():
            F.scaled_dot_product_attention(q, k, v, is_causal=True)

    from polytensors_b200 import _lib

    _lib.profile_query("flash_attn_fwd")
    _lib.profile_enable(True)
    fwd_ms, _ = _timed(forward_only, args.steps, 1, device, world)
    _lib.profile_enable(False)
    kms, klaunch = _lib.profile_query("flash_attn_fwd")
    ms, clocks = _timed(step, args.steps, args.warmup, device, world)
    # per-kernel device time of one fwd+bwd step (separate, untimed pass with the event hooks on)
    names = ("flash_attn_fwd", "attn_probs_gemm", "attn_dscores_gemm", "poly_gemm", "attn_probs", "attn_dscores",
             "series_map")
    for nm in names:
        _lib.profile_query(nm)
    _lib.profile_enable(True)
    _timed(step, 2, 0, device, world)
    _lib.profile_enable(False)
    kernels = {}
    for nm in names:
        kt, kl = _lib.profile_query(nm)
        if kl:
            kernels[nm] = {"ms_per_step": kt / 2, "launches_per_step": kl // 2}
    flops = attention_flops(B, H, L, D, n)
    fwd_flops = flops / 3
    pk, source = peaks()
    value = world * flops / (ms / 1e3) / 1e12
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, desc, kind = cpu_attention_rate(min(L, 1024), os.cpu_count() or 1, D)
        cpu = {"value": rate, "unit": "TFLOP/s", "cores": os.cpu_count() or 1, "kind": kind, "sample": desc}
    return {
        "cpu_baseline": cpu,
        "metric": f"poly-attention coeff TFLOP/s (causal, ({B}, {H}, {L}, {D}), degree 3, {args.dtype}, fwd+bwd)",
        "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.dtype,
        "data": "synthetic: planes N(0,1)/k!, seeded",
        "config": {"workload": f"attention B={B} H={H} L={L} D={D} degree 3 causal {args.dtype}",
                   "flops": "12*T*B*H*L(L+1)/2*D (causal pairs, no recompute)"},
        "roofline": {"bound": "tensor", "achieved": value / world, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": value / world / pk["bf16_tflops"], "traffic": None,
                     "peak_source": f"bf16_tflops ({source})"},
        "kernels": kernels,
        "forward": {"ms": fwd_ms, "TFLOP/s": fwd_flops / (fwd_ms / 1e3) / 1e12,
                    "fused_kernel_ms": kms / klaunch if klaunch else None,
                    "fused_kernel_TFLOP/s": fwd_flops / (kms / klaunch / 1e3) / 1e12 if klaunch else None},
        "clocks": clocks,
    }


def transformer_init(layers=12, d=768, heads=12, mlp=3072, vocab=32000, degree=3, seed=0, higher_seed=None):
    """Parameter series of the configs[4] transformer on the CPU: name -> list of degree+1 planes.
    Weights N(0, 0.02), norm weights 1; higher coefficients zero (the config), or with
    ``higher_seed`` N(0, 0.02)/k! (the parity sample, so that every coefficient plane of the
    forward and backward is exercised)."""
    g = torch.Generator().manual_seed(seed)
    gh = torch.Generator().manual_seed(higher_seed) if higher_seed is not None else None

    def series(*shape, ones=False):
        base = torch.ones(*shape) if ones else 0.02 * torch.randn(*shape, generator=g)
        if gh is None:
            return [base] + [torch.zeros(*shape) for _ in range(degree)]
        return [base] + [0.02 * torch.randn(*shape, generator=gh) / math.factorial(k) for k in range(1, degree + 1)]

    p = {"emb": series(vocab, d)}
    for l in range(layers):
        p[f"n1.{l}"], p[f"n2.{l}"] = series(d, ones=True), series(d, ones=True)
        for nm in ("wq", "wk", "wv", "wo"):
            p[f"{nm}.{l}"] = series(d, d)
        p[f"w1.{l}"], p[f"w2.{l}"] = series(mlp, d), series(d, mlp)
    p["nf"] = series(d, ones=True)
    p["head"] = series(vocab, d)
    return p


class TinyGPT:
    """decoder-only transformer with PolyTensor parameters (degree 3, float32):
    embedding, L x [RMSNorm, q/k/v/o linears, causal SDPA, RMSNorm, GELU MLP], RMSNorm, untied head."""

    def __init__(self, device, init, layers=12, d=768, heads=12, vocab=32000, degree=3, poly_cls=None):
        from polytensors_b200 import PolyTensor as Ours

        PolyTensor = poly_cls or Ours   # the reference arm passes the reference's own class
        self.layers, self.d, self.heads, self.vocab, self.degree = layers, d, heads, vocab, degree
        self.p = {}
        for name, planes in init.items():
            if all(not bool(c.any()) for c in planes[1:]):
                poly = PolyTensor((planes[0].to(device),), degree=degree)
            else:
                poly = PolyTensor(tuple(c.to(device) for c in planes))
            self.p[name] = torch.nn.Parameter(poly)

    def parameters(self):
        return list(self.p.values())

    def loss(self, inp, tgt, Z, lam):
        import torch.nn.functional as F

        P, d, H = self.p, self.d, self.heads
        Bt, T = inp.shape
        x = F.embedding(inp, P["emb"])
        for l in range(self.layers):
            h = F.rms_norm(x, (d,), P[f"n1.{l}"])
            q, k, v = (F.linear(h, P[f"{nm}.{l}"]).view(Bt, T, H, d // H).transpose(1, 2) for nm in ("wq", "wk", "wv"))
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(Bt, T, d)
            x = x + F.linear(a, P[f"wo.{l}"])
            h = F.rms_norm(x, (d,), P[f"n2.{l}"])
            x = x + F.linear(F.gelu(F.linear(h, P[f"w1.{l}"])), P[f"w2.{l}"])
        logits = F.linear(F.rms_norm(x, (d,), P["nf"]), P["head"])
        return F.cross_entropy(logits.reshape(-1, self.vocab), tgt.reshape(-1)) * (1 - lam * Z)


def oracle_train_sample(init, ids, layers, dtype, threads, d=768, heads=12, vocab=32000, lam=0.5):
    """The reference algorithm for one configs[4] forward + backward on the host CPU: the oracle
    restatement of the plain-range rules (embedding, RMSNorm, series linear, causal SDPA, GELU,
    cross entropy, the (1 - lam Z) factor) with the swapped-cotangent series backward.
    Returns (seconds, loss series, {name: gradient series})."""
    from oracle import polyref as R

    torch.set_num_threads(threads)
    names = list(init)
    inp, tgt = ids[:, :-1], ids[:, 1:]
    n = len(init[names[0]]) - 1

    def linear(X, W):
        return R.cauchy(X, [w.t() for w in W], lambda a, b: a @ b)

    def loss(*series):
        p = dict(zip(names, series))
        Bt, T = inp.shape
        x = [w[inp] for w in p["emb"]]
        for l in range(layers):
            h = R.rms_norm(x, (d,), p[f"n1.{l}"])
            split = lambda Y: [y.view(Bt, T, heads, d // heads).transpose(1, 2) for y in Y]   # noqa: E731
            q, k, v = (split(linear(h, p[f"{nm}.{l}"])) for nm in ("wq", "wk", "wv"))
            a = [y.transpose(1, 2).reshape(Bt, T, d) for y in R.attention(q, k, v, is_causal=True)]
            x = [u + w for u, w in zip(x, linear(a, p[f"wo.{l}"]))]
            h = R.rms_norm(x, (d,), p[f"n2.{l}"])
            x = [u + w for u, w in zip(x, linear(R.gelu(linear(h, p[f"w1.{l}"])), p[f"w2.{l}"]))]
        logits = linear(R.rms_norm(x, (d,), p["nf"]), p["head"])
        ce = R.cross_entropy([z.reshape(-1, vocab) for z in logits], tgt.reshape(-1))
        factor = [torch.tensor(1.0, dtype=dtype), torch.tensor(-lam, dtype=dtype)] + \
                 [torch.tensor(0.0, dtype=dtype)] * (n - 1)   # 1 - lam Z, Z = (0, 1, 0, ...)
        return R.cauchy(ce, factor)

    series = [[c.to(dtype) for c in init[k]] for k in names]
    seed = [torch.tensor(1.0, dtype=dtype)] + [torch.tensor(0.0, dtype=dtype)] * n
    t0 = time.perf_counter()
    leaves = [[c.detach().clone().requires_grad_(True) for c in X] for X in series]
    out = loss(*leaves)
    objective = sum((seed[k] * out[n - k]).sum() for k in range(n + 1))
    flat = [c for X in leaves for c in X]
    grads = torch.autograd.grad(objective, flat, allow_unused=True)
    dt = time.perf_counter() - t0
    result, pos = {}, 0
    for name, X in zip(names, leaves):
        g = [grads[pos + i] if grads[pos + i] is not None else torch.zeros_like(X[i]) for i in range(n + 1)]
        pos += n + 1
        result[name] = [g[n - j].detach() for j in range(n + 1)]
    return dt, [c.detach() for c in out], result


def reference_train_sample(init, ids, layers, threads, lam=0.5):
    """The reference's own CPU implementation of one configs[4] forward + backward: its PolyTensor
    (the package pip-installed in baseline/_ref) on host tensors inside plain_range(), through the
    same model code (TinyGPT) and inputs as the GPU arm.  Returns the seconds it took, or None
    when the package is absent."""
    pt = _reference_package()
    if pt is None:
        return None
    RP = pt.PolyTensor
    torch.set_num_threads(threads)
    model = TinyGPT(torch.device("cpu"), init, layers=layers, poly_cls=RP)
    Z = RP((torch.tensor(0.0), 1.0), degree=3)
    t0 = time.perf_counter()
    with RP.plain_range(), RP.retain_wrappers():
        loss = model.loss(ids[:, :-1], ids[:, 1:], Z, lam)
        loss.backward()
    return time.perf_counter() - t0


def train_config(layers):
    """The configs[4] workload description, identical in both arms of the bench."""
    return {"workload": f"train transformer layers={layers} d=768 heads=12 mlp=3072 vocab=32000 seq=1024 "
                        f"global_batch=64 degree 3 float32 SGD(lr=0.1)",
            "layers": layers, "d_model": 768, "heads": 12, "mlp": 3072, "vocab": 32000, "seq": 1024,
            "global_batch": 64, "degree": 3, "dtype": "float32", "l2": "inputs and weights larger than L2 (no flush)"}


def matmul_config(cfg):
    M, n = cfg["M"], cfg["degree"]
    return {"workload": f"poly_matmul M=N=K={M} degree {n} {cfg['dtype']}", "M": M, "N": cfg["N"], "K": cfg["K"],
            "degree": n, "dtype": cfg["dtype"], "l2": "inputs larger than L2 (no flush)"}


def train_sample_ids(batch, seq, seed=4321):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 32000, (batch, seq + 1), generator=g)


def train_parity_and_cpu(layers, device, threads, batch=4, seq=256):
    """configs[4] at full width on a bounded sample (batch x seq tokens, parameters with nonzero
    higher coefficients): the GPU forward + backward against the oracle in float64 (parity), and
    the oracle in float32 timed on the host cores (the CPU baseline).  The float32 oracle's own
    distance from float64 is reported beside the GPU's: some loss and gradient coefficients are
    ill-conditioned in float32 whatever computes them, so the pass criterion per plane is
    err <= max(1e-4, 3 x the float32 reference's err), as in the training parity tests."""
    from oracle import polyref as R
    from polytensors_b200 import PolyTensor

    init = transformer_init(layers=layers, seed=0, higher_seed=7)
    ids = train_sample_ids(batch, seq)
    model = TinyGPT(device, init, layers=layers)
    Z = PolyTensor((torch.tensor(0.0, device=device), 1.0), degree=3)
    dev_ids = ids.to(device)
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        loss = model.loss(dev_ids[:, :-1], dev_ids[:, 1:], Z, 0.5)
        loss.backward()
    got_loss = [c.detach().cpu() for c in loss.coeffs]
    got = {k: [c.detach().cpu() for c in p.grad.coeffs] for k, p in model.p.items()}
    del model, loss
    torch.cuda.empty_cache()
    _, want_loss, want = oracle_train_sample(init, ids, layers, torch.float64, threads)
    dt, r32_loss, r32 = oracle_train_sample(init, ids, layers, torch.float32, threads)
    worst = {"err": 0.0, "ratio": 0.0}
    ok = True
    for name, g, w, r in [("loss", got_loss, want_loss, r32_loss)] + [(k, got[k], want[k], r32[k]) for k in want]:
        e_gpu, e_ref = R.plane_errors(g, w), R.plane_errors(r, w)
        for k, (a, b) in enumerate(zip(e_gpu, e_ref)):
            bound = max(1e-4, 3 * b)
            ok &= a <= bound
            if a > worst["err"]:
                worst.update(err=a, name=f"{name}[{k}]", reference_f32_err=b)
            if a / bound > worst["ratio"]:
                worst.update(ratio=a / bound, ratio_at=f"{name}[{k}]")
    tokens = batch * seq
    parity = {"max_plane_err": worst["err"], "at": worst.get("name"),
              "reference_f32_err_there": worst.get("reference_f32_err"),
              "max_err_over_bound": worst["ratio"], "bound_worst_at": worst.get("ratio_at"),
              "within_tolerance": bool(ok),
              "tol": "per plane: err <= max(1e-4, 3 x the float32 reference's err)",
              "metric": "per coefficient plane max|x - oracle64| / max|oracle64|",
              "against": "oracle restatement of the reference's plain-range rules, float64, CPU",
              "sample": f"forward + backward of the full-width model on {batch} x {seq} tokens, "
                        "weights with N(0,0.02)/k! higher coefficients: loss and every parameter gradient"}
    cpu = {"value": tokens / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
           "sample": f"oracle forward + series backward, full width ({layers} layers), {batch} x {seq} tokens, "
                     f"float32, {dt:.1f} s",
           "extrapolated_s_per_step": dt * 64 * 1024 / tokens}
    # the reference's own code on the same sample (zero higher weight coefficients, as the bench's
    # model), when its package is installed
    ref_init = transformer_init(layers=layers, seed=0)
    dt_ref = reference_train_sample(ref_init, ids[:1, :17], layers, threads)   # untimed: one-time setup
    if dt_ref is not None:
        dt_ref = reference_train_sample(ref_init, ids, layers, threads)
    if dt_ref is not None:
        cpu = {"value": tokens / dt_ref, "unit": "tokens/s", "cores": threads, "kind": "reference",
               "sample": f"the reference's PolyTensor (baseline/_ref) forward + backward on host tensors, full width "
                         f"({layers} layers), {batch} x {seq} tokens, float32, {dt_ref:.1f} s",
               "extrapolated_s_per_step": dt_ref * 64 * 1024 / tokens,
               "oracle_port_tokens_per_s": tokens / dt}
    return parity, cpu


def readme_fit_data(seed=0):
    """the README's regression data, seeded: Y = X A + b + E (noise 0.1), independent
    X', Y' of matching variance, and the ten minibatches of 16 indices each."""
    g = torch.Generator().manual_seed(seed)
    n, d, noise = 64, 3, 0.1
    A, b = torch.randn(d, generator=g), torch.randn((), generator=g)
    X = torch.randn(n, d, generator=g)
    E = noise * torch.randn(n, generator=g)
    Y = X @ A + b + E
    Xp = torch.randn(n, d, generator=g)
    Yp = (d + 1 + noise ** 2) ** 0.5 * torch.randn(n, generator=g)
    batches = [(torch.randint(n, (16,), generator=g), torch.randint(n, (16,), generator=g)) for _ in range(10)]
    return X, Y, Xp, Yp, batches


def gpu_readme_fit(device, data, degree=5, poly_cls=None):
    """The README fit through this package's API on the GPU (plain range): 10 SGD steps of
    loss = (signal + (1 - Z) noise) / 2; returns the coefficient planes of w and c.  With the
    reference's PolyTensor class and a CPU device it is the reference's own fit on the host."""
    from polytensors_b200 import PolyTensor as Ours

    PolyTensor = poly_cls or Ours
    X, Y, Xp, Yp = (t.to(device) for t in data[:4])
    batches = [(i.to(device), j.to(device)) for i, j in data[4]]
    Z = PolyTensor((torch.tensor(0.0, device=device), 1.0), degree=degree)
    w = (torch.zeros(X.shape[1], device=device) + 0 * Z).requires_grad_()
    c = (torch.zeros((), device=device) + 0 * Z).requires_grad_()
    opt = torch.optim.SGD([w, c], lr=0.1, foreach=False)
    with PolyTensor.plain_range():
        for i, j in batches:
            opt.zero_grad(set_to_none=True)
            with PolyTensor.retain_wrappers():
                signal = (X[i] @ w + c - Y[i]).square().mean()
                noise = (Xp[j] @ w + c - Yp[j]).square().mean()
                loss = (signal + (1 - Z) * noise) / 2
                loss.backward()
                opt.step()
    return list(w.detach().coeffs), list(c.detach().coeffs)


def oracle_readme_fit(data, dtype, degree=5):
    """The same fit through the oracle restatement of the reference's plain-range rules on the
    CPU: series residuals, squares and means, the (1 - Z) weight, the series backward and the
    per-plane SGD update."""
    from oracle import polyref as R

    X, Y, Xp, Yp = (t.to(dtype) for t in data[:4])
    d, P = X.shape[1], degree + 1
    w = [torch.zeros(d, dtype=dtype) for _ in range(P)]
    c = [torch.zeros((), dtype=dtype) for _ in range(P)]
    one_minus_z = [torch.tensor(1.0, dtype=dtype), torch.tensor(-1.0, dtype=dtype)] + \
                  [torch.tensor(0.0, dtype=dtype)] * (P - 2)
    seed = [torch.tensor(1.0, dtype=dtype)] + [torch.tensor(0.0, dtype=dtype)] * degree

    def loss(i, j):
        def mse(Xs, Ys, ws, cs):
            r = [Xs @ wk + ck - (Ys if k == 0 else 0) for k, (wk, ck) in enumerate(zip(ws, cs))]
            return [q.mean() for q in R.cauchy(r, r)]
        return lambda ws, cs: [(a + b) / 2 for a, b in zip(mse(X[i], Y[i], ws, cs),
                                                           R.cauchy(one_minus_z, mse(Xp[j], Yp[j], ws, cs)))]

    for i, j in data[4]:
        gw, gc = R.series_vjp(loss(i, j), [w, c], seed)
        w = [a - 0.1 * g for a, g in zip(w, gw)]
        c = [a - 0.1 * g for a, g in zip(c, gc)]
    return w, c


def readme_fit_line(device, steps, warmup):
    """device time of the README fit (10 SGD steps) through the API, and its final
    w, c series against the float64 oracle (with the float32 oracle's own error beside it)."""
    from oracle import polyref as R

    data = readme_fit_data()
    for _ in range(max(1, warmup)):
        gw, gc = gpu_readme_fit(device, data)
    torch.cuda.synchronize(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(device)
    s.record(stream)
    for _ in range(steps):
        gw, gc = gpu_readme_fit(device, data)
    e.record(stream)
    torch.cuda.synchronize(device)
    ms = s.elapsed_time(e) / steps
    w64, c64 = oracle_readme_fit(data, torch.float64)
    t0 = time.perf_counter()
    w32, c32 = oracle_readme_fit(data, torch.float32)
    cpu_ms = (time.perf_counter() - t0) * 1e3
    cpu_kind, cpu_what = "port", "the whole fit through the oracle, float32"
    pt = _reference_package()
    if pt is not None:
        # the reference's own fit on host tensors (after an untimed first fit)
        gpu_readme_fit(torch.device("cpu"), data, poly_cls=pt.PolyTensor)
        t0 = time.perf_counter()
        gpu_readme_fit(torch.device("cpu"), data, poly_cls=pt.PolyTensor)
        cpu_ms = (time.perf_counter() - t0) * 1e3
        cpu_kind, cpu_what = "reference", "the whole fit through the reference's PolyTensor on host tensors, float32"
    worst, ok = 0.0, True
    for got, r32, want in ((gw, w32, w64), (gc, c32, c64)):
        for a, b in zip(R.plane_errors([x.cpu() for x in got], want), R.plane_errors(r32, want)):
            worst = max(worst, a)
            ok &= a <= max(1e-4, 3 * b)
    return {"metric": "README fit (configs[0]): 10 SGD steps of the degree-5 series regression, ms per fit",
            "value": ms, "unit": "ms", "higher_is_better": False, "steps": steps,
            "config": {"workload": "readme_fit n=64 d=3 degree 5 float32 SGD(lr=0.1) 10 steps, plain range"},
            "parity": {"max_plane_err": worst, "within_tolerance": bool(ok),
                       "tol": "per plane: err <= max(1e-4, 3 x the float32 oracle's err)",
                       "against": "oracle restatement of the fit, float64, CPU"},
            "cpu_baseline": {"value": cpu_ms, "unit": "ms", "cores": torch.get_num_threads(), "kind": cpu_kind,
                             "sample": cpu_what}}


def default_mode_line(device, steps, warmup, M=2048, n=4, sample_rows=1024):
    """§8(f)3: the series matrix product in the reference's default (extended-range) mode, i.e.
    outside plain_range(): float32 M x M x M, degree 4, each of the (n+1)(n+2)/2 products rescaled
    by its operands' largest exponents on the product kernel, sums kept as mantissa / exponent
    pairs.  Parity: against the reference's own default-mode product on the host (a row sample of
    A) and against the plain-range product; the CPU leg times that reference run."""
    from polytensors_b200 import PolyTensor
    from oracle import polyref as R

    A_host = make_series((M, M), n, 1, torch.float32)
    B_host = make_series((M, M), n, 2, torch.float32)
    a = PolyTensor(tuple(p.to(device) for p in A_host))
    b = PolyTensor(tuple(p.to(device) for p in B_host))
    ms, clocks = _timed(lambda: a @ b, steps, warmup, device, 1)
    c = a @ b
    with PolyTensor.plain_range():
        c_plain = a @ b
    vs_plain = max(R.plane_errors([x.cpu() for x in c.coeffs], [x.cpu().double() for x in c_plain.coeffs]))
    line = {"metric": f"default-mode poly-matmul coeff TFLOP/s (float32, M=N=K={M}, degree {n})",
            "value": matmul_flops(M, M, M, n) / (ms / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
            "steps": steps, "clocks": clocks,
            "config": {"workload": f"default-mode (extended-range) poly_matmul M=N=K={M} degree {n} float32"},
            "parity": {"vs_plain_range_product": vs_plain}}
    ref = _reference_package()
    if ref is not None:
        torch.set_num_threads(os.cpu_count() or 1)
        ra = ref.PolyTensor(tuple(p[:sample_rows] for p in A_host))
        rb = ref.PolyTensor(tuple(B_host))
        t0 = time.perf_counter()
        rc = ra @ rb
        dt = time.perf_counter() - t0
        err = R.plane_errors([x[:sample_rows].cpu().double() for x in c.coeffs], [x.double() for x in rc.coeffs])
        line["parity"].update({"max_plane_err": max(err), "tol": 1e-4, "within_tolerance": bool(max(err) <= 1e-4),
                               "against": "the reference's own default-mode product (its ScaledTensor rules), "
                                          f"CPU, rows 0..{sample_rows - 1} of A"})
        line["cpu_baseline"] = {"value": matmul_flops(sample_rows, M, M, n) / dt / 1e12, "unit": "TFLOP/s",
                                "cores": os.cpu_count() or 1, "kind": "reference",
                                "sample": f"{sample_rows} of {M} rows of A, the reference's default mode, "
                                          f"{dt:.1f} s"}
    return line


def run_train(args, rank, world, device):
    """configs[4] (the default workload): global batch 64 x seq 1024 sharded over the ranks,
    micro-batches of args.micro sequences per rank with gradient accumulation, one bucketed
    NCCL all-reduce of the gradient series, SGD(lr=0.1, foreach=False).  A timed step is the
    whole global batch (unless --micro-batches bounds it); value = tokens/s of the whole job.
    The configs[1] polynomial product is measured first on every rank and reported under
    ``poly_matmul``."""
    from polytensors_b200 import PolyTensor, _lib
    from polytensors_b200.parallel import OverlappedAllReduce

    threads = os.cpu_count() or 1
    extras = {}
    if not args.no_matmul:
        mm_args = argparse.Namespace(steps=min(args.steps, 10), warmup=max(args.warmup, 1))
        mm = run_matmul(mm_args, WORKLOADS["poly_matmul"], rank, world, device, parity=(rank == 0))
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            rate, desc, kind = cpu_matmul_rate(WORKLOADS["poly_matmul"], threads)
            mm["cpu_baseline"] = {"value": rate, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": desc}
        extras["poly_matmul"] = {k: mm.get(k) for k in ("metric", "value", "unit", "ms_per_step", "steps", "config",
                                                        "e2e", "roofline", "parity", "cpu_baseline", "gpu_launches",
                                                        "kernel_ms_per_launch", "clocks")}
        torch.cuda.empty_cache()
    if world == 1 and not args.no_extras:
        extras["readme_fit"] = readme_fit_line(device, min(args.steps, 5), args.warmup)
        extras["default_mode"] = default_mode_line(device, min(args.steps, 5), max(args.warmup, 2))
        torch.cuda.empty_cache()
        # configs[2] and configs[3] on the same GPU, a few steps each (per-op lines carried here so
        # that every config is measured in the default run)
        ns = argparse.Namespace(steps=min(args.steps, 3), warmup=2, rows=16384, seq=4096, batch=8,
                                no_cpu_baseline=args.no_cpu_baseline, dtype="bf16")
        keep = ("metric", "value", "unit", "ms_per_step", "steps", "config", "roofline", "kernels", "linear",
                "forward", "cpu_baseline", "clocks")
        keep = keep + ("peak_memory_gb", "fused_head")
        extras["norm_ce"] = {k: v for k, v in run_norm_ce(ns, rank, world, device).items() if k in keep}
        torch.cuda.empty_cache()
        ns.fused_head, ns.no_cpu_baseline = True, True
        extras["norm_ce_fused_head"] = {k: v for k, v in run_norm_ce(ns, rank, world, device).items()
                                        if k in keep and k != "cpu_baseline"}
        ns.fused_head, ns.no_cpu_baseline = False, args.no_cpu_baseline
        torch.cuda.empty_cache()
        for dt in ("bf16", "f32"):
            ns.dtype = dt
            extras[f"attention_{dt}"] = {k: v for k, v in run_attention(ns, rank, world, device).items() if k in keep}
            torch.cuda.empty_cache()

    parity = cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        parity, cpu = train_parity_and_cpu(args.layers, device, threads)

    seq, global_batch, n = 1024, 64, 3
    model = TinyGPT(device, transformer_init(layers=args.layers, seed=0), layers=args.layers)
    opt = torch.optim.SGD(model.parameters(), lr=0.1, foreach=False)
    Z = PolyTensor((torch.tensor(0.0, device=device), 1.0), degree=n)
    per_rank = global_batch // world
    g = torch.Generator().manual_seed(1234)
    ids_host = torch.randint(0, 32000, (global_batch, seq + 1), generator=g)[rank * per_rank:(rank + 1) * per_rank]
    ids_host = ids_host.contiguous().pin_memory()
    ids = ids_host.to(device)
    micro = min(args.micro, per_rank)
    n_micro = per_rank // micro if args.micro_batches <= 0 else min(args.micro_batches, per_rank // micro)
    stream = torch.cuda.current_stream(device)
    ar_events = []
    # gradient series averaged over the ranks in buckets launched from the gradient hooks of the last
    # micro-batch's backward (NCCL overlaps them with the remaining backward); finish() waits for
    # what is still in flight and unpacks
    reducer = OverlappedAllReduce(model.parameters()) if world > 1 else None

    def step(ids_dev, record_allreduce=False):
        opt.zero_grad(set_to_none=True)
        total = None
        with PolyTensor.plain_range():
            for m in range(n_micro):
                chunk = ids_dev[m * micro:(m + 1) * micro]
                if reducer is not None and m == n_micro - 1:
                    reducer.arm()
                with PolyTensor.retain_wrappers():
                    loss = model.loss(chunk[:, :-1], chunk[:, 1:], Z, 0.5) * (micro / per_rank)
                    loss.backward()
                    planes = torch.stack([c.detach() for c in loss.coeffs])
                    total = planes if total is None else total + planes
            if record_allreduce:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record(stream)
            if reducer is not None:
                reducer.finish()
            if record_allreduce:
                ev[1].record(stream)
                ar_events.append(ev)
            with PolyTensor.retain_wrappers():
                opt.step()
        return total

    for _ in range(args.warmup):
        step(ids)
    torch.cuda.synchronize(device)
    barrier(world)
    _lib.launch_count(reset=True)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clocks:
        torch.cuda.synchronize(device)
        barrier(world)
        start.record(stream)
        for _ in range(args.steps):
            last = step(ids, record_allreduce=True)
        end.record(stream)
        torch.cuda.synchronize(device)
        barrier(world)
    launches = _lib.launch_count()
    ms = max_over_ranks(start.elapsed_time(end) / args.steps, world, device)
    ar_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in ar_events) / len(ar_events), world, device)
    final_loss = [float(x) for x in last.cpu()]

    # end to end through the public API: every step copies the rank's token ids in from pinned
    # host memory and the loss series out to pinned host memory
    e2e_steps = min(args.steps, 5)
    loss_host = torch.empty(n + 1, dtype=torch.float32).pin_memory()
    dev_ids = torch.empty_like(ids)
    torch.cuda.synchronize(device)
    barrier(world)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(e2e_steps):
        dev_ids.copy_(ids_host, non_blocking=True)
        loss_host.copy_(step(dev_ids), non_blocking=True)
    e_end.record(stream)
    torch.cuda.synchronize(device)
    barrier(world)
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end) / e2e_steps, world, device)

    # device time per kernel family and the products' algorithmic flops over one more step, with
    # the library's launch timing on (outside the timed region: per-launch events perturb it)
    names = ("poly_gemm", "flash_attn_fwd", "attn_probs_gemm", "attn_dscores_gemm", "attn_probs", "attn_dscores",
             "rmsnorm_fwd", "rmsnorm_bwd", "series_map", "softmax_fwd", "softmax_bwd", "cross_entropy_fwd",
             "cross_entropy_bwd")
    for nm in names:
        _lib.profile_query(nm)
    _lib.take_gemm_flops()
    _lib.profile_enable(True)
    step(ids)
    torch.cuda.synchronize(device)
    _lib.profile_enable(False)
    gemm_flops = _lib.take_gemm_flops()
    breakdown = {}
    for nm in names:
        kt, kl = _lib.profile_query(nm)
        if kl:
            breakdown[nm] = {"ms_per_step": kt, "launches_per_step": kl}
    gemm_ms = breakdown.get("poly_gemm", {}).get("ms_per_step")
    pk, source = peaks()
    peak = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    achieved = gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms else None
    tokens = world * n_micro * micro * seq
    tps = tokens / (ms / 1e3)
    whole = n_micro * micro == per_rank
    result = {
        "metric": "train tokens/s (configs[4]: 12-layer d768 PolyTensor transformer, degree 3, float32, "
                  "global batch 64 x 1024)",
        "value": tps, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32 (polynomial products as bf16x3 splits on tcgen05, fp32 accumulate)",
        "data": "synthetic: uniform random token ids, random-init N(0,0.02) weights with zero higher coefficients",
        "config": train_config(args.layers),
        "parallelism": f"dp{world}", "micro_batch": micro, "micro_batches_per_rank": n_micro,
        "steps_per_s": 1e3 / ms if whole else None,
        "extrapolated_steps_per_s": tps / (global_batch * seq),
        "final_loss": final_loss,
        "allreduce": {"exposed_ms_per_step": ar_ms, "share_of_step": ar_ms / ms,
                      "buckets": len(reducer.buckets) if reducer is not None else 0,
                      "what": "gradient-series all-reduce (NCCL AVG) in buckets launched during the last "
                              "micro-batch's backward; exposed time = OverlappedAllReduce.finish() (wait for the "
                              "collectives still in flight + unpack) per step, CUDA events on the compute stream, "
                              "max over ranks"},
        "e2e": {"value": world * n_micro * micro * seq / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": ids_host.numel() * ids_host.element_size() * world,
                "d2h_bytes_per_step": (n + 1) * 4 * world, "ms_per_step": e2e_ms, "steps": e2e_steps,
                "api": "PolyTensor API (F.embedding / F.linear / F.rms_norm / SDPA / F.gelu / F.cross_entropy, "
                       "backward, SGD) with token ids copied in from pinned host memory and the loss series "
                       "copied out every step"},
        "roofline": {"bound": "tensor", "kernel": "polynomial products (tc_poly_gemm / tc_allplanes)",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak if achieved else None,
                     "traffic": _TRAIN_GEMM_BYTES_PER_FLOP * gemm_flops,
                     "traffic_unit": "DRAM bytes per step, all product launches (ncu capture of a reduced step "
                                     "scaled by algorithmic flops)",
                     "peak_source": f"bf16_tflops_sustained ({source}): a kernel timed inside a long step",
                     "device_ms_per_step": gemm_ms, "algorithmic_tflop_per_step": gemm_flops / 1e12,
                     "note": "algorithmic flops of the product launches as issued (float32 products execute "
                             "3 bf16 MMAs each)"},
        "step_tflops": gemm_flops / (ms / 1e3) / 1e12,
        "gpu_launches": launches,
        "gpu_launches_per_step": launches / args.steps,
        "kernels": breakdown,
        "parity": parity,
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
    }
    result.update(extras)
    return result


def _reference_package():
    """The reference package (samuel-gunn/poly-tensors) pip-installed into baseline/_ref."""
    import importlib

    path = ROOT / "baseline" / "_ref"
    if not (path / "polytensors").is_dir():
        return None
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))
    return importlib.import_module("polytensors")


def run_degree1(args, rank, world, device):
    """Same-box bar: the reference's degree-1 Triton kernels (its fused attention, cross entropy,
    RMSNorm and activation gates, through its own PolyTensor API inside plain_range()) against the
    pk:: kernels through this package's API, forward + backward, same inputs; per op the device
    time per step of both and the largest plane difference between their results."""
    import torch.nn.functional as F
    from polytensors_b200 import PolyTensor as Ours

    ref = _reference_package()
    if ref is None:
        return {"metric": "degree-1 pk:: vs reference Triton", "unavailable": "baseline/_ref is not installed"}
    Ref = ref.PolyTensor
    g = torch.Generator(device=device).manual_seed(5)

    def planes(shape, dtype):
        return tuple(torch.randn(*shape, generator=g, device=device, dtype=torch.float32).to(dtype) for _ in range(2))

    cases = {
        "attention_bf16_D128": ([(4, 16, 2048, 128)] * 3, torch.bfloat16,
                                lambda q, k, v: F.scaled_dot_product_attention(q, k, v, is_causal=True)),
        "attention_bf16_D64": ([(4, 16, 2048, 64)] * 3, torch.bfloat16,
                               lambda q, k, v: F.scaled_dot_product_attention(q, k, v, is_causal=True)),
        "cross_entropy_softcap_V32000": ([(8192, 32000)], torch.float32, None),
        "rms_norm_4096": ([(16384, 4096)], torch.float32, lambda x: F.rms_norm(x, (4096,))),
        "gelu": ([(16384, 4096)], torch.float32, lambda x: F.gelu(x)),
    }
    target = torch.randint(0, 32000, (8192,), generator=g, device=device)
    out = {}
    for name, (shapes, dtype, fn) in cases.items():
        data = [planes(sh, dtype) for sh in shapes]
        grad_seed = planes(shapes[0], dtype) if fn is not None else None
        res = {}
        for impl, P in (("reference_triton", Ref), ("polykern", Ours)):
            xs = [P(d, requires_grad=True) for d in data]

            def step(P=P, xs=xs):
                for x in xs:
                    x.grad = None
                with P.plain_range(), P.retain_wrappers():
                    if fn is None:
                        y = P.cross_entropy(xs[0], target, softcap=30.0)
                        y.backward()
                    else:
                        y = fn(*xs)
                        y.backward(P(grad_seed))
                    return [c.detach() for c in y.coeffs], [c.detach() for c in xs[0].grad.coeffs]
            try:
                for _ in range(max(args.warmup, 2)):
                    step()
                ms, _ = _timed(step, max(3, min(args.steps, 10)), 0, device, world)
                res[impl] = {"ms_per_step": ms, "result": step()}
            except Exception as e:   # noqa: BLE001  (a reference path that does not run here is reported)
                res[impl] = {"error": f"{type(e).__name__}: {e}"[:300]}
        entry = {k: {kk: vv for kk, vv in v.items() if kk != "result"} for k, v in res.items()}
        if all("result" in v for v in res.values()):
            diffs = []
            for a, b in zip(sum(res["polykern"]["result"], []), sum(res["reference_triton"]["result"], [])):
                a, b = a.double(), b.double()
                diffs.append(((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item())
            entry["max_plane_diff"] = max(diffs)
            entry["speedup"] = res["reference_triton"]["ms_per_step"] / res["polykern"]["ms_per_step"]
        out[name] = entry
        torch.cuda.empty_cache()
    # kernel level for the activation: the reference's Triton kernel through its gate function
    # (src/polytensors/_fused_activation.py:5-24, forward and backward) against pk_series_map
    from importlib import import_module

    from polytensors_b200 import _kernels as K

    act = import_module(f"{ref.__name__}._fused_activation")
    X = planes((16384, 4096), torch.float32)
    Gs = planes((16384, 4096), torch.float32)
    kern = {}
    for impl, fwd, bwd in (("reference_triton", lambda: act.maybe_activation(X, "gelu"),
                            lambda: act.maybe_activation(X, "gelu", Gs)),
                           ("polykern", lambda: K.series_map("gelu", 1, list(X)),
                            lambda: K.series_map("gelu_bwd", 1, list(Gs), list(X)))):
        step = lambda fwd=fwd, bwd=bwd: (fwd(), bwd())   # noqa: E731
        for _ in range(3):
            step()
        ms, _ = _timed(step, 10, 0, device, world)
        kern[impl] = {"ms_per_step": ms, "GB/s": 2 * 4 * 16384 * 4096 * (2 + 3) / (ms / 1e3) / 1e9}
    kern["speedup"] = kern["reference_triton"]["ms_per_step"] / kern["polykern"]["ms_per_step"]
    out["gelu_kernels_fwd_bwd"] = kern
    return {"metric": "degree-1 forward+backward ms per step: pk:: kernels vs the reference's Triton kernels "
                      "(same B200, each through its own PolyTensor API in plain_range; gelu_kernels_fwd_bwd: the "
                      "activation kernels called directly)",
            "value": None, "unit": "ms", "n_gpus": world, "ops": out}


def run_matmul_sweep(args, rank, world, device):
    """every size / degree / dtype point, one line per point in 'sweep'."""
    from polytensors_b200 import _kernels

    points = []
    for dtype in ("float32", "float64"):
        for N in (1024, 4096, 8192):
            for n in (2, 4, 8):
                if dtype == "float64" and N == 8192 and n == 8 and not args.full_sweep:
                    continue
                points.append((dtype, N, n))
    points.append(("complex128", 4096, 2))
    out = []
    for dtype, N, n in points:
        if dtype == "complex128":
            A = [torch.randn(N, N, dtype=torch.float64, device=device)] + \
                [torch.complex(torch.randn(N, N, dtype=torch.float64, device=device),
                               torch.randn(N, N, dtype=torch.float64, device=device)) / math.factorial(k)
                 for k in range(1, n + 1)]
            B = [a.clone() for a in A]
            T = 1 + 4 * n + 4 * ((n + 1) * (n + 2) // 2 - 1 - 2 * n)
            flops = 2.0 * N ** 3 * T
        else:
            dt = getattr(torch, dtype)
            A = [t.to(device) for t in make_series((N, N), n, 1, dt)]
            B = [t.to(device) for t in make_series((N, N), n, 2, dt)]
            flops = matmul_flops(N, N, N, n)
        steps = max(1, min(args.steps, int(2e14 // flops) or 1))
        ms, _ = _timed(lambda: _kernels.poly_matmul(A, B), steps, 1, device, world)
        out.append({"dtype": dtype, "M=N=K": N, "degree": n, "ms": ms,
                    "coeff_TFLOP/s": flops / (ms / 1e3) / 1e12})
        del A, B
        torch.cuda.empty_cache()
    return {"metric": "poly-matmul coeff TFLOP/s sweep (configs[1])", "value": None, "unit": "TFLOP/s",
            "n_gpus": world, "sweep": out, "higher_is_better": True}


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
    """--impl reference for the poly_matmul workload: the reference's own plain-range product (the
    oracle restatement of plain_polynomial_product without its package) on all host cores over
    bounded row samples of the same config."""
    threads = os.cpu_count() or 1
    samples, desc, kind = [], "", "port"
    if args.warmup:
        cpu_matmul_rate(cfg, threads, target_s=2.0)
    for _ in range(args.steps):
        rate, desc, kind = cpu_matmul_rate(cfg, threads, target_s=8.0)
        samples.append(rate)
    value = statistics.median(samples)
    M, n = cfg["M"], cfg["degree"]
    return {
        "impl": "reference",
        "metric": f"poly-matmul coeff TFLOP/s ({cfg['dtype']}, M=N=K={M}, degree {n})",
        "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": cfg["dtype"],
        "data": "synthetic: planes N(0,1)/k!, seeded",
        "config": matmul_config(cfg),
        "parallelism": "host CPU",
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": desc},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def reference_arm_train(args, budget_s=150.0):
    """--impl reference for the default (configs[4] training) workload: the reference's own CPU
    implementation (its PolyTensor from baseline/_ref on host tensors, the same model code) for the
    full-width model's forward and backward on the host cores, each step a bounded sample of
    4 x 256 tokens; without the package, the oracle restatement of its plain-range rules.  Steps
    beyond a ~150 s budget are not run (the count is reported)."""
    threads = os.cpu_count() or 1
    init = transformer_init(layers=args.layers, seed=0)
    ids = train_sample_ids(4, 256)
    use_ref = _reference_package() is not None

    def one():
        if use_ref:
            return reference_train_sample(init, ids, args.layers, threads)
        return oracle_train_sample(init, ids, args.layers, torch.float32, threads)[0]

    for _ in range(min(args.warmup, 1)):
        one()
    rates, used = [], 0.0
    for _ in range(args.steps):
        dt = one()
        rates.append(ids[:, 1:].numel() / dt)
        used += dt
        if used > budget_s:
            break
    value = statistics.median(rates)
    what = ("the reference's PolyTensor (baseline/_ref) forward + backward on host tensors" if use_ref
            else "oracle forward + series backward")
    sample = (f"{what} of the full-width model ({args.layers} layers), 4 x 256 tokens per step, float32, "
              f"{len(rates)} of {args.steps} steps run")
    return {
        "impl": "reference",
        "metric": "train tokens/s (configs[4]: 12-layer d768 PolyTensor transformer, degree 3, float32, "
                  "global batch 64 x 1024)",
        "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": len(rates), "warmup": args.warmup,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: uniform random token ids, random-init N(0,0.02) weights with zero higher coefficients",
        "config": train_config(args.layers),
        "parallelism": "host CPU",
        "extrapolated_s_per_step": 64 * 1024 / value,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference" if use_ref else "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="train",
                    choices=sorted(WORKLOADS) + ["norm_ce", "attention", "attention_fwd", "train",
                                                 "poly_matmul_sweep", "degree1", "default_mode"])
    ap.add_argument("--no-matmul", action="store_true", help="train: skip the configs[1] product line")
    ap.add_argument("--no-extras", action="store_true", help="train: skip the configs[2] / configs[3] lines")
    ap.add_argument("--impl", default="polykern", choices=["polykern", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rows", type=int, default=16384, help="norm_ce: rows (batch*seq)")
    ap.add_argument("--seq", type=int, default=4096, help="attention: sequence length")
    ap.add_argument("--batch", type=int, default=8, help="attention / attention_fwd: batch")
    ap.add_argument("--dtype", default="f32", choices=["f32", "bf16"], help="attention: storage dtype")
    ap.add_argument("--heads", type=int, default=32, help="attention: heads")
    ap.add_argument("--head-dim", type=int, default=128, help="attention: head dimension")
    ap.add_argument("--layers", type=int, default=12, help="train: transformer layers")
    ap.add_argument("--micro", type=int, default=8, help="train: sequences per micro-batch")
    ap.add_argument("--micro-batches", type=int, default=0,
                    help="train: micro-batches per rank and step (0 = the whole global batch)")
    ap.add_argument("--full-sweep", action="store_true")
    ap.add_argument("--fused-head", action="store_true",
                    help="norm_ce: linear + cross entropy through PolyTensor.linear_cross_entropy (chunked logits)")
    args = ap.parse_args()
    cfg = WORKLOADS.get(args.workload)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        # the reference's CPU path on the host cores; under torchrun rank 0 alone runs it
        if rank == 0:
            if args.workload == "train":
                print(json.dumps(reference_arm_train(args)), flush=True)
            elif cfg is not None:
                print(json.dumps(reference_arm(args, cfg)), flush=True)
            else:
                print(json.dumps({"impl": "reference", "unavailable": f"--impl reference covers the train and "
                                  f"poly_matmul workloads, not {args.workload}"}), flush=True)
        return

    if args.warmup < 3:
        print("note: fewer than 3 warm-up steps", file=sys.stderr)
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)
    secondary = {"norm_ce": run_norm_ce, "attention": run_attention, "attention_fwd": run_attention_fwd,
                 "train": run_train, "degree1": run_degree1,
                 "poly_matmul_sweep": run_matmul_sweep,
                 "default_mode": lambda a, r, w, d: default_mode_line(d, a.steps, max(a.warmup, 2))}
    if args.workload in secondary:
        result = secondary[args.workload](args, rank, world, device)
        if rank == 0:
            print(json.dumps(result), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    result = run_matmul(args, cfg, rank, world, device, parity=(rank == 0))
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, desc, kind = cpu_matmul_rate(cfg, os.cpu_count() or 1)
        result["cpu_baseline"] = {"value": rate, "unit": "TFLOP/s", "cores": os.cpu_count() or 1,
                                  "kind": kind, "sample": desc}
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
