"""Benchmark of the B200 FP64-on-INT8 (Ozaki-II / CRT) GEMM: emulated FP64 TFLOPS = 2 M N K / t.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c3] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (the driver's multi-GPU launch)

One step = one call of the drop-in entry point ``OzakiCRT.run(A, B, C, graph=True)`` (statistics, the device rule,
the host read of (N, p), residue split, the N INT8 tensor-core products with the fused reduction, reconstruction)
on inputs resident in HBM.  Default workload: the metric's n = 16384 configuration (c3: M = N = K = 16384, entries
(U - 0.5) exp(2 N(0,1)), seed 0, dynamic plane rule).  With --gpus N > 1 the same product is split into an R x S
grid of C blocks, one per rank (DistributedOzakiCRT: S = 2 from 4 ranks on, else row blocks; strong scaling).

Printed (rank 0, one JSON line): value (device time, max over ranks), e2e (the same call from pinned host buffers,
H2D + D2H inside the timed region), roofline of the INT8 product kernel (live CUDA-event time of its launches), the
CPU baseline (the C/OpenMP port of the reference's algorithm on a bounded sample), clocks sampled by nvidia-smi during
the timed region, and the count of this library's kernel launches.

``--impl reference`` times the reference's algorithm on the host cores instead (the CPU port in oracle/, all
threads), on a bounded sample of the same workload, and prints the same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import __graft_entry__  # noqa: E402

METRIC = "emulated FP64 GEMM TFLOPS (2MNK/t) at n=16384, 1-8 B200; max rel error"
# DRAM bytes (read + write) of one gemm_tc_kernel launch on one GPU, from one-pass ncu captures of this bench's own
# command (profiles/dram_traffic_c3_n16384.md); workloads without a capture report null
GEMM_TRAFFIC_BYTES = {"c3": 66.9e9 + 4.8e9, "c2": 537.7e6 + 242.9e6}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="c3")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=6)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-accuracy", action="store_true")
    ap.add_argument("--cpu-sample", type=int, default=0, help="rows = cols of the CPU sample block (0: auto)")
    ap.add_argument("--mode", default="sampled", choices=["sampled", "certified", "config", "persist", "chain"],
                    help="sampled: the reference's timed path (default); certified: the plane count from the "
                         "full-matrix certificate; config: the single-graph path with (N, p) given (the sampled "
                         "rule's choice); persist: PersistA, A encoded once per step and --q products")
    ap.add_argument("--q", type=int, default=4, help="products per step in --mode persist")
    ap.add_argument("--planes", type=int, default=0, help="force the plane count N (0: the workload's rule)")
    return ap.parse_args()


# ------------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, path: str | None):
        self.gpu = gpu_index
        self.path = path
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.path:
            with open(self.path, "w") as f:
                f.write(self.FIELDS + "\n" + "\n".join(self.lines) + "\n")

    def summary(self):
        sm, mx, pw, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
                pw.append(float(f[3]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(mx)), "power_w_max": float(max(pw)),
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------------ peaks
def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


def int8_peak_tops(torch, dev):
    """Dense INT8 tensor throughput of cuBLASLt (torch._int_mm, 8192^3, best of 10) on this GPU, in TOPS."""
    n = 8192
    a = torch.randint(-128, 127, (n, n), dtype=torch.int8, device=dev)
    b = torch.randint(-128, 127, (n, n), dtype=torch.int8, device=dev).t()
    for _ in range(3):
        torch._int_mm(a, b)
    best = 1e9
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1) / 1e3)
    del a, b
    return 2 * n ** 3 / best / 1e12


# ------------------------------------------------------------------------------------------------ CPU baseline
def cpu_baseline(pkg, A_host, B_host, N, sample, phi):
    """The CPU port of the reference's algorithm (oracle/, C + OpenMP, all host threads) on a sample block of the same
    workload: rows [0, s) of A and columns [0, s) of B with the full K, N planes forced to the GPU run's N."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # noqa: E402  (timed CPU baseline; not part of the product path)
    oracle.build()
    As = np.ascontiguousarray(A_host[:sample])
    Bs = np.ascontiguousarray(B_host[:, :sample])
    oracle.run(As[:8], Bs[:, :32], force_N=N)       # warm the thread pool
    t0 = time.perf_counter()
    C, info = oracle.run(As, Bs, force_N=N)
    t = time.perf_counter() - t0
    k = As.shape[1]
    return {"value": 2.0 * sample * sample * k / t / 1e12, "unit": "TFLOPS", "cores": oracle.num_threads(),
            "kind": "port", "seconds": t,
            "sample": f"rows 0..{sample} of A x columns 0..{sample} of B, full K={k}, N={N} forced, phi={phi}; "
                      "stats + split + exact INT8 products + CRT reconstruction"}


def auto_sample(k, N, threads):
    # about 10-15 s of CPU work: the port's int8 products ran at ~7.7 G MAC/s per thread on the GPU boxes' host cores
    macs = 12.0 * 7.0e9 * max(1, threads)
    s = int((macs / (k * N)) ** 0.5)
    return max(32, min(2048, (s // 32) * 32))


# ------------------------------------------------------------------------------------------------ reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    pkg = __graft_entry__.load_package()
    m, k, n, phi, alt, forceN, desc = pkg.CONFIGS[args.workload]
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # noqa: E402
    oracle.build()
    threads = oracle.num_threads()
    N = forceN or {"c1": 16, "c2": 16, "c3": 19, "c4": 16}.get(args.workload, 16)
    s = args.cpu_sample or auto_sample(k, N, threads) // 2
    # the sample block of the workload: the same generator, only the rows / columns that are used
    A, B = pkg.make_inputs(m if m * k <= (1 << 28) else s, k, n if k * n <= (1 << 28) else s, phi, 0, alt)
    As, Bs = np.ascontiguousarray(A[:s]), np.ascontiguousarray(B[:, :s])
    times = []
    for it in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        oracle.run(As, Bs, force_N=N)
        dt = time.perf_counter() - t0
        if it >= args.warmup:
            times.append(dt)
    t = float(np.mean(times))
    v = 2.0 * s * s * k / t / 1e12
    line = {"metric": METRIC, "value": v, "unit": "TFLOPS", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64 (int8 residue arithmetic)", "data": "synthetic", "impl": "reference",
            "config": {"workload": args.workload, "desc": desc, "m": m, "n": n, "k": k, "planes": N},
            "cpu_baseline": {"value": v, "unit": "TFLOPS", "cores": threads, "kind": "port",
                             "sample": f"rows 0..{s} x cols 0..{s} of the {args.workload} product, full K={k}, N={N}"},
            "e2e": {"value": v, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------ residue chain
def bench_chain(args):
    """--mode chain (single GPU): an exact integer chain A_1 A_2 A_3 of the workload's square size n with 8-bit
    entries, kept in INT8 residue form between the products (matrix_numbers_b200.chain); the plane count is the
    reference model's fixed base for R = H^3 n^2, H = 255.  Metric: exact integer TOPS = 2 n^3 (q - 1) / t."""
    import torch
    pkg = __graft_entry__.load_package()
    torch.cuda.set_device(0)
    _, _, n, _, _, _, desc = pkg.CONFIGS[args.workload]
    q, b = 3, 8
    rs = np.random.RandomState(0)
    mats = [torch.from_numpy(rs.randint(-255, 256, size=(n, n)).astype(np.float64)).cuda() for _ in range(q)]
    ch = pkg.ResidueChain()
    for _ in range(args.warmup):
        _, info = ch.product(mats, b=b)
    torch.cuda.synchronize()
    l0 = ch.launches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0, None) as clocks:
        time.sleep(0.3)
        e0.record()
        for _ in range(args.steps):
            _, info = ch.product(mats, b=b)
        e1.record()
        torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / args.steps
    ops = 2.0 * n ** 3 * (q - 1)
    peak = int8_peak_tops(torch, torch.device("cuda", 0))
    int8_ops = ops * info["N"]
    print(json.dumps({"metric": f"exact integer chain TOPS (A1 A2 A3, {b}-bit entries, residue form)",
                      "value": ops / t / 1e12, "unit": "TOPS", "n_gpus": 1, "steps": args.steps,
                      "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "strong",
                      "vs_baseline": None, "dtype": "int8 residues", "data": "synthetic",
                      "config": {"workload": args.workload, "n": n, "q": q, "bits": b, "planes": info["N"],
                                 "gemms_per_step": info["gemms"], "mode": "chain"},
                      "roofline": {"bound": "tensor", "achieved": int8_ops / t / 1e12, "peak": peak,
                                   "unit": "TOPS (INT8, whole chain incl. splits and reconstruction)",
                                   "frac": int8_ops / t / 1e12 / peak, "traffic": None},
                      "clocks": clocks.summary(), "gpu_launches": ch.launches - l0}), flush=True)


# ------------------------------------------------------------------------------------------------ our arm
def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.mode == "chain":
        bench_chain(args)
        return
    import torch
    import torch.distributed as dist

    pkg = __graft_entry__.load_package()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    m, k, n, phi, alt, forceN, desc = pkg.CONFIGS[args.workload]
    if args.planes:
        forceN = args.planes

    # inputs: generated on the host (numpy, seed 0); rank a S + b of the R x S grid holds A's row block a and B's
    # column block b (R = world, S = 1 for a plain row split)
    t_gen = time.perf_counter()
    A_host, B_host = pkg.make_inputs(m, k, n, phi, 0, alt)
    from matrix_numbers_b200.distributed import default_grid
    R, S = default_grid(world) if world > 1 else (1, 1)
    ga, gb = divmod(rank, S)
    rows, cols = m // R, n // S
    assert rows % 4 == 0 and cols % 32 == 0, "block shape rule"
    r0, c0 = ga * rows, gb * cols
    A_blk = A_host[r0:r0 + rows]
    B_blk = np.ascontiguousarray(B_host[:, c0:c0 + cols]) if S > 1 else B_host
    A = torch.from_numpy(A_blk).to(dev)
    B = torch.from_numpy(B_blk).to(dev)
    C = torch.empty((rows, cols), dtype=torch.float64, device=dev)
    t_gen = time.perf_counter() - t_gen

    step_events = []
    products = 1
    if world > 1:
        assert args.mode in ("sampled", "certified"), "--mode config / persist are single-GPU"
        E = pkg.DistributedOzakiCRT(grid=(R, S))
        cert = args.mode == "certified"
        call = lambda ev=None: E.run(A, B, C, force_N=forceN, certify=cert)  # noqa: E731
    else:
        E = pkg.OzakiCRT()
        call = lambda ev=None: E.run_fast(A, B, C, force_N=forceN, events=ev)  # noqa: E731
        if args.mode == "certified":
            call = lambda ev=None: E.run_fast(A, B, C, events=ev, certify=True)  # noqa: E731
        elif args.mode == "config":
            _, i0 = E.run_fast(A, B, C, force_N=forceN)
            cfg_N, cfg_p = i0["N"], i0["p"]
            call = lambda ev=None: E.run_fast(A, B, C, force_N=cfg_N, force_p=cfg_p, events=ev)  # noqa: E731
        elif args.mode == "persist":
            PA = pkg.PersistA(E, A, B, n)
            products = args.q

            def call(ev=None):
                PA.encode()
                for _ in range(args.q):
                    PA.product(B, C)
                return C, {"N": PA.N, "p": PA.p}

    for _ in range(args.warmup):
        _, info = call()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches0 = E.launches
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk_path = os.path.join(ROOT, "gpurun_out", f"clocks_rank{rank}.csv") if os.path.isdir(os.path.join(ROOT, "gpurun_out")) else None
    with ClockSampler(local, clk_path) as clocks:
        time.sleep(0.3)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0.record(stream)
        for _ in range(args.steps):
            ev = [] if world == 1 else None
            _, info = call(ev)
            if ev:
                step_events.append(ev)
        e1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    t_dev = e0.elapsed_time(e1) / 1e3 / args.steps
    launches = E.launches - launches0
    if world > 1:
        tt = torch.tensor([t_dev], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_dev = float(tt.item())
    flops = 2.0 * m * n * k * products
    value = flops / t_dev / 1e12

    # stage times inside the timed calls (CUDA events between the parts of run_fast)
    in_step = {}
    for ev in step_events:
        for (n0, a), (n1, b_) in zip(ev[:-1], ev[1:]):
            in_step[n1] = in_step.get(n1, 0.0) + a.elapsed_time(b_) / len(step_events)

    # roofline of the dominant kernel (the INT8 products with the fused reduction): live CUDA-event time per launch
    Nplanes = info.get("N") or forceN
    prof = {}
    engine = E.engine if world > 1 else E
    b = engine.buffers(rows, cols, k, Nplanes)
    for _ in range(3):
        engine.core(A, B, b, Nplanes, C, prof=prof)
    t_gemm = prof["gemm+reduce"] / 3
    int8_ops = 2.0 * Nplanes * rows * cols * k
    peak_int8 = int8_peak_tops(torch, dev)
    hbm_peak, bf16_peak, peak_src = measured_peaks()
    achieved = int8_ops / t_gemm / 1e12
    roofline = {"bound": "tensor", "kernel": "gemm_tc_kernel<residue> (tcgen05.mma kind::i8)", "achieved": achieved,
                "peak": peak_int8, "unit": "TOPS (INT8)", "frac": achieved / peak_int8,
                "peak_source": "cuBLASLt INT8 GEMM 8192^3 burst measured in this run (torch._int_mm)",
                "bf16_measured_tflops_x2": 2 * bf16_peak, "frac_of_2x_bf16": achieved / (2 * bf16_peak),
                "traffic": GEMM_TRAFFIC_BYTES.get(args.workload) if world == 1 and args.mode == "sampled" else None,
                "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
                "algorithmic_ops_per_launch": int8_ops, "ms_per_launch": t_gemm * 1e3,
                "stages_ms": {k_: v * 1e3 / 3 for k_, v in prof.items()}, "timed_call_stages_ms": in_step}
    # the emulated-FP64 ceiling is the INT8 rate over the plane count (one INT8 product per plane); the residue split
    # moves (8 + N)(rows k + k cols) bytes (FP64 in, N planes out) against the measured copy bandwidth
    t_split = prof["residues"] / 3
    split_bytes = (8.0 + Nplanes) * (rows * k + k * cols)
    roofline["emulated_ceiling_tflops"] = peak_int8 / Nplanes
    roofline["frac_of_int8_over_N"] = (2.0 * rows * cols * k / (t_dev / products) / 1e12) / (peak_int8 / Nplanes)
    roofline["split"] = {"bound": "hbm", "achieved": split_bytes / t_split / 1e9, "peak": hbm_peak, "unit": "GB/s",
                         "frac": split_bytes / t_split / 1e9 / hbm_peak, "bytes_per_call": split_bytes}

    # accuracy on a sample (rank 0's block): E1 / E2 against the correctly rounded product, native DGEMM beside it
    acc = None
    if rank == 0 and not args.no_accuracy:
        Cn = A @ B
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        torch.matmul(A, B, out=Cn)
        t1.record()
        torch.cuda.synchronize()
        t_nat = t0.elapsed_time(t1) / 1e3
        Smp = pkg.Sample(A, B, Cn, nr=24, nc=24)
        acc = {"engine": Smp.errors(C), "native_dgemm": Smp.errors(Cn),
               "native_dgemm_tflops": 2.0 * rows * cols * k / t_nat / 1e12}
        del Cn

    # end to end through the public API with host buffers (pinned), H2D + D2H inside the timed region
    e2e = None
    if args.e2e_steps > 0:
        Ah = torch.from_numpy(A_blk).pin_memory()
        Bh = torch.from_numpy(B_blk).pin_memory()
        Ch = torch.empty((rows, cols), dtype=torch.float64).pin_memory()
        call()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        host_api = world == 1 and args.mode == "sampled"
        if host_api:
            E.run_host(Ah, Bh, Ch, force_N=forceN)          # warm-up of the host-buffer path
            torch.cuda.synchronize()
        f0.record(stream)
        for _ in range(args.e2e_steps):
            if host_api:
                # the public host-buffer call: H2D of A and B, the product, D2H of C overlapped block by block
                E.run_host(Ah, Bh, Ch, force_N=forceN)
            else:
                A.copy_(Ah, non_blocking=True)
                B.copy_(Bh, non_blocking=True)
                call()
                Ch.copy_(C, non_blocking=True)
        f1.record(stream)
        torch.cuda.synchronize()
        t_e2e = f0.elapsed_time(f1) / 1e3 / args.e2e_steps
        if world > 1:
            tt = torch.tensor([t_e2e], dtype=torch.float64, device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t_e2e = float(tt.item())
        e2e = {"value": flops / t_e2e / 1e12, "unit": "TFLOPS", "ms_per_step": t_e2e * 1e3,
               "api": "OzakiCRT.run_host (host buffers)" if host_api else "device run between host copies",
               "h2d_bytes_per_step": (Ah.numel() + Bh.numel()) * 8 * world, "d2h_bytes_per_step": Ch.numel() * 8 * world}
        if world > 1:
            # the same stream of products through DistributedOzakiCRT.run_host_many on every rank
            cert = args.mode == "certified"
            E.run_host_many([(Ah, Bh, Ch)] * 2, force_N=forceN, certify=cert)
            torch.cuda.synchronize()
            dist.barrier()
            f0.record(stream)
            E.run_host_many([(Ah, Bh, Ch)] * args.e2e_steps, force_N=forceN, certify=cert)
            f1.record(stream)
            torch.cuda.synchronize()
            tt = torch.tensor([f0.elapsed_time(f1) / 1e3 / args.e2e_steps], dtype=torch.float64, device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t_many = float(tt.item())
            e2e_single = e2e
            e2e = {"value": flops / t_many / 1e12, "unit": "TFLOPS", "ms_per_step": t_many * 1e3,
                   "api": f"DistributedOzakiCRT.run_host_many ({args.e2e_steps} products per rank; each step's H2D of "
                          "the rank's blocks, product and D2H of its C block inside the timed region, the next step's "
                          "H2D overlapped with this step's product)",
                   "h2d_bytes_per_step": e2e_single["h2d_bytes_per_step"],
                   "d2h_bytes_per_step": e2e_single["d2h_bytes_per_step"], "single_call": e2e_single}
        if host_api:
            # a stream of e2e_steps products through OzakiCRT.run_host_many: every step still copies its A and B in
            # and its C out, but the next step's H2D runs while this step computes (the pipeline fill is included)
            E.run_host_many([(Ah, Bh, Ch)] * 2, force_N=forceN)   # warm-up of the second slot
            torch.cuda.synchronize()
            f0.record(stream)
            E.run_host_many([(Ah, Bh, Ch)] * args.e2e_steps, force_N=forceN)
            f1.record(stream)
            torch.cuda.synchronize()
            t_many = f0.elapsed_time(f1) / 1e3 / args.e2e_steps
            e2e_single = e2e
            e2e = {"value": flops / t_many / 1e12, "unit": "TFLOPS", "ms_per_step": t_many * 1e3,
                   "api": f"OzakiCRT.run_host_many (host buffers, {args.e2e_steps} products; each step's H2D, product "
                          "and D2H inside the timed region, the next step's H2D overlapped with this step's product)",
                   "h2d_bytes_per_step": e2e_single["h2d_bytes_per_step"],
                   "d2h_bytes_per_step": e2e_single["d2h_bytes_per_step"], "single_call": e2e_single}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle  # noqa: E402
        s = args.cpu_sample or auto_sample(k, Nplanes, oracle.num_threads())
        cpu = cpu_baseline(pkg, A_host, B_host, Nplanes, s, phi)

    if world > 1:
        dist.barrier()
    if rank == 0:
        metric = METRIC if args.mode == "sampled" else METRIC + f" [{args.mode} mode]"
        line = {"metric": metric, "value": value, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": t_dev * 1e3, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f64 (int8 residue arithmetic)", "data": "synthetic",
                "config": {"workload": args.workload, "desc": desc, "m": m, "n": n, "k": k, "phi": phi,
                           "planes": Nplanes, "p": info.get("p"), "mode": args.mode, "products_per_step": products,
                           "parallelism": f"{R} x {S} grid of C blocks" if world > 1 else "single GPU",
                           "l2": "inputs larger than L2 (2 x 2.1 GB fp64)", "input_generation_s": t_gen},
                "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "accuracy": acc, "clocks": clocks.summary(),
                "gpu_launches": launches, "hbm_peak_gbs": hbm_peak, "peaks": peak_src}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
