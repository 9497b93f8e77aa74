"""Benchmark of the B200 FP64-on-INT8 (Ozaki-II / CRT) GEMM: emulated FP64 TFLOPS = 2 M N K / t.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c3] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (the driver's multi-GPU launch)

One step = one call of the drop-in entry point ``OzakiCRT.run(A, B, C, graph=True)`` (statistics, the device rule,
the host read of (N, p), residue split, the N INT8 tensor-core products with the fused reduction, reconstruction)
on inputs resident in HBM.  Default workload: the metric's n = 16384 configuration (c3: M = N = K = 16384, entries
(U - 0.5) exp(2 N(0,1)), seed 0, dynamic plane rule).  With --gpus N > 1 the same product is split into an R x S
grid of C blocks, one per rank (DistributedOzakiCRT: S = 2 from 4 ranks on, else row blocks; strong scaling).

Printed (rank 0, one JSON line): value (device time, max over ranks), e2e (the same product from pinned host
buffers, H2D + D2H inside the timed region: OzakiCRT.run_host_many on one GPU, DistributedOzakiCRT.run_host_many
with each rank loading its share of the operands on N), roofline of the INT8 product kernel (live CUDA-event
time of its launches), the CPU baseline (the C/OpenMP port of the reference's algorithm on a bounded sample),
clocks sampled by nvidia-smi during the timed region, and the count of this library's kernel launches.

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
# DRAM bytes (read + write) of one gemm_tc_kernel launch on one GPU: constants from one-pass ncu captures
# (dram__bytes_read.sum + dram__bytes_write.sum) of this bench's own command at the named workload; other workloads
# report null.  They are not measured by the bench run itself ("traffic_source" in the JSON line says so).
GEMM_TRAFFIC_BYTES = {"c3": 66.9e9 + 4.8e9, "c2": 537.7e6 + 242.9e6}
GEMM_TRAFFIC_SOURCE = "constant from a one-pass ncu capture of `bench.py --workload {w}` (not measured in this run)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="c3")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=-1,
                    help="products in the end-to-end stream from host buffers (default: max(6, --steps); 0: skip)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-accuracy", action="store_true")
    ap.add_argument("--cpu-sample", type=int, default=0, help="rows = cols of the CPU sample block (0: auto)")
    ap.add_argument("--mode", default="sampled", choices=["sampled", "certified", "config", "persist", "chain"],
                    help="sampled: the reference's timed path (default); certified: the plane count from the "
                         "full-matrix certificate; config: the single-graph path with (N, p) given (the sampled "
                         "rule's choice); persist: PersistA, A encoded once per step and --q products")
    ap.add_argument("--q", type=int, default=4, help="products per step in --mode persist")
    ap.add_argument("--planes", type=int, default=0, help="force the plane count N (0: the workload's rule)")
    ap.add_argument("--clock-log", default="", help="also write the raw nvidia-smi clock samples to this CSV file")
    args = ap.parse_args()
    if args.e2e_steps < 0:
        args.e2e_steps = max(6, args.steps)
    return args


def workload_config(args, m, n, k, phi, planes, p, world, grid, products=1):
    """The `config` object of the JSON line, the same for both arms (the reference arm adds only its sample)."""
    R, S = grid
    return {"workload": args.workload, "desc": _desc(args.workload), "m": m, "n": n, "k": k, "phi": phi,
            "planes": planes, "p": p, "mode": args.mode, "products_per_step": products,
            "parallelism": f"{R} x {S} grid of C blocks" if world > 1 else "single GPU",
            "l2": "inputs larger than L2 (2 x 2.1 GB fp64)"}


def _desc(workload):
    pkg = __graft_entry__.load_package()
    return pkg.CONFIGS[workload][6]


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
def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # noqa: E402  (the CPU port: timed baseline and reference arm only, never the product path)
    oracle.build()
    return oracle


def oracle_decision(oracle, A_host, B_host, force_N=None):
    """The reference algorithm's own decision on the workload's FULL inputs (CPU port, untimed): statistics over all
    of A and B, the probe set and probe product, the rule -> (statistics, N, p)."""
    m, k = A_host.shape
    n = B_host.shape[1]
    st = oracle.stats(A_host, B_host, True)
    I, J = oracle.probe_sets(st, m, n, k, 0)
    D = oracle.probe_D(A_host, B_host, I, J) if not force_N else np.zeros((len(I), len(J)))
    ru = oracle.rule(st, m, n, k, I, J, D, force_N=force_N)
    return st, ru["N"], ru["p"]


def cpu_step(oracle, A_host, B_host, st, N, p, s):
    """One CPU step on the sample block rows [0, s) x columns [0, s), full K: the block's statistics (timed work of
    the step) and the core (split, exact INT8 products, CRT reconstruction) at the workload's own (N, p) and global
    scalings, so the planes are those of the full product.  Returns seconds."""
    As = np.ascontiguousarray(A_host[:s])
    Bs = np.ascontiguousarray(B_host[:, :s])
    sub = {"gam": st["gam"], "r": st["r"][:s], "c": st["c"][:s]}
    t0 = time.perf_counter()
    oracle.stats(As, Bs, True)
    oracle.core(As, Bs, sub, N, p)
    return time.perf_counter() - t0


def cpu_baseline(oracle, A_host, B_host, st, N, p, sample, phi):
    """The CPU port of the reference's algorithm (oracle/, C + OpenMP, all host threads) on a sample block of the
    same workload (``cpu_step``), best of one timed step after a small warm-up."""
    k = A_host.shape[1]
    cpu_step(oracle, A_host[:8], B_host[:, :32], st, N, p, 8)          # warm the thread pool
    t = cpu_step(oracle, A_host, B_host, st, N, p, sample)
    return {"value": 2.0 * sample * sample * k / t / 1e12, "unit": "TFLOPS", "cores": oracle.num_threads(),
            "kind": "port", "seconds": t,
            "sample": f"rows 0..{sample} of A x columns 0..{sample} of B, full K={k}, phi={phi}, the full product's "
                      f"N={N}, p={p} and scalings; block statistics + split + exact INT8 products + CRT "
                      "reconstruction"}


def auto_sample(k, N, threads):
    # about 10-15 s of CPU work: the port's int8 products ran at ~7.7 G MAC/s per thread on the GPU boxes' host cores
    macs = 12.0 * 7.0e9 * max(1, threads)
    s = int((macs / (k * N)) ** 0.5)
    return max(32, min(2048, (s // 32) * 32))


# ------------------------------------------------------------------------------------------------ reference arm
def run_reference(args):
    """The reference arm: the reference's algorithm on the host cores (the C/OpenMP port in oracle/; the reference
    itself has no CPU engine and its GPU path needs Windows DLLs).  The plane count and p are the rule's own answer on
    the workload's full inputs, exactly as our arm decides them; each step is ``cpu_step`` on a sample block."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    pkg = __graft_entry__.load_package()
    m, k, n, phi, alt, forceN, desc = pkg.CONFIGS[args.workload]
    if args.planes:
        forceN = args.planes
    oracle = _oracle()
    threads = oracle.set_threads(len(os.sched_getaffinity(0)))   # all host cores, also under torchrun
    A, B = pkg.make_inputs(m, k, n, phi, 0, alt)
    st, N, p = oracle_decision(oracle, A, B, forceN)
    s = args.cpu_sample or auto_sample(k, N, threads) // 2
    times = []
    for it in range(args.warmup + args.steps):
        dt = cpu_step(oracle, A, B, st, N, p, s if it >= args.warmup else min(s, 64))
        if it >= args.warmup:
            times.append(dt)
    t = float(np.mean(times))
    v = 2.0 * s * s * k / t / 1e12
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    from matrix_numbers_b200.distributed import default_grid
    grid = default_grid(world) if world > 1 else (1, 1)
    line = {"metric": METRIC, "value": v, "unit": "TFLOPS", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64 (int8 residue arithmetic)", "data": "synthetic", "impl": "reference",
            "config": workload_config(args, m, n, k, phi, N, p, world, grid),
            "cpu_baseline": {"value": v, "unit": "TFLOPS", "cores": threads, "kind": "port",
                             "sample": f"rows 0..{s} x cols 0..{s} of the {args.workload} product, full K={k}, the "
                                       f"rule's N={N}, p={p} on the full inputs (block statistics + core per step)"},
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
def timed_calls(torch, dist, call, steps, warmup, world, stream, clocks_rank=None, clock_log=None, stage_events=False):
    """W untimed calls, then K calls bracketed by synchronize (+ barrier) and CUDA events on the launching stream;
    returns (seconds per call, max over ranks; last info; per-stage seconds of this rank; clock summary or None)."""
    info = None
    for _ in range(warmup):
        _, info = call(None)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    per_step = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(clocks_rank, clock_log) if clocks_rank is not None else None
    if sampler is not None:
        sampler.__enter__()
        time.sleep(0.3)
    try:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0.record(stream)
        for _ in range(steps):
            ev = [] if stage_events else None
            _, info = call(ev)
            if ev:
                per_step.append(ev)
        e1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    finally:
        if sampler is not None:
            sampler.__exit__(None, None, None)
    t = e0.elapsed_time(e1) / 1e3 / steps
    if world > 1:
        tt = torch.tensor([t], dtype=torch.float64, device=torch.device("cuda", torch.cuda.current_device()))
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt.item())
    stages = {}
    for ev in per_step:
        for (_, a), (name, b) in zip(ev[:-1], ev[1:]):
            stages[name] = stages.get(name, 0.0) + a.elapsed_time(b) / 1e3 / len(per_step)
    return t, info, stages, (sampler.summary() if sampler is not None else None)


def stages_over_ranks(torch, dist, stages, world):
    """Per-stage milliseconds of every rank (all_gather of this rank's figures; same stage names on all ranks)."""
    names = list(stages)
    if world == 1:
        return {"rank0": {n_: stages[n_] * 1e3 for n_ in names}}
    v = torch.tensor([stages[n_] * 1e3 for n_ in names], dtype=torch.float64, device="cuda")
    out = torch.empty(world * len(names), dtype=torch.float64, device="cuda")
    dist.all_gather_into_tensor(out, v)
    out = out.view(world, len(names)).cpu().tolist()
    return {f"rank{r}": dict(zip(names, out[r])) for r in range(world)}


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
    stream = torch.cuda.current_stream()
    clock_log = args.clock_log.replace(".csv", f"_rank{rank}.csv") if args.clock_log else None

    # inputs: generated on the host (numpy, seed 0)
    t_gen = time.perf_counter()
    A_host, B_host = pkg.make_inputs(m, k, n, phi, 0, alt)
    t_gen = time.perf_counter() - t_gen
    products = 1
    extra = {}
    if world == 1:
        R, S = 1, 1
        rows, cols = m, n
        A = torch.from_numpy(A_host).to(dev)
        B = torch.from_numpy(B_host).to(dev)
        C = torch.empty((m, n), dtype=torch.float64, device=dev)
        E = pkg.OzakiCRT()
        engine = E
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
        launches_of = lambda: E.launches  # noqa: E731
    else:
        # headline on N GPUs: blocks of C on the default grid (R x S, S = 2 from 4 ranks on); A's row block a lives on
        # the ranks of grid row a and C's blocks on their ranks; B lives on rank 0 only and is sent (FP64) over NCCL
        # inside every timed call -- whole to every rank on a row grid, column block b to grid column b otherwise
        assert args.mode in ("sampled", "certified"), "--mode config / persist are single-GPU"
        cert = args.mode == "certified"
        from matrix_numbers_b200.distributed import default_grid
        R, S = default_grid(world)
        ga, gb = divmod(rank, S)
        rows, cols = m // R, n // S
        assert rows % 4 == 0 and cols % 32 == 0, "block shape rule"
        A = torch.from_numpy(np.ascontiguousarray(A_host[ga * rows:(ga + 1) * rows])).to(dev)
        B_root = torch.from_numpy(B_host).to(dev) if rank == 0 else None
        # rank 0 keeps B as its S contiguous column blocks (the layout the column groups receive)
        B_parts = ([torch.from_numpy(np.ascontiguousarray(B_host[:, q * cols:(q + 1) * cols])).to(dev)
                    for q in range(S)] if (rank == 0 and S > 1) else B_root)
        C = torch.empty((rows, cols), dtype=torch.float64, device=dev)
        D = pkg.DistributedOzakiCRT(grid=(R, S))
        engine = D.engine
        call = lambda ev=None: D.run_broadcast_b(A, B_parts, C, root=0, force_N=forceN, certify=cert, events=ev)  # noqa: E731
        launches_of = lambda: D.launches  # noqa: E731

    launches0 = launches_of()
    t_dev, info, stages, clocks = timed_calls(torch, dist, call, args.steps, args.warmup, world, stream,
                                              clocks_rank=local, clock_log=clock_log, stage_events=True)
    launches = launches_of() - launches0
    flops = 2.0 * m * n * k * products
    value = flops / t_dev / 1e12
    stage_ms = stages_over_ranks(torch, dist, stages, world)

    if world > 1:
        # beside the headline: the same product with every operand pre-placed (no operand bytes on NVLink), on the
        # default grid; and with A and B on rank 0 only (A scattered, B broadcast, C gathered into rank 0)
        gR, gS = default_grid(world)
        br, bc = m // gR, n // gS
        A_g = torch.from_numpy(np.ascontiguousarray(A_host[ga * br:(ga + 1) * br])).to(dev)
        B_g = torch.from_numpy(np.ascontiguousarray(B_host[:, gb * bc:(gb + 1) * bc])).to(dev)
        C_g = torch.empty((br, bc), dtype=torch.float64, device=dev)
        Dg = pkg.DistributedOzakiCRT(grid=(gR, gS))
        cert = args.mode == "certified"
        t_pre, _, st_pre, _ = timed_calls(
            torch, dist, lambda ev=None: Dg.run(A_g, B_g, C_g, force_N=forceN, certify=cert, events=ev),
            args.steps, args.warmup, world, stream, stage_events=True)
        extra["presharded"] = {"value": flops / t_pre / 1e12, "ms_per_step": t_pre * 1e3,
                               "grid": f"{gR} x {gS} grid of C blocks",
                               "what": "A's row blocks and B's column blocks already on their ranks; only the "
                                       "statistics vectors and the probe product cross NVLink",
                               "stages_ms": stages_over_ranks(torch, dist, st_pre, world)}
        del A_g, B_g, C_g, Dg
        A_root = torch.from_numpy(A_host).to(dev) if rank == 0 else None
        C_root = torch.empty((m, n), dtype=torch.float64, device=dev) if rank == 0 else None
        Dr = pkg.DistributedOzakiCRT(grid=(world, 1))
        t_root, _, st_root, _ = timed_calls(
            torch, dist,
            lambda ev=None: Dr.run_from_root(A_root, B_root, C_root, root=0, force_N=forceN, certify=cert, events=ev),
            args.steps, args.warmup, world, stream, stage_events=True)
        extra["from_root"] = {"value": flops / t_root / 1e12, "ms_per_step": t_root * 1e3,
                              "what": "A and B on rank 0 only: A's row blocks scattered, B broadcast, C's row "
                                      "blocks gathered into rank 0, all inside the timed call",
                              "stages_ms": stages_over_ranks(torch, dist, st_root, world)}
        del A_root, C_root
        torch.cuda.empty_cache()
        # the exchange that limits the headline: the largest stage time of a collective step, over ranks
        coll = [x for x in next(iter(stage_ms.values())) if x != "core"]
        worst = max(((r_, x, v) for r_, d in stage_ms.items() for x, v in d.items() if x in coll),
                    key=lambda z: z[2], default=None)
        extra["limiting_collective"] = None if worst is None else {"stage": worst[1], "rank": worst[0],
                                                                   "ms": worst[2]}

    # roofline of the dominant kernel (the INT8 products with the fused reduction): live CUDA-event time per launch
    Nplanes = info.get("N") or forceN
    prof = {}
    b = engine.buffers(rows, cols, k, Nplanes)
    B_core = B if world == 1 else D.last_b
    for _ in range(3):
        engine.core(A, B_core, b, Nplanes, C, prof=prof)
    t_gemm = prof["gemm+reduce"] / 3
    int8_ops = 2.0 * Nplanes * rows * cols * k
    peak_int8 = int8_peak_tops(torch, dev)
    hbm_peak, bf16_peak, peak_src = measured_peaks()
    achieved = int8_ops / t_gemm / 1e12
    has_traffic = world == 1 and args.mode == "sampled" and args.workload in GEMM_TRAFFIC_BYTES
    roofline = {"bound": "tensor", "kernel": "gemm_tc_kernel<residue> (tcgen05.mma kind::i8)", "achieved": achieved,
                "peak": peak_int8, "unit": "TOPS (INT8)", "frac": achieved / peak_int8,
                "peak_source": "cuBLASLt INT8 GEMM 8192^3 burst measured in this run (torch._int_mm)",
                "bf16_measured_tflops_x2": 2 * bf16_peak, "frac_of_2x_bf16": achieved / (2 * bf16_peak),
                "traffic": GEMM_TRAFFIC_BYTES[args.workload] if has_traffic else None,
                "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
                "traffic_source": GEMM_TRAFFIC_SOURCE.format(w=args.workload) if has_traffic else None,
                "algorithmic_ops_per_launch": int8_ops, "ms_per_launch": t_gemm * 1e3,
                "stages_ms": {k_: v * 1e3 / 3 for k_, v in prof.items()}, "timed_call_stages_ms": stage_ms}
    # the emulated-FP64 ceiling is the INT8 rate over the plane count (one INT8 product per plane); the residue split
    # moves (8 + N)(rows k + k cols) bytes (FP64 in, N planes out) and the reconstruction (N + 8) rows cols bytes
    t_split, t_recon = prof["residues"] / 3, prof["recon"] / 3
    split_bytes = (8.0 + Nplanes) * (rows * k + k * cols)
    recon_bytes = (8.0 + Nplanes) * rows * cols
    roofline["emulated_ceiling_tflops"] = peak_int8 / Nplanes
    roofline["frac_of_int8_over_N"] = (2.0 * rows * cols * k / (t_dev / products) / 1e12) / (peak_int8 / Nplanes)
    roofline["split"] = {"bound": "hbm", "achieved": split_bytes / t_split / 1e9, "peak": hbm_peak, "unit": "GB/s",
                         "frac": split_bytes / t_split / 1e9 / hbm_peak, "bytes_per_call": split_bytes}
    roofline["recon"] = {"bound": "hbm", "achieved": recon_bytes / t_recon / 1e9, "peak": hbm_peak, "unit": "GB/s",
                         "frac": recon_bytes / t_recon / 1e9 / hbm_peak, "bytes_per_call": recon_bytes}

    # accuracy on a sample (rank 0's block): E1 / E2 against the correctly rounded product, native DGEMM beside it
    acc = None
    if rank == 0 and not args.no_accuracy:
        Cn = A @ B_core
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        torch.matmul(A, B_core, out=Cn)
        t1.record()
        torch.cuda.synchronize()
        t_nat = t0.elapsed_time(t1) / 1e3
        Smp = pkg.AccuracySample(A, B_core, Cn, nr=24, nc=24)
        acc = {"engine": Smp.errors(C), "native_dgemm": Smp.errors(Cn),
               "native_dgemm_tflops": 2.0 * rows * cols * k / t_nat / 1e12,
               "native_dgemm_shape": [rows, cols, k]}
        del Cn

    # end to end through the public API with host buffers (pinned), H2D + D2H inside the timed region
    e2e = None
    if args.e2e_steps > 0:
        single = None
        if world == 1:
            Ah = torch.from_numpy(A_host).pin_memory()
            Bh = torch.from_numpy(B_host).pin_memory()
            Ch = torch.empty((m, n), dtype=torch.float64).pin_memory()
        if world == 1 and args.mode == "sampled":
            E.run_host(Ah, Bh, Ch, force_N=forceN)             # warm-up of the host-buffer path
            torch.cuda.synchronize()
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f0.record(stream)
            for _ in range(args.e2e_steps):
                E.run_host(Ah, Bh, Ch, force_N=forceN)
            f1.record(stream)
            torch.cuda.synchronize()
            t_single = f0.elapsed_time(f1) / 1e3 / args.e2e_steps
            E.run_host_many([(Ah, Bh, Ch)] * 2, force_N=forceN)   # warm-up of the second slot
            torch.cuda.synchronize()
            f0.record(stream)
            E.run_host_many([(Ah, Bh, Ch)] * args.e2e_steps, force_N=forceN)
            f1.record(stream)
            torch.cuda.synchronize()
            t_e2e = f0.elapsed_time(f1) / 1e3 / args.e2e_steps
            api = (f"OzakiCRT.run_host_many (host buffers, {args.e2e_steps} products; each step's H2D, product and "
                   "D2H inside the timed region, the next step's H2D overlapped with this step's product)")
            single = {"value": flops / t_single / 1e12, "ms_per_step": t_single * 1e3,
                      "api": "OzakiCRT.run_host (one call at a time)"}
        elif world == 1:
            def host_step(ev=None):
                A.copy_(Ah, non_blocking=True)
                B.copy_(Bh, non_blocking=True)
                out = call(None)
                Ch.copy_(C, non_blocking=True)
                return out
            t_e2e, _, _, _ = timed_calls(torch, dist, host_step, args.e2e_steps, 1, world, stream)
            api = "H2D of A and B, OzakiCRT.run_fast, D2H of C"
        else:
            # every rank loads its share of its blocks from pinned host memory (each byte of A and B crosses PCIe
            # once, spread over all ranks' links), the grid rows and columns gather the blocks over NCCL, then the
            # grid product and the D2H of each C block; the next step's loads and this step's D2H overlap the product
            eR, eS = default_grid(world)
            ea, eb = divmod(rank, eS)
            br, bc = m // eR, n // eS
            sr, sk = br // eS, k // eR
            Ah = torch.from_numpy(np.ascontiguousarray(A_host[ea * br + eb * sr:ea * br + (eb + 1) * sr])).pin_memory()
            Bh = torch.from_numpy(np.ascontiguousarray(B_host[ea * sk:(ea + 1) * sk, eb * bc:(eb + 1) * bc]))
            Bh = Bh.pin_memory()
            Ch = torch.empty((br, bc), dtype=torch.float64).pin_memory()
            assert (eR, eS) == (D.R, D.S)
            kw_e = dict(shares=True, force_N=forceN, certify=args.mode == "certified")
            D.run_host_many([(Ah, Bh, Ch)] * 2, **kw_e)              # warm-up of both slots
            t_e2e, _, _, _ = timed_calls(
                torch, dist, lambda ev=None: D.run_host_many([(Ah, Bh, Ch)] * args.e2e_steps, **kw_e)[-1],
                1, 0, world, stream)
            t_e2e /= args.e2e_steps
            api = (f"DistributedOzakiCRT.run_host_many(shares=True) on the {eR} x {eS} grid, {args.e2e_steps} "
                   "products: each rank H2D of its share of A's row block and of B's column block, all_gather within grid rows "
                   "and columns, the grid product, D2H of its C block; the next step's H2D and this step's D2H "
                   "overlap the product")
        e2e = {"value": flops / t_e2e / 1e12, "unit": "TFLOPS", "ms_per_step": t_e2e * 1e3, "api": api,
               "h2d_bytes_per_step": (m * k + k * n) * 8, "d2h_bytes_per_step": m * n * 8}
        if single is not None:
            e2e["single_call"] = single

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        oracle = _oracle()
        st_full, N_o, p_o = oracle_decision(oracle, A_host, B_host, forceN)
        s = args.cpu_sample or auto_sample(k, N_o, oracle.num_threads())
        cpu = cpu_baseline(oracle, A_host, B_host, st_full, N_o, p_o, s, phi)
        cpu["decision_equals_gpu"] = bool((N_o, p_o) == (Nplanes, info.get("p")))

    if world > 1:
        dist.barrier()
    if rank == 0:
        metric = METRIC if args.mode == "sampled" else METRIC + f" [{args.mode} mode]"
        line = {"metric": metric, "value": value, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": t_dev * 1e3, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f64 (int8 residue arithmetic)", "data": "synthetic",
                "config": workload_config(args, m, n, k, phi, Nplanes, info.get("p"), world, (R, S), products),
                "input_generation_s": t_gen,
                "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "accuracy": acc, "clocks": clocks,
                "gpu_launches": launches, "hbm_peak_gbs": hbm_peak, "peaks": peak_src}
        if world > 1:
            line["operands"] = ("A's row block a on the ranks of grid row a, C's blocks on their ranks; B on rank 0, "
                                "sent (FP64) over NCCL inside every timed call: whole to every rank on a row grid, "
                                "column block b to the ranks of grid column b otherwise")
            line.update(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
