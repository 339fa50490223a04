"""Benchmark of the B200 FP16 GEMM (the path behind the reference's `solve`).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--M 8192 --N 8192 --K 8192] [--chunks C] [--workload gemm8192|sharded32k]

Workload: FP16 GEMM C = A @ B (alpha=1, beta=0), row-major, A/B full-entropy U[-1,1) from the
reference benchmark's counter-hash fill (three_way.cu:22-33, seeds three_way.cu:71-72).
One step = one GEMM (plus, with N GPUs, the all-gather of C). At N=1 the shape is 8192^3, the
configuration the metric is quoted on. With N GPUs (torchrun, one process per GPU) the
default job keeps the per-GPU work fixed (weak scaling): M = 8192*N rows split by rank, B
replicated, and every rank ends each step with the whole C: one kernel per rank computes its
rows and its epilogue stores each finished tile into every rank's C over NVLink (16-byte
stores into peer buffers mapped with CUDA IPC), followed by a one-warp device flag barrier
across the ranks (`--exchange nccl`, or when some rank cannot map the peers' buffers: the
GEMM then an NCCL all-gather instead). `--workload sharded32k`
runs BASELINE configs[4] instead: the 32768x32768x16384 GEMM split by rows over the N GPUs
(strong scaling).

Timing follows the reference methodology (three_way.cu): L2 flushed (memset of 3x the L2
size) before every timed launch, one launch between two CUDA events on the launching stream,
cuBLAS cublasGemmEx timed interleaved on the same data; W >= 3 warm-up steps; K timed
steps bracketed by barrier + synchronize; the max over ranks. `value` = whole-job TFLOPS over
the K steps; `e2e` = the same metric through the C ABI with host buffers (pinned H2D of A
and B, D2H of C inside the timed region): at N=1 `hgemm_launch_host`, which overlaps those
copies with the GEMM in row blocks, with the reference's copy / `solve` / copy sequence
reported beside it (`e2e.solve_path`); at N>1 `hgemm_sharded_rank` between the copies.

After the timed steps every rank checks its whole C (its own rows and the rows the other
ranks stored into it) against the same GEMM run on one GPU in one launch (bit equality) and
against cuBLAS (rel_l2); the line reports the worst rank. Every run also measures BASELINE
configs[4] at the same N (`config5`: the 32768x32768x16384 GEMM split by rows over the GPUs,
strong scaling, same exchange and the same whole-C checks), unless --no-config5.
`--grid` runs each shape of the grid in a process of its own.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_PEAK_TFLOPS = 1590.0
FALLBACK_SUSTAINED_TFLOPS = 1400.0
DEFAULT_CHUNKS = 1  # --exchange nccl: measured fastest on 2 B200s (one in-place all-gather)
FALLBACK_HBM_GBS = 6650.0
# Peer copy over NVLink 5, measured on this pool's B200s (per direction per GPU); the bound
# for the bytes a fused step must move to the other ranks.
NVLINK_PEER_GBS = 770.0
# the row-sharded 32768 x 32768 x 16384 GEMM.
C5_M, C5_N, C5_K = 32768, 32768, 16384


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--M", type=int, default=8192, help="rows per GPU")
    ap.add_argument("--N", type=int, default=8192)
    ap.add_argument("--K", type=int, default=8192)
    ap.add_argument("--chunks", type=int, default=0,
                    help="row chunks per rank for gather overlap (N>1; 0 = automatic)")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="N>1: peer = one kernel per rank stores its tiles into every rank's C "
                         "over NVLink (CUDA IPC); nccl = GEMM then NCCL all-gather / send-recv")
    ap.add_argument("--reserved-sms", type=int, default=-1,
                    help="SMs the chunk GEMMs leave to the exchange (N>1; -1 = library default)")
    ap.add_argument("--workload", default="gemm8192", choices=["gemm8192", "sharded32k"],
                    help="gemm8192: 8192 rows x 8192 x 8192 per GPU (weak scaling); sharded32k: "
                         "the 32768x32768x16384 GEMM split by rows over the GPUs (strong)")
    ap.add_argument("--force-bm", type=int, default=0, help="tile rows (0 = automatic)")
    ap.add_argument("--force-bn", type=int, default=0, help="tile columns (0 = automatic)")
    ap.add_argument("--group-m", type=int, default=0, help="raster band height (0 = automatic)")
    ap.add_argument("--grid", action="store_true",
                    help="the reference's 31-shape grid (perf_shapes.h) plus the ragged and thin-K "
                         "configs, one JSON line per shape, ours vs cuBLAS interleaved")
    ap.add_argument("--grid-reps", type=int, default=25)
    ap.add_argument("--grid-shapes", default="",
                    help="with --grid: only these shapes, comma-separated MxNxK[:alpha/beta] "
                         "(e.g. 1024x1024x1024,3000x1000x2000:1.5/0.5)")
    ap.add_argument("--no-config5", dest="config5", action="store_false",
                    help="skip the BASELINE configs[4] block (32768x32768x16384 split by rows "
                         "over the N GPUs, strong scaling) that every run adds by default")
    ap.add_argument("--config5-steps", type=int, default=10)
    ap.add_argument("--grid-child", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--grid-index", type=int, default=0, help=argparse.SUPPRESS)
    ap.add_argument("--peer-standins", type=int, default=0,
                    help="with --grid: run the peer-store flavour of the fused multi-GPU path with "
                         "this many same-GPU buffers standing in for the peers' C (0-7)")
    ap.add_argument("--grid-misalign", type=int, default=0,
                    help="with --grid: start A, B and C this many halves past a 16-byte boundary "
                         "(1-7): ours then restrides A and B and writes C with the SIMT-store "
                         "epilogue, cuBLAS runs its own misaligned-operand kernels")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def peaks(sustained=False):
    """(dense bf16 TFLOP/s, HBM GB/s, source) from MEASURED_PEAKS.json: the burst GEMM figure
    for a kernel timed alone, the sustained (power-capped) one for seconds of back-to-back
    work."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
        return float(p[key]), float(p["hbm_gbs"]), "measured"
    except Exception:
        return (FALLBACK_SUSTAINED_TFLOPS if sustained else FALLBACK_PEAK_TFLOPS,
                FALLBACK_HBM_GBS, "fallback")


def profiled_traffic(M, N, K):
    """dram bytes per launch from the committed ncu summary for this kernel and shape."""
    path = os.path.join(ROOT, "profiles", "hgemm_tc_kernel_8192x8192x8192.md")
    if (M, N, K) != (8192, 8192, 8192) or not os.path.exists(path):
        return None
    for line in open(path):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """SM clock, power and throttle reasons sampled through NVML every 2 ms while the timed
    region runs (falls back to `nvidia-smi -lms 100` when pynvml is missing)."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, index):
        self.index = index
        self.samples = []  # (sm_mhz, max_mhz, power_w, reasons_bitmask)
        self.stop = threading.Event()
        self.thread = None

    def _poll_nvml(self):
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        while not self.stop.is_set():
            try:
                self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), mx,
                                     pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0,
                                     pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)))
            except pynvml.NVMLError:
                pass
            self.stop.wait(0.002)

    def _poll_smi(self):
        fields = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                  "clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        bits = [0x8, 0x40, 0x20, 0x4]
        proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={fields}",
                                 "--format=csv,noheader,nounits", "-lms", "100"],
                                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        try:
            for line in proc.stdout:
                if self.stop.is_set():
                    break
                p = [x.strip() for x in line.split(",")]
                try:
                    mask = sum(b for b, v in zip(bits, p[3:7]) if v.lower() == "active")
                    self.samples.append((float(p[0]), float(p[1]), float(p[2]), mask))
                except (ValueError, IndexError):
                    continue
        finally:
            proc.terminate()

    def __enter__(self):
        try:
            import pynvml  # noqa: F401
            target = self._poll_nvml
        except ImportError:
            target = self._poll_smi
        self.thread = threading.Thread(target=target, daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *exc):
        self.stop.set()
        self.thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        mask = 0
        for s in self.samples:
            mask |= int(s[3])
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": self.samples[0][1],
                "power_w_median": statistics.median(s[2] for s in self.samples),
                "reasons": sorted(k for k, b in self.REASONS.items() if mask & b),
                "samples": len(self.samples)}


def hash_fill_(t, seed):
    """three_way.cu:22-33 counter-hash fill, computed on the device with torch int64 ops."""
    import torch
    flat = t.view(-1)
    n = flat.numel()
    step = 1 << 25
    m32 = 0xFFFFFFFF
    for b in range(0, n, step):
        e = min(n, b + step)
        i = torch.arange(b, e, device=t.device, dtype=torch.int64)
        h = ((i * 2654435761) & m32) ^ (seed & m32)
        h ^= h >> 15
        h = (h * 2246822519) & m32
        h ^= h >> 13
        h = (h * 3266489917) & m32
        h ^= h >> 16
        flat[b:e] = ((h & 0xFFFF).to(torch.float32) / 32768.0 - 1.0).to(torch.float16)
    return t


def cpu_baseline(M, N, K, budget_s=10.0):
    """The oracle (restated reference fp64 GEMM) on a bounded row sample of the workload,
    all host threads; TFLOPS of the sample."""
    import numpy as np
    from oracle import oracle as orc
    orc.build()
    threads = orc.max_threads()
    B = orc.hash_fill_half((K, N), 0x85EBCA6B)
    rows_probe = max(4, threads)  # one row per thread, so the probe rate scales
    A = orc.hash_fill_half((rows_probe, K), 0x9E3779B9)
    t0 = time.perf_counter()
    orc.gemm_f64(A, B, rows=np.arange(rows_probe), threads=threads)
    dt = time.perf_counter() - t0
    rows = int(max(threads, min(M, rows_probe * budget_s / max(dt, 1e-6))))
    rows = max(threads, (rows // threads) * threads)
    A = orc.hash_fill_half((rows, K), 0x9E3779B9)
    t0 = time.perf_counter()
    orc.gemm_f64(A, B, rows=np.arange(rows), threads=threads)
    dt = time.perf_counter() - t0
    return {"value": 2.0 * rows * N * K / dt / 1e12, "unit": "TFLOPS", "cores": threads,
            "kind": "port",
            "sample": f"rows 0..{rows - 1} of the {M}x{N}x{K} GEMM ({rows}x{N}x{K} MACs), "
                      f"fp64 accumulate in k order (check_fp64.cu:39-44), {dt:.1f} s"}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU implementation of the path (the fp64 host GEMM
    of check_fp64.cu:39-44, restated in oracle/ because the reference's own file cannot run
    without an sm_90 GPU), timed on this box's host cores over bounded samples."""
    if rank != 0:
        return
    import numpy as np
    from oracle import oracle as orc
    orc.build()
    M, N, K = args.M * world, args.N, args.K
    threads = orc.max_threads()
    B = orc.hash_fill_half((K, N), 0x85EBCA6B)
    rows = 8 * threads
    A = orc.hash_fill_half((rows, K), 0x9E3779B9)
    for _ in range(max(args.warmup, 0)):
        orc.gemm_f64(A, B, rows=np.arange(threads), threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        orc.gemm_f64(A, B, rows=np.arange(rows), threads=threads)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = 2.0 * rows * N * K * len(times) / total / 1e12
    sample = f"{rows} rows of the {M}x{N}x{K} GEMM per step ({rows}x{N}x{K} MACs, fp64)"
    print(json.dumps({
        "impl": "reference", "metric": "fp16_gemm_tflops", "value": value, "unit": "TFLOPS",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / len(times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": f"gemm_{M}x{N}x{K}_rowsharded" if world > 1 else f"gemm_{M}x{N}x{K}",
                   "alpha": 1.0, "beta": 0.0},
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)


# perf_shapes.h:2-11 (the reference's 31-shape benchmark grid) and BASELINE.json configs.
GRID_SHAPES = [
    (2048, 2048, 2048), (4096, 4096, 4096), (8192, 8192, 8192), (16384, 16384, 16384),
    (8192, 8192, 1024), (8192, 8192, 2048), (8192, 8192, 4096), (8192, 8192, 16384),
    (16384, 8192, 4096), (4096, 4096, 8192), (32768, 8192, 2048), (4096, 4096, 1024),
    (8192, 1024, 8192), (8192, 4096, 8192), (4096, 8192, 8192), (16384, 4096, 8192),
    (4096, 8192, 128), (4096, 8192, 256), (4096, 8192, 512), (4096, 8192, 1024),
    (8192, 8192, 128), (16384, 8192, 128), (3000, 1000, 2000), (384, 2048, 2048),
    (1024, 1024, 1024), (2048, 2048, 512), (4096, 512, 4096),
    (4096, 4095, 4096), (2048, 2047, 2048), (4095, 4095, 4095), (1024, 1023, 1024),
]
GRID_RAGGED = [(4095, 4095, 4095), (4096, 4095, 4096), (2048, 2047, 2048), (3000, 1000, 2000)]


def run_grid(args):
    import ctypes
    """Reference methodology per shape (three_way.cu): hash-filled A/B, 5 interleaved
    warm-ups, then `reps` rounds of {3x L2 memset, event, one launch, event} for ours, for
    cuBLAS and (16-byte aligned shapes, when it was built) for the CUTLASS SM100 comparator;
    median TFLOPS and the median of per-round paired ratios. The ragged configs are also run
    with alpha=1.5, beta=0.5 (BASELINE configs[1])."""
    import torch
    import hopper_gemm_b200 as hg
    from hopper_gemm_b200._native import cublas_ref_lib, cutlass_ref_lib
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    cub = cublas_ref_lib()
    cut = cutlass_ref_lib()  # third column (None if the comparator was not built)
    flush = torch.empty(3 * torch.cuda.get_device_properties(dev).L2_cache_size,
                        dtype=torch.uint8, device=dev)
    cases = [(M, N, K, 1.0, 0.0) for (M, N, K) in GRID_SHAPES]
    cases += [(M, N, K, 1.5, 0.5) for (M, N, K) in GRID_RAGGED]
    if args.grid_shapes:
        cases = []
        for spec in args.grid_shapes.split(","):
            dims, _, ab = spec.partition(":")
            M, N, K = (int(v) for v in dims.split("x"))
            al, be = (float(v) for v in ab.split("/")) if ab else (1.0, 0.0)
            cases.append((M, N, K, al, be))
    if not args.grid_child:
        # One shape per process, as the reference's harness runs them (Makefile:78-79,
        # three_way.cu's single-shape mode): a shape measured after others inherits their heat.
        for i, (M, N, K, al, be) in enumerate(cases):
            spec = f"{M}x{N}x{K}:{al}/{be}"
            subprocess.run([sys.executable, os.path.abspath(__file__), "--grid", "--grid-child",
                            "--grid-shapes", spec, "--grid-index", str(i),
                            "--grid-reps", str(args.grid_reps),
                            "--peer-standins", str(args.peer_standins),
                            "--grid-misalign", str(args.grid_misalign)], check=True)
        return
    for i, (M, N, K, al, be) in enumerate(cases, start=args.grid_index):
        off = args.grid_misalign

        def mat(rows, cols):
            # a rows x cols view that starts `off` halves into a fresh (256-byte aligned) buffer
            return torch.empty(rows * cols + off, dtype=torch.float16, device=dev)[off:].view(
                rows, cols)

        A = hash_fill_(mat(M, K), 0x9E3779B9 ^ i)
        B = hash_fill_(mat(K, N), 0x85EBCA6B ^ i)
        C = hash_fill_(mat(M, N), 0x1234 ^ i)
        R, C0, T = mat(M, N), mat(M, N), mat(M, N)
        R.copy_(C)
        C0.copy_(C)
        T.copy_(C)
        use_cut = cut is not None and N % 8 == 0 and K % 8 == 0 and K > 0 and off == 0
        # --peer-standins P: ours runs the fused multi-GPU path's peer-store kernel flavour
        # with P same-GPU buffers standing in for the peers' C (the SM-side cost of the peer
        # copies on one GPU, and a one-GPU target for profiling that kernel)
        stand = [torch.empty((M, N), dtype=torch.float16, device=dev)
                 for _ in range(args.peer_standins)]
        stand_arr = (ctypes.c_void_p * max(1, len(stand)))(*[t.data_ptr() for t in stand])

        def ours():
            if stand:
                st = hg.lib.hgemm_launch_peers(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K,
                                               al, be, sptr, stand_arr, len(stand), 0)
            else:
                st = hg.lib.hgemm_launch(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, al,
                                         be, sptr)
            if st != 0:
                raise RuntimeError(hg.status_string(st))

        def cbl():
            cub.hgemm_cublas_ref(A.data_ptr(), B.data_ptr(), R.data_ptr(), M, N, K, al, be, sptr)

        def ctl():
            st = cut.hgemm_cutlass_ref(A.data_ptr(), B.data_ptr(), T.data_ptr(), M, N, K, al, be,
                                       sptr)
            if st != 0:
                raise RuntimeError(f"hgemm_cutlass_ref status {st}")

        def sample(fn):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            flush.fill_(0x5A)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            return e0.elapsed_time(e1)

        # correctness of this shape against cuBLAS from the same C input
        C.copy_(C0)
        R.copy_(C0)
        T.copy_(C0)
        ours()
        cbl()
        if use_cut:
            ctl()
        torch.cuda.synchronize()
        l2 = float((C.float() - R.float()).norm() / (R.float().norm() + 1e-30))
        l2t = (float((C.float() - T.float()).norm() / (T.float().norm() + 1e-30))
               if use_cut else None)
        for _ in range(5):
            ours()
            cbl()
            if use_cut:
                ctl()
        torch.cuda.synchronize()
        to, tc, tt = [], [], []
        for _ in range(args.grid_reps):
            to.append(sample(ours))
            tc.append(sample(cbl))
            if use_cut:
                tt.append(sample(ctl))
        fl = 2.0 * M * N * K
        plan = hg.plan(M, N, K, beta=be, aligned16=(off == 0))
        print(json.dumps({
            "shape": f"{M}x{N}x{K}", "alpha": al, "beta": be,
            "ours_tflops": fl / (statistics.median(to) * 1e-3) / 1e12,
            "cublas_tflops": fl / (statistics.median(tc) * 1e-3) / 1e12,
            "paired_ratio_median": statistics.median(c / o for o, c in zip(to, tc)),
            "cutlass_tflops": fl / (statistics.median(tt) * 1e-3) / 1e12 if tt else None,
            "paired_ratio_vs_cutlass": (statistics.median(t / o for o, t in zip(to, tt))
                                        if tt else None),
            "rel_l2_vs_cublas": l2, "rel_l2_vs_cutlass": l2t,
            "tile": f"{plan['tile_m']}x{plan['tile_n']}", "peer_standins": len(stand),
            "path": {0: "none", 1: "tcgen05", 2: "scalar kernel"}[plan["path"]],
            "misalign_halves": off,
            "restride": bool(plan["pad_a"] or plan["pad_b"])}), flush=True)
        del A, B, C, R, C0, T, stand
        torch.cuda.empty_cache()


def fused_roofline(rows, N, K, world, step_ms, peak_tflops):
    """Roofline of one rank's fused step (GEMM whose epilogue stores every tile into the other
    ranks' C over NVLink): the target time is the slower of the math at the measured GEMM peak
    and the rows this rank must send at the measured peer-copy bandwidth; frac = target / the
    measured step (kernel + exit barrier)."""
    flops = 2.0 * rows * N * K
    link_bytes = (world - 1) * rows * N * 2.0  # sent per rank (and received, by symmetry)
    t_math = flops / (peak_tflops * 1e12)
    t_link = link_bytes / (NVLINK_PEER_GBS * 1e9)
    step_s = step_ms * 1e-3
    if t_math >= t_link:
        return {"bound": "tensor", "achieved": flops / step_s / 1e12, "peak": peak_tflops,
                "unit": "TFLOP/s", "frac": t_math / step_s, "traffic": None,
                "nvlink_gbs_per_direction": link_bytes / step_s / 1e9,
                "kernel": "hgemm_tc_kernel peer-store flavour (+ one-warp exit barrier)"}
    return {"bound": "nvlink", "achieved": link_bytes / step_s / 1e9, "peak": NVLINK_PEER_GBS,
            "unit": "GB/s", "frac": t_link / step_s, "traffic": None,
            "tflops": flops / step_s / 1e12,
            "kernel": "hgemm_tc_kernel peer-store flavour (+ one-warp exit barrier)"}


class Job:
    """One row-sharded GEMM job on this rank: A rows [rb, rb + Ml) of an M x K matrix, B
    replicated, C the full M x N on every rank (gathered by hgemm_sharded_rank for N > 1)."""

    def __init__(self, hg, dev, rank, world, M, N, K, a_blocks):
        import torch
        self.hg, self.dev, self.rank, self.world = hg, dev, rank, world
        self.M, self.N, self.K = M, N, K
        self.rb, self.Ml = hg.shard_rows(M, world, rank)
        self.a_blocks = a_blocks  # (row_begin, rows, seed) blocks that make up the full A
        self.A = self.fill_a(self.rb, self.Ml)
        self.B = hash_fill_(torch.empty((K, N), dtype=torch.float16, device=dev), 0x85EBCA6B)
        self.C = torch.empty((M, N), dtype=torch.float16, device=dev)

    def fill_a(self, r0, rows):
        """Rows [r0, r0 + rows) of the full A, each block filled with its own seed."""
        import torch
        out = torch.empty((rows, self.K), dtype=torch.float16, device=self.dev)
        for b0, n, seed in self.a_blocks:
            lo, hi = max(b0, r0), min(b0 + n, r0 + rows)
            if lo < hi:
                blk = hash_fill_(torch.empty((n, self.K), dtype=torch.float16, device=self.dev),
                                 seed)
                out[lo - r0:hi - r0].copy_(blk[lo - b0:hi - b0])
                del blk
        return out

    def full_check(self):
        """The whole gathered C on this rank against (a) the same GEMM computed here on one GPU
        in one launch (bit equality: every row block is the same kernel's arithmetic) and (b)
        cuBLAS on the full problem (rel_l2). Untimed."""
        import torch
        from hopper_gemm_b200._native import cublas_ref_lib
        torch.cuda.synchronize()
        A = self.fill_a(0, self.M)
        ref = torch.empty_like(self.C)
        st = self.hg.lib.hgemm_launch(A.data_ptr(), self.B.data_ptr(), ref.data_ptr(), self.M,
                                      self.N, self.K, 1.0, 0.0, None)
        assert st == 0, self.hg.status_string(st)
        torch.cuda.synchronize()
        same = bool(torch.equal(self.C.view(torch.int16), ref.view(torch.int16)))
        st = cublas_ref_lib().hgemm_cublas_ref(A.data_ptr(), self.B.data_ptr(), ref.data_ptr(),
                                               self.M, self.N, self.K, 1.0, 0.0, None)
        assert st == 0
        torch.cuda.synchronize()
        num = den = 0.0
        step = max(1, (1 << 27) // max(self.N, 1))
        for r0 in range(0, self.M, step):
            c = self.C[r0:r0 + step].float()
            r = ref[r0:r0 + step].float()
            num += float(((c - r) ** 2).sum())
            den += float((r * r).sum())
        del A, ref
        torch.cuda.empty_cache()
        return same, (num / (den + 1e-30)) ** 0.5


def main():
    args = parse()
    if args.grid:
        run_grid(args)
        return
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    import hopper_gemm_b200 as hg
    from hopper_gemm_b200._native import cublas_ref_lib

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=120))

    if args.workload == "sharded32k":
        # A 32768x16384 split by rows, B 16384x32768 replicated.
        M, N, K = C5_M, C5_N, C5_K
        if M % world:
            raise SystemExit("sharded32k needs a GPU count that divides 32768")
        blocks = [(0, M, 0x9E3779B9)]
    else:
        N, K = args.N, args.K
        M = args.M * world
        blocks = [(hg.shard_rows(M, world, r)[0], hg.shard_rows(M, world, r)[1], 0x9E3779B9 ^ r)
                  for r in range(world)]
    if args.chunks <= 0:
        args.chunks = 1 if world == 1 else DEFAULT_CHUNKS
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    job = Job(hg, dev, rank, world, M, N, K, blocks)
    Ml, rb = job.Ml, job.rb
    flops_job = 2.0 * M * N * K
    R = torch.empty((Ml, N), dtype=torch.float16, device=dev)  # cuBLAS output
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    flush = torch.empty(3 * l2, dtype=torch.uint8, device=dev)

    comm = None
    peer_fallback = None
    if world > 1:
        import ctypes
        idbuf = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            host_id = (ctypes.c_ubyte * 128)()
            st = hg.lib.hgemm_comm_unique_id(host_id, 128)
            assert st == 0, hg.status_string(st)
            idbuf.copy_(torch.tensor(list(host_id), dtype=torch.uint8))
        dist.broadcast(idbuf, 0)
        id_bytes = bytes(idbuf.cpu().tolist())
        comm_p = ctypes.c_void_p()
        st = hg.lib.hgemm_comm_init(ctypes.byref(comm_p), world, id_bytes, 128, rank)
        assert st == 0, hg.status_string(st)
        comm = comm_p
        if args.reserved_sms >= 0:
            st = hg.lib.hgemm_comm_set_reserved_sms(comm, args.reserved_sms)
            assert st == 0, hg.status_string(st)

    def register(C):
        """Collective: the fused path for output C (every rank agrees on the outcome)."""
        nonlocal peer_fallback
        if comm is None or args.exchange != "peer":
            return
        st = hg.lib.hgemm_comm_register_output(comm, C.data_ptr(), C.numel() * C.element_size())
        if st != 0:
            peer_fallback = hg.status_string(st)
            args.exchange = "nccl"

    def step_fn(j, A=None, B=None):
        A = j.A if A is None else A
        B = j.B if B is None else B

        def fn():
            if comm is None:
                st = hg.lib.hgemm_launch_ex(A.data_ptr(), B.data_ptr(), j.C.data_ptr(), j.Ml,
                                            j.N, j.K, 1.0, 0.0, sptr, args.force_bm,
                                            args.force_bn, args.group_m)
            else:
                st = hg.lib.hgemm_sharded_rank(comm, A.data_ptr(), B.data_ptr(), j.C.data_ptr(),
                                               j.M, j.N, j.K, 1.0, 0.0, args.chunks, sptr)
            if st != 0:
                raise RuntimeError(hg.status_string(st))
        return fn

    register(job.C)
    ours = step_fn(job)
    cub = cublas_ref_lib()

    def cublas():
        st = cub.hgemm_cublas_ref(job.A.data_ptr(), job.B.data_ptr(), R.data_ptr(), Ml, N, K,
                                  1.0, 0.0, sptr)
        if st != 0:
            raise RuntimeError("cublas failed")

    def sample(fn):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        flush.fill_(0x5A)
        e0.record(stream)
        fn()
        e1.record(stream)
        return e0, e1

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(vals):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(v) for v in t]

    # warm-up (interleaved, as three_way.cu:141)
    for _ in range(args.warmup):
        ours()
        cublas()
    barrier()

    # timed region: K steps of ours, cuBLAS interleaved round-robin
    ev_ours, ev_cub = [], []
    region0 = torch.cuda.Event(enable_timing=True)
    region1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        region0.record(stream)
        for _ in range(args.steps):
            ev_ours.append(sample(ours))
            ev_cub.append(sample(cublas))
        region1.record(stream)
        barrier()
    t_ours = [a.elapsed_time(b) for a, b in ev_ours]
    t_cub = [a.elapsed_time(b) for a, b in ev_cub]
    region_ms = region0.elapsed_time(region1)
    tot = max_over_ranks([sum(t_ours), sum(t_cub)])
    ms_ours = tot[0] / args.steps
    ms_cub = tot[1] / args.steps
    value = flops_job / (ms_ours * 1e-3) / 1e12
    cub_value = flops_job / (ms_cub * 1e-3) / 1e12 if world == 1 else None
    ratios = [c / o for o, c in zip(t_ours, t_cub)]

    # the whole gathered C on every rank: bit equality with a one-GPU launch, rel_l2 vs cuBLAS
    same, full_l2 = job.full_check()
    chk = max_over_ranks([0.0 if same else 1.0, full_l2])
    st_dev, where = hg.device_status(clear=False)
    st_max = max_over_ranks([float(st_dev)])[0]

    # end to end through the C ABI with host buffers
    e2e = None
    e2e_call = None
    if not args.no_e2e:
        hA = torch.empty((Ml, K), dtype=torch.float16, pin_memory=True)
        hB = torch.empty((K, N), dtype=torch.float16, pin_memory=True)
        hC = torch.empty((Ml, N), dtype=torch.float16, pin_memory=True)
        hA.copy_(job.A)
        hB.copy_(job.B)
        dA2 = torch.empty_like(job.A)
        dB2 = torch.empty_like(job.B)
        e2e_steps = max(3, min(args.steps, 10))
        e2e_call = step_fn(job, dA2, dB2)

        def copy_step():
            # copies in, the GEMM through the C ABI on device buffers, copy out
            dA2.copy_(hA, non_blocking=True)
            dB2.copy_(hB, non_blocking=True)
            if comm is None:
                hg.lib.solve(dA2.data_ptr(), dB2.data_ptr(), job.C.data_ptr(), Ml, N, K, 1.0, 0.0)
            else:
                e2e_call()
            hC.copy_(job.C[rb:rb + Ml], non_blocking=True)

        def host_step():
            # hgemm_launch_host: the same copies, in row blocks overlapped with the GEMM
            st = hg.lib.hgemm_launch_host(hA.data_ptr(), hB.data_ptr(), hC.data_ptr(),
                                          dA2.data_ptr(), dB2.data_ptr(), job.C.data_ptr(),
                                          Ml, N, K, 1.0, 0.0, sptr)
            if st != 0:
                raise RuntimeError(hg.status_string(st))

        def timed_e2e(step):
            for _ in range(2):
                step()
            barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(e2e_steps):
                step()
            e1.record(stream)
            barrier()
            return max_over_ranks([e0.elapsed_time(e1)])[0] / e2e_steps

        solve_ms = timed_e2e(copy_step)
        e2e_ms = timed_e2e(host_step) if comm is None else solve_ms
        e2e = {"value": flops_job / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOPS",
               "h2d_bytes_per_step": 2 * (Ml * K + K * N), "d2h_bytes_per_step": 2 * Ml * N,
               "ms_per_step": e2e_ms,
               "path": "hgemm_launch_host() C ABI, pinned host buffers (row blocks of A and C "
                       "copied in overlap with the GEMM)" if comm is None else
                       "hgemm_sharded_rank() C ABI, pinned host buffers"}
        if comm is None:
            # the reference's sequence on the same buffers: copy A and B in, solve(), copy C out
            e2e["solve_path"] = {"value": flops_job / (solve_ms * 1e-3) / 1e12,
                                 "ms_per_step": solve_ms,
                                 "path": "cudaMemcpyAsync in, solve() C ABI, cudaMemcpyAsync out"}
            # both leave the same C in the host buffer
            ref_c = hC.clone()
            copy_step()
            torch.cuda.synchronize()
            e2e["host_path_matches_solve_path"] = bool(torch.equal(ref_c, hC))
        assert hg.last_status() == 0, hg.status_string(hg.last_status())
        del hA, hB, hC, dA2, dB2

    peak, hbm, src = peaks()
    if world == 1:
        roofline = {"bound": "tensor", "achieved": 2.0 * Ml * N * K / (ms_ours * 1e-3) / 1e12,
                    "peak": peak, "unit": "TFLOP/s", "traffic": profiled_traffic(Ml, N, K),
                    "peak_source": f"{src} bf16 dense (burst)"}
        roofline["frac"] = roofline["achieved"] / peak
    else:
        # the fused kernel inside the timed step is the dominant kernel
        roofline = fused_roofline(Ml, N, K, world, ms_ours, peak)
        roofline["peak_source"] = (f"{src} bf16 dense (burst); NVLink: measured peer copy "
                                   f"{NVLINK_PEER_GBS:.0f} GB/s per direction")
    exchange_desc = None if world == 1 else (
        "fused GEMM epilogue stores every tile to all ranks' C over NVLink (16-byte stores, "
        "CUDA IPC peer mappings), gated on the peers' step-entry flags, + device flag exit "
        "barrier" if args.exchange == "peer" else
        f"NCCL all-gather / send-recv, {args.chunks} chunk(s)" +
        (f" (peer mapping unavailable: {peer_fallback})" if peer_fallback else ""))
    main_workload = (f"gemm_{M}x{N}x{K}" if world == 1 else
                     f"gemm_{M}x{N}x{K}_rowsharded_" +
                     ("peerstore" if args.exchange == "peer" else "allgather"))
    gpu_launches = args.steps * (1 if comm is None else
                                 2 if args.exchange == "peer" else max(1, args.chunks))
    clk = clocks.summary()
    del R

    # BASELINE configs[4] at every N: the 32768 x 32768 x 16384 GEMM split by rows over the
    # ranks (strong scaling), same exchange, full gathered-C check on every rank.
    c5 = None
    if args.config5 and args.workload != "sharded32k" and C5_M % world == 0:
        j5 = Job(hg, dev, rank, world, C5_M, C5_N, C5_K, [(0, C5_M, 0x9E3779B9)])
        register(j5.C)  # collective; unmaps the peers' previous output buffers first
        del job, ours, cublas, e2e_call
        torch.cuda.empty_cache()
        f5 = step_fn(j5)
        for _ in range(3):
            f5()
        barrier()
        with ClockSampler(local_rank) as clk5:
            ev5 = [sample(f5) for _ in range(args.config5_steps)]
            barrier()
        ms5 = max_over_ranks([sum(a.elapsed_time(b) for a, b in ev5)])[0] / len(ev5)
        same5, l2_5 = j5.full_check()
        chk5 = max_over_ranks([0.0 if same5 else 1.0, l2_5])
        st5 = hg.device_status(clear=False)[0]
        st5 = max_over_ranks([float(st5)])[0]
        # tens of ms of back-to-back GEMM per rank: the power-capped (sustained) peak
        peak5, _, src5 = peaks(sustained=True)
        rl5 = (fused_roofline(j5.Ml, C5_N, C5_K, world, ms5, peak5) if world > 1 else
               {"bound": "tensor", "achieved": 2.0 * C5_M * C5_N * C5_K / (ms5 * 1e-3) / 1e12,
                "peak": peak5, "unit": "TFLOP/s", "traffic": None})
        if world == 1:
            rl5["frac"] = rl5["achieved"] / peak5
        rl5["peak_source"] = f"{src5} bf16 dense (sustained)"
        c5 = {"workload": f"gemm_{C5_M}x{C5_N}x{C5_K}_rowsharded{world}",
              "baseline_config": "configs[4]", "scaling": "strong",
              "M": C5_M, "N": C5_N, "K": C5_K, "rows_per_gpu": j5.Ml,
              "steps": len(ev5), "warmup": 3, "ms_per_step": ms5,
              "value": 2.0 * C5_M * C5_N * C5_K / (ms5 * 1e-3) / 1e12, "unit": "TFLOPS",
              "roofline": rl5, "full_c_bit_identical_to_one_gpu_launch": chk5[0] == 0.0,
              "full_c_rel_l2_vs_cublas_max_over_ranks": chk5[1], "device_status": int(st5),
              "clocks": clk5.summary(),
              "gpu_launches": len(ev5) * (1 if comm is None else 2)}
        del j5, f5

    if comm is not None:
        hg.lib.hgemm_comm_destroy(comm)

    if rank == 0:
        line = {
            "metric": "fp16_gemm_tflops", "value": value, "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_ours,
            "higher_is_better": True,
            "scaling": "strong" if args.workload == "sharded32k" else "weak",
            "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (three_way.cu counter-hash fill, U[-1,1))",
            "config": {"workload": main_workload, "exchange": exchange_desc,
                       "M": M, "N": N, "K": K, "alpha": 1.0, "beta": 0.0,
                       "rows_per_gpu": Ml, "parallelism": f"rowshard{world}",
                       "l2": "flushed (3x L2 memset) before every timed launch",
                       "timing": "CUDA events around each launch on the launching stream"},
            "roofline": roofline,
            "cublas": {"value": cub_value, "ms_per_step": ms_cub,
                       "paired_ratio_median": statistics.median(ratios) if ratios else None,
                       "call": "cublasGemmEx(CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT)",
                       "note": None if world == 1 else
                       "cuBLAS times this rank's local GEMM only (no exchange)"},
            "median_ms": statistics.median(t_ours),
            "region_ms_incl_flush_and_cublas": region_ms,
            "full_c_bit_identical_to_one_gpu_launch": chk[0] == 0.0,
            "full_c_rel_l2_vs_cublas_max_over_ranks": chk[1],
            "check_rel_l2_vs_cublas": chk[1],
            "device_status": int(st_max),
            "e2e": e2e,
            # our kernels per step: the GEMM; with the peer exchange also the one-warp
            # exit barrier kernel; with NCCL one GEMM per chunk (NCCL's own kernels not counted)
            "gpu_launches": gpu_launches,
            "clocks": clk,
        }
        if c5 is not None:
            line["config5"] = c5
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(Ml, N, K)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
