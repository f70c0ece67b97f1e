#!/usr/bin/env python3
"""Benchmark of the x100-gemm hot path on B200 (one process per GPU).

Default workload (the BASELINE metric's first item, configs[1]): the exact
int8 x int8 -> int32 GEMM C += A.B at M = N = K = 8192 through the tcgen05
kernel of libx100gemm_b200.so.  With --gpus N (under torchrun) B and C are
split by columns across ranks (8192/N columns each, A replicated): total
work is fixed, so scaling is "strong"; no collective touches the data path.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload W]
                  [--impl reference]

Prints ONE JSON line on rank 0.  `value` is whole-job throughput with the
operands resident in HBM (CUDA events on the launching stream, max over
ranks); `e2e` is the same metric through the reference-signature host API
(gemm_ime_i8 with pinned host buffers: H2D of A, B, C and D2H of C inside
the timed region).  --impl reference times the reference's own CPU code
(oracle/_ref/libx100ref.so: the reference's src/gemm_ref.c compiled
unchanged) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "x100-gemm_b200"))
sys.path.insert(0, os.path.join(REPO, "oracle"))
from x100b import shard  # noqa: E402  (how the path splits over GPUs; no device code)

L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="x100", choices=["x100", "reference"])
    ap.add_argument("--workload", default="gemm_i8",
                    choices=["gemm_i8", "gemm_f16", "gemm_f32", "q4gemv", "moe", "decode", "prefill"])
    ap.add_argument("--size", type=int, default=8192, help="M = N = K of the GEMM workloads")
    ap.add_argument("--batch", type=int, default=1, help="tokens per step for q4gemv / moe")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=48, help="layers of the decode / prefill workloads")
    ap.add_argument("--tokens", type=int, default=512, help="prompt tokens of the prefill workload")
    ap.add_argument("--combine", default="p2p", choices=["p2p", "nccl"],
                    help="N > 1 expert-parallel sum: the library's peer-memory kernel or an NCCL all-reduce")
    return ap.parse_args()


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def load_traffic(key):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary
    (profiles/roofline_traffic.txt lines: '<key> <bytes>')."""
    p = os.path.join(REPO, "profiles", "roofline_traffic.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        parts = line.split()
        if len(parts) >= 2 and parts[0] == key:
            try:
                return float(parts[1])
            except ValueError:
                return None
    return None


# ---- clocks --------------------------------------------------------------------
class ClockSampler:
    """SM clock and throttle reasons sampled while the timed region runs:
    NVML every 5 ms (reads only; no setting is changed), else nvidia-smi."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.nvml = None
        self.samples = []
        self.stop_ev = threading.Event()

    def _nvml_loop(self, nv, h):
        names = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                 "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                 "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                 "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
        while not self.stop_ev.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((mhz, {k for k, bit in names.items() if rs & bit}))
            except Exception:  # noqa: BLE001 - sampling is best effort
                pass
            self.stop_ev.wait(0.001)

    def start(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByUUID(self.gpu) if str(self.gpu).startswith("GPU-") else \
                nv.nvmlDeviceGetHandleByIndex(int(self.gpu))
            self.maxmhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self.nvml = nv
            self.th = threading.Thread(target=self._nvml_loop, args=(nv, h), daemon=True)
            self.th.start()
            return
        except Exception:  # noqa: BLE001 - fall back to nvidia-smi
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.nvml is not None:
            self.stop_ev.set()
            self.th.join(timeout=2)
            if not self.samples:
                return None
            reasons = set()
            for _, r in self.samples:
                reasons |= r
            return {"sm_mhz": statistics.median([m for m, _ in self.samples]), "sm_max_mhz": self.maxmhz,
                    "reasons": sorted(reasons), "samples": len(self.samples), "source": "nvml 1 ms"}
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.th.join(timeout=2)
        mhz, maxmhz, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            c = [x.strip() for x in ln.split(",")]
            if len(c) < 9:
                continue
            try:
                mhz.append(float(c[1]))
                maxmhz = float(c[2])
            except ValueError:
                continue
            for nm, v in zip(names, c[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not mhz:
            return None
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": maxmhz, "reasons": sorted(reasons),
                "samples": len(mhz)}


# ---- distributed plumbing ---------------------------------------------------------------
class Dist:
    def __init__(self, n):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world != n:
            raise SystemExit(f"--gpus {n} but WORLD_SIZE={self.world}")

    def init(self):
        import torch
        torch.cuda.set_device(self.local)
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()

    def ep_group(self, max_floats):
        """The library's peer-memory combine for this process group."""
        import x100b

        def exchange(h):
            out = [None] * self.world
            self.pg.all_gather_object(out, h)
            return out
        return x100b.EpGroup(self.world, self.rank, max_floats, exchange)

    def physical_gpu(self):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            ids = [x for x in vis.split(",") if x]
            if self.local < len(ids):
                return ids[self.local]
        return str(self.local)


# ---- CPU baseline (reference code on the host cores) -----------------------------------------
def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def ref_gemm_i8_rows(M, N, K, rows, nthreads):
    """Run the reference's gemm_ref_i8 (oracle/_ref/libx100ref.so) on a
    `rows` x N x K slice of the M x N x K problem, row-sliced over
    `nthreads` host threads; returns (seconds, ops, kind)."""
    import numpy as np
    import py_oracle as po
    ref = po.ref_lib()
    kind = "reference"
    if ref is None:
        kind = "port"
    A = po.rand_i8(11, rows * K).reshape(rows, K)
    B = po.rand_i8(12, K * N).reshape(K, N)
    C = np.zeros((rows, N), np.int32)
    per = [(rows * t) // nthreads for t in range(nthreads + 1)]

    def work(t):
        r0, r1 = per[t], per[t + 1]
        if r1 <= r0:
            return
        a = A[r0:r1]
        c = C[r0:r1]
        if ref is not None:
            ref.gemm_ref_i8(r1 - r0, N, K, a.ctypes.data, B.ctypes.data, c.ctypes.data)
        else:
            po.lib().orc_gemm_i8(r1 - r0, N, K, po._ptr(a), po._ptr(B), po._ptr(c))

    th = [threading.Thread(target=work, args=(t,)) for t in range(nthreads)]
    t0 = time.perf_counter()
    for x in th:
        x.start()
    for x in th:
        x.join()
    dt = time.perf_counter() - t0
    return dt, 2.0 * rows * N * K, kind


def cpu_baseline_gemm_i8(size, target_s=8.0):
    nt = cpu_threads()
    # calibrate on one row per thread, then size the sample for ~target_s
    dt, ops, kind = ref_gemm_i8_rows(size, size, size, nt, nt)
    rate = ops / max(dt, 1e-9)
    rows = int(min(size, max(nt, rate * target_s / (2.0 * size * size))))
    rows = max(nt, rows // nt * nt)
    dt, ops, kind = ref_gemm_i8_rows(size, size, size, rows, nt)
    return {"value": ops / dt / 1e12, "unit": "TOPS", "cores": nt, "kind": kind,
            "sample": f"gemm_ref_i8 on rows 0..{rows - 1} of the {size}^3 problem ({rows}x{size}x{size}), "
                      f"row-sliced over {nt} host threads, {dt:.2f} s"}


# ---- GEMM workloads -----------------------------------------------------------------------
def bench_gemm(args, dist, peaks, peak_src):
    import numpy as np
    import torch
    import x100b

    kind = args.workload
    S = args.size
    world, rank = dist.world, dist.rank
    if S % world:
        raise SystemExit("size must divide by the GPU count")
    M, K = S, S
    n0, n1 = shard.gemm_cols(S, world, rank)
    N = n1 - n0                          # this rank's column slice of B and C
    es = {"gemm_i8": 1, "gemm_f16": 2, "gemm_f32": 4}[kind]
    ce = 2 if kind == "gemm_f16" else 4
    set_bytes = M * K * es + K * N * es + M * N * ce
    nsets = max(1, -(-2 * L2_BYTES // set_bytes))     # rotate so reuse distance > 2 x L2
    nsets = min(nsets, 8)
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    sets = []
    for _ in range(nsets):
        if kind == "gemm_i8":
            A = torch.randint(-128, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
            B = torch.randint(-128, 128, (K, N), dtype=torch.int8, device="cuda", generator=g)
            C = torch.zeros((M, N), dtype=torch.int32, device="cuda")
        else:
            dt_ = torch.float16 if kind == "gemm_f16" else torch.float32
            A = (torch.rand((M, K), device="cuda", generator=g) * 2 - 1).to(dt_)
            B = (torch.rand((K, N), device="cuda", generator=g) * 2 - 1).to(dt_)
            C = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        sets.append((A, B, C))
    fn = {"gemm_i8": "gemm_ime_i8_dev", "gemm_f16": "gemm_f16_f32acc_dev", "gemm_f32": "gemm_f32_dev"}[kind]
    stream = torch.cuda.current_stream()
    L = x100b.lib()
    cfn = getattr(L, fn)
    sptr = stream.cuda_stream

    def step(i):
        A, B, C = sets[i % nsets]
        rc = cfn(M, N, K, A.data_ptr(), B.data_ptr(), C.data_ptr(), sptr)
        if rc:
            raise x100b.X100Error(rc, fn)

    # parity spot-check before timing (tensor cores vs the exact CUDA-core kernel)
    if kind == "gemm_i8":
        A, B, _ = sets[0]
        Ct = torch.zeros((256, N), dtype=torch.int32, device="cuda")
        Cr = torch.zeros_like(Ct)
        x100b.gemm_dev("gemm_ime_i8_dev", A[:256], B, Ct)
        x100b.gemm_dev("gemm_ref_i8_dev", A[:256], B, Cr)
        x100b.sync()
        assert torch.equal(Ct, Cr), "tensor-core GEMM disagrees with the exact kernel"

    for i in range(args.warmup):
        step(i)
    x100b.sync()
    dist.barrier()
    torch.cuda.synchronize()
    clk = ClockSampler(dist.physical_gpu())
    clk.start()
    # two events around the K launches: an event between two launches would
    # serialise them (no programmatic-dependent-launch overlap) and add its own
    # gap, ~3 us per launch at the 8-GPU shard (measured)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    dist.barrier()
    torch.cuda.synchronize()
    ev[0].record(stream)
    for i in range(args.steps):
        step(i)
    ev[1].record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    clocks = clk.stop()
    st = x100b.lib().x100_sync(sptr)
    if st:
        raise x100b.X100Error(st, "device status after timing")
    rank_ms = ev[0].elapsed_time(ev[1])
    total_ms = dist.max(rank_ms)
    ops_rank = 2.0 * M * N * K
    ops_total = 2.0 * S * S * S
    value = ops_total * args.steps / (total_ms / 1e3) / 1e12
    kernel_ms = rank_ms / args.steps           # this rank's average launch, back to back
    achieved = ops_rank / (kernel_ms / 1e3) / 1e12
    if kind == "gemm_i8":
        peak = 2.0 * peaks["bf16_tflops"]
        peak_note = (f"2 x bf16_tflops ({peak_src} MEASURED_PEAKS.json burst): tcgen05 kind::i8 issues at "
                     "twice the kind::f16 dense rate (4.5 vs 2.25 POPS nominal)")
        unit = "TOPS"
    elif kind == "gemm_f16":
        peak = peaks["bf16_tflops"]
        peak_note = f"bf16_tflops ({peak_src} MEASURED_PEAKS.json burst); kind::f16 runs at the bf16 rate"
        unit = "TFLOP/s"
    else:
        # three tf32 products per fp32 product, tf32 issuing at half the
        # kind::f16 rate: the fp32-equivalent ceiling is bf16 / 2 / 3
        peak = peaks["bf16_tflops"] / 6.0
        peak_note = (f"bf16_tflops / 6 ({peak_src} MEASURED_PEAKS.json burst): each fp32 product is three "
                     "kind::tf32 products (hi.hi + hi.lo + lo.hi) and tf32 issues at half the kind::f16 rate")
        unit = "TFLOP/s"
    traffic = load_traffic(f"{kind}_{S}_{world}")

    # ---- end to end through the reference-signature host API ----
    e2e = None
    if kind in ("gemm_i8", "gemm_f32"):
        hostfn = {"gemm_i8": L.gemm_ime_i8, "gemm_f32": L.gemm_rvv_f32}[kind]
        A, B, C = sets[0]
        Ah = torch.empty(A.shape, dtype=A.dtype, pin_memory=True).copy_(A)
        Bh = torch.empty(B.shape, dtype=B.dtype, pin_memory=True).copy_(B)
        Ch = torch.zeros(C.shape, dtype=C.dtype, pin_memory=True)
        e2e_steps = max(3, min(args.steps, 10))
        hostfn(M, N, K, Ah.data_ptr(), Bh.data_ptr(), Ch.data_ptr())        # warm-up
        x100b.check_last("host gemm warm-up")
        dist.barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            hostfn(M, N, K, Ah.data_ptr(), Bh.data_ptr(), Ch.data_ptr())
        x100b.check_last("host gemm")
        dt = dist.max(time.perf_counter() - t0)
        dist.barrier()
        e2e = {"value": ops_total * e2e_steps / dt / 1e12, "unit": unit,
               "h2d_bytes_per_step": int(A.numel() * A.element_size() + B.numel() * B.element_size()
                                         + C.numel() * C.element_size()),
               "d2h_bytes_per_step": int(C.numel() * C.element_size()),
               "steps": e2e_steps,
               "api": f"{hostfn.__name__}(M,N,K,A,B,C) with pinned host buffers (synchronous call)"}

    cpu = None
    if kind == "gemm_i8" and world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline_gemm_i8(S)

    metric = {"gemm_i8": "int8 GEMM TOPS", "gemm_f16": "fp16 GEMM (fp32 accumulate) TFLOP/s",
              "gemm_f32": "fp32 GEMM TFLOP/s"}[kind]
    line = {
        "metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": {"gemm_i8": "int8", "gemm_f16": "fp16", "gemm_f32": "fp32"}[kind],
        "data": "synthetic (uniform int8 in [-128,127] / uniform [-1,1]), generated on device",
        "config": {"workload": f"{kind} C+=A.B M=N=K={S}" + (f", B/C column-sharded 1/{world} per GPU"
                                                              if world > 1 else ""),
                   "M": S, "N": S, "K": S, "parallelism": f"n-shard{world}" if world > 1 else "single",
                   "l2": f"inputs rotate over {nsets} buffer set(s) of {set_bytes / 2**20:.0f} MiB per GPU "
                         f"(> L2 between reuses)"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 1), "unit": unit,
                     "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": peak_note,
                     "kernel": "x100::tc::gemm_tc2_kernel (2-SM, TMA reduce-add epilogue)" if kind != "gemm_f32" else
                               "x100::tc::gemm_tc2_kernel<3> (three kind::tf32 products, 512-k accumulator pieces)",
                     "algorithmic_ops_per_launch": ops_rank,
                     "kernel_ms_mean": round(kernel_ms, 4)},
        "clocks": clocks,
        "e2e": e2e,
        "gpu_launches": args.steps,
        "cpu_baseline": cpu,
    }
    return line



# ---- quantised decode workloads ------------------------------------------------------------
def wellformed_blocks_dev(qtype, nblocks, gen, on_device=False):
    """Random well-formed GGUF blocks built on the device: random payload
    bytes, fp16 scales in the range N(0, 0.02) weights give (host copy, or
    the device tensor with on_device)."""
    import numpy as np
    import torch
    bb = {2: 18, 8: 34, 11: 110, 12: 144}[qtype]
    blk = torch.randint(0, 256, (nblocks, bb), dtype=torch.uint8, device="cuda", generator=gen)
    def f16(lo, hi, sign):
        v = torch.rand(nblocks, device="cuda", generator=gen) * (hi - lo) + lo
        if sign:
            v = v * (torch.randint(0, 2, (nblocks,), device="cuda", generator=gen) * 2 - 1)
        return v.half().view(torch.uint8).view(nblocks, 2)
    if qtype in (2, 8):
        blk[:, 0:2] = f16(0.004, 0.012, True)
    elif qtype == 12:
        blk[:, 0:2] = f16(0.0002, 0.002, False)
        blk[:, 2:4] = f16(0.0, 0.001, False)
    else:
        blk[:, 108:110] = f16(0.0002, 0.002, True)
    if on_device:
        return blk.reshape(-1)
    return np.ascontiguousarray(blk.cpu().numpy().reshape(-1))


def timed_graph(fn, steps, warmup, dist, stream):
    """Warm up, capture one call of fn() in a CUDA graph, replay it `steps`
    times between CUDA events; returns (total_ms, clocks)."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    clk = ClockSampler(dist.physical_gpu())
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    clocks = clk.stop()
    ms = dist.max(e0.elapsed_time(e1))
    del g
    return ms, clocks


def bench_q4gemv(args, dist, peaks, peak_src):
    """Q4_0 6144 x 2048 GEMV at batch B.  64 distinct
    weight copies (453 MB, > L2) are rotated inside one CUDA graph; a step is
    one graph replay = 64 GEMV calls.  The value times independent calls
    (X100Q_GEMV_INDEPENDENT), the way the reference's bench/q4_gemv.c times
    repeated GEMVs; the chain of dependent calls (each waiting for the
    previous kernel, as inside a decode step) is reported beside it."""
    import numpy as np
    import torch
    import x100b
    N, K, B, COPIES = 6144, 2048, args.batch, 64
    gen = torch.Generator(device="cuda").manual_seed(77)
    lins = [x100b.Lin(x100b.Q4_0, N, K, wellformed_blocks_dev(2, N * K // 32, gen)) for _ in range(COPIES)]
    xs = torch.randn((COPIES, B, K), device="cuda", generator=gen)
    ys = torch.empty((COPIES, B, N), device="cuda")
    stream = torch.cuda.Stream()
    L = x100b.lib()

    def make_run(flags):
        def run():
            s = torch.cuda.current_stream().cuda_stream
            for c in range(COPIES):
                rc = L.x100q_lin_gemv_dev_flags(lins[c].h, xs[c].data_ptr(), ys[c].data_ptr(), B, flags, s)
                if rc:
                    raise x100b.X100Error(rc, "x100q_lin_gemv_dev_flags")
        return run
    with torch.cuda.stream(stream):
        ms_chain, _ = timed_graph(make_run(0), args.steps, args.warmup, dist, stream)
        ms, clocks = timed_graph(make_run(1), args.steps, args.warmup, dist, stream)
    calls = args.steps * COPIES
    wbytes = N * K // 32 * 18
    alg = wbytes + B * (4 * K + 4 * N)
    per_call_s = ms / 1e3 / calls
    gbs = alg / per_call_s / 1e9
    chain_gbs = alg / (ms_chain / 1e3 / calls) / 1e9
    # parity spot check of the last outputs against the oracle
    import py_oracle as po  # checker only
    blk = wellformed_blocks_dev(2, N * K // 32, torch.Generator(device="cuda").manual_seed(5))
    chk = x100b.Lin(x100b.Q4_0, N, K, blk)
    xh = np.random.default_rng(1).normal(0, 1, size=(B, K)).astype(np.float32)
    yh = np.empty((B, N), np.float32)
    chk.gemv(xh, yh, B)
    err = po.rel_l2(yh, po.qgemv(po.Q4_0, blk, N, K, xh, nthreads=cpu_threads()))
    assert err <= 1e-3, err
    # e2e: host x in pinned memory -> y on host, through the synchronous API
    xh_p = torch.empty((B, K), pin_memory=True).copy_(xs[0])
    yh_p = torch.empty((B, N), pin_memory=True)
    for _ in range(5):
        L.x100q_lin_gemv(lins[0].h, xh_p.data_ptr(), yh_p.data_ptr(), B)
    e2e_steps = 200
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        rc = L.x100q_lin_gemv(lins[i % COPIES].h, xh_p.data_ptr(), yh_p.data_ptr(), B)
    dt = dist.max(time.perf_counter() - t0)
    if rc:
        raise x100b.X100Error(rc, "x100q_lin_gemv")
    cpu = None
    if dist.world == 1 and not args.no_cpu_baseline:
        nt = cpu_threads()
        reps = 20
        t0 = time.perf_counter()
        for _ in range(reps):
            po.qgemv(po.Q4_0, blk, N, K, xh, nthreads=nt)
        cdt = (time.perf_counter() - t0) / reps
        cpu = {"value": round(alg / cdt / 1e9, 3), "unit": "GB/s", "cores": nt, "kind": "port",
               "sample": f"oracle scalar dequant-GEMV (restates qwen_moe.c:164-165 + fp32 dot) on the full "
                         f"{N}x{K} Q4_0 matrix, batch {B}, {reps} reps, row-sliced over {nt} threads"}
    return {
        "metric": "Q4_0 dequant-GEMV HBM GB/s", "value": round(gbs * dist.world, 2), "unit": "GB/s",
        "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": "q4_0 weights, fp32 activations (int32 dot products on 16-bit split x: " +
                 ("dp4a)" if B <= 4 else "integer mma.sync)"),
        "data": "synthetic random well-formed Q4_0 blocks, x ~ N(0,1)",
        "config": {"workload": f"Q4_0 GEMV y=W.x W {N}x{K} batch {B}", "N": N, "K": K, "batch": B,
                   "l2": f"{COPIES} weight copies rotated per step ({COPIES * wbytes / 2**20:.0f} MiB > L2)",
                   "graph": f"one CUDA graph of {COPIES} GEMV launches per step",
                   "calls": "independent (X100Q_GEMV_INDEPENDENT), as the reference's bench/q4_gemv.c repeats "
                            "its GEMV; the dependent chain is roofline.dependent_chain"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": load_traffic(f"q4gemv_b{B}"),
                     "peak_source": f"hbm_gbs ({peak_src} MEASURED_PEAKS.json)",
                     # independent calls of up to 4 tokens run on the dp4a kernel, larger
                     # batches on the tensor-core kernel (the dependent chain: 2+ tokens)
                     "kernel": ("x100::q::qgemv_kernel<Q4_0> (dp4a)" if B <= 4 else
                                "x100::q::qgemv_mma_kernel<Q4_0> (integer mma.sync)"),
                     "algorithmic_bytes_per_launch": alg,
                     "kernel_us_mean": round(per_call_s * 1e6, 3), "parity_rel_l2": err,
                     "dependent_chain": {"achieved": round(chain_gbs, 1),
                                         "frac": round(chain_gbs / peaks["hbm_gbs"], 4),
                                         "kernel_us_mean": round(ms_chain * 1e3 / calls, 3),
                                         "note": "each call waits for the previous kernel (decode-step order)"}},
        "clocks": clocks,
        "e2e": {"value": round(alg * e2e_steps / dt / 1e9, 3), "unit": "GB/s",
                "h2d_bytes_per_step": 4 * B * K, "d2h_bytes_per_step": 4 * B * N,
                "api": "x100q_lin_gemv(lin, x, y, batch) with pinned host x, y (synchronous)"},
        "gpu_launches": calls,
        "cpu_baseline": cpu,
    }


def bench_moe(args, dist, peaks, peak_src):
    """one MoE layer (d 2048, 128 experts, top-8, ffn 768,
    Q4_K).  Each rank holds 128/N experts (expert parallel) and the full
    router; per step every rank runs the layer for `batch` tokens and the
    partial outputs are summed with an NCCL all-reduce."""
    import numpy as np
    import torch
    import x100b
    d, E, k, ffn, B = 2048, 128, 8, 768, args.batch
    world, rank = dist.world, dist.rank
    lo, hi = shard.expert_slice(E, world, rank)
    gen = torch.Generator(device="cuda").manual_seed(99)
    router = (torch.randn((E, d), device="cuda", generator=gen) * 0.02).cpu().numpy()
    nb_d = ffn * d // 256
    layers = []
    host0 = None
    LAYERS = 8          # 8 copies x 340 MB of experts: no expert is re-read from L2 between its uses
    for li in range(LAYERS):
        # full-size tensors, only the local slice [lo, hi) is uploaded
        gate = np.zeros(E * nb_d * 144, np.uint8)
        up = np.zeros_like(gate)
        down = np.zeros_like(gate)
        sl = slice(lo * nb_d * 144, hi * nb_d * 144)
        gate[sl] = wellformed_blocks_dev(12, (hi - lo) * nb_d, gen)
        up[sl] = wellformed_blocks_dev(12, (hi - lo) * nb_d, gen)
        down[sl] = wellformed_blocks_dev(12, (hi - lo) * nb_d, gen)
        layers.append(x100b.Moe(d, E, k, ffn, x100b.Q4_K, router, gate, up, down, lo, hi))
        if li == 0:
            host0 = (gate, up, down)
    POOL = 64
    hns = torch.randn((POOL, B, d), device="cuda", generator=gen)
    out = torch.empty((POOL, B, d), device="cuda")
    L = x100b.lib()
    stream = torch.cuda.Stream()
    state = {"i": 0}

    ep = dist.ep_group(B * d) if world > 1 and args.combine == "p2p" else None

    def one(i):
        s = torch.cuda.current_stream().cuda_stream
        rc = L.x100q_moe_ffn_dev(layers[i % LAYERS].h, hns[i % POOL].data_ptr(), out[i % POOL].data_ptr(), B,
                                 None, None, s)
        if rc:
            raise x100b.X100Error(rc, "x100q_moe_ffn_dev")
        if ep is not None:
            ep.allreduce_dev(out[i % POOL], out[i % POOL], B * d)
        elif world > 1:
            dist.pg.all_reduce(out[i % POOL])

    PER = 16   # MoE calls per captured graph (each a different hn, layer copy)

    def run():
        for j in range(PER):
            one(j)
    with torch.cuda.stream(stream):
        # N > 1: the NCCL all-reduces are captured in the same CUDA graph
        # (the warm-up calls initialise the communicator first)
        ms, clocks = timed_graph(run, args.steps, args.warmup, dist, stream)
        calls = args.steps * PER
    tok_s = calls * B / (ms / 1e3)
    # Algorithmic bytes of one call: the experts its tokens select, each
    # streamed once however many of the tokens share it (the measured union
    # U, read back from the library's own routing of that call's tokens),
    # plus the 1 MB fp32 router (read every call; with the expert stream in
    # between it is not L2-resident) and the tokens' activations in and out.
    EXPERT_BYTES, ROUTER_BYTES = 2654208, 4 * E * d
    sel_t = torch.empty((B, k), dtype=torch.int32, device="cuda")
    scratch_out = torch.empty((B, d), device="cuda")
    unions = []
    for j in range(PER):
        layers[j % LAYERS].ffn_dev(hns[j % POOL], scratch_out, B, sel_t)
        torch.cuda.synchronize()
        unions.append(len(set(sel_t.cpu().numpy().reshape(-1).tolist())))
    alg_call = [u * EXPERT_BYTES + ROUTER_BYTES + B * 2 * 4 * d for u in unions]
    per_call_us = ms * 1e3 / calls
    achieved = sum(alg_call) / PER / (per_call_us / 1e6) / 1e9 / world   # per-GPU share
    # parity of one step against the oracle on the same weights (1 GPU only)
    err = None
    if world == 1:
        import py_oracle as po  # checker only
        hh = hns[0].cpu().numpy()
        eo, sel, _ = layers[0].ffn_host(hh)
        ref, rsel, _ = po.moe_ffn(d, E, k, ffn, po.Q4_K, router, *host0, hh, nthreads=cpu_threads())
        assert np.array_equal(sel, rsel), "expert selection differs from the oracle"
        err = po.rel_l2(eo, ref)
        assert err <= 1e-3, err
    # e2e through the synchronous host API
    hn_p = torch.empty((B, d), pin_memory=True).copy_(hns[0])
    eo_p = torch.empty((B, d), pin_memory=True)
    for _ in range(5):
        L.x100q_moe_ffn(layers[0].h, hn_p.data_ptr(), eo_p.data_ptr(), B, None, None)
    e2e_steps = 100
    dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        rc = L.x100q_moe_ffn(layers[i % LAYERS].h, hn_p.data_ptr(), eo_p.data_ptr(), B, None, None)
        if world > 1:
            t = torch.from_numpy(eo_p.numpy()).cuda()
            dist.pg.all_reduce(t)
            eo_p.copy_(t)
    dt = dist.max(time.perf_counter() - t0)
    if rc:
        raise x100b.X100Error(rc, "x100q_moe_ffn")
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        import py_oracle as po
        rng = np.random.default_rng(0)
        nt = cpu_threads()
        hh = rng.normal(0, 1, size=(1, d)).astype(np.float32)
        t0 = time.perf_counter()
        reps = 3
        for _ in range(reps):
            po.moe_ffn(d, E, k, ffn, po.Q4_K, router, *host0, hh, nthreads=nt)
        cdt = (time.perf_counter() - t0) / reps
        cpu = {"value": round(1.0 / cdt, 3), "unit": "tokens/s", "cores": nt, "kind": "port",
               "sample": f"oracle MoE block (restates qwen_moe.c:295-311, fp32 router, exact SiLU) for one "
                         f"token through the same {E}-expert Q4_K layer, {reps} reps, GEMV rows over {nt} threads"}
    return {
        "metric": "Q4_K MoE layer decode tokens/s", "value": round(tok_s, 1), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "q4_k weights, fp32 activations",
        "data": "synthetic: random well-formed Q4_K expert blocks, fp32 router N(0,0.02), hn ~ N(0,1)",
        "config": {"workload": f"MoE layer d={d} experts={E} top-{k} ffn={ffn} Q4_K, batch {B}",
                   "batch": B, "expert_parallel": f"{E // world} experts per GPU",
                   "l2": f"{LAYERS} layer copies ({LAYERS * E * 2654208 / 2**30:.2f} GiB of experts) x "
                         f"{PER} hn batches rotated",
                   "graph": f"{PER} MoE calls per CUDA graph" + ("" if world == 1 else
                                                                  f", each followed by the {args.combine} sum of eout")},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": load_traffic(f"moe_b{B}"),
                     "peak_source": f"hbm_gbs ({peak_src} MEASURED_PEAKS.json)",
                     "kernel": ("router_logits + moe_fused (2 launches per call)" if B == 1 else
                                "router_logits + route_group + gate_up_ws + prep_slots + down_ws + combine "
                                "(6 launches per call)"),
                     "algorithmic_bytes_per_call": round(sum(alg_call) / PER),
                     "expert_union_mean": round(sum(unions) / PER, 2),
                     "bytes_rule": "U * 2654208 (distinct experts of the call's tokens) + 1048576 router + "
                                   "B * 16384 activations",
                     "call_us_mean": round(per_call_us, 3),
                     "parity": err},
        "clocks": clocks,
        "e2e": {"value": round(e2e_steps * B / dt, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": 4 * B * d, "d2h_bytes_per_step": 4 * B * d,
                "api": "x100q_moe_ffn(moe, hn, eout, batch) with pinned host hn, eout (synchronous)"},
        "gpu_launches": calls * ((2 if B == 1 else 6) + (1 if ep is not None else 0)),
        "cpu_baseline": cpu,
    }


def bench_reference(args):
    """--impl reference: the reference's own CPU GEMM on this host's cores."""
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    S = args.size
    nt = cpu_threads()
    vals = []
    for i in range(args.warmup + args.steps):
        rows = nt * 2
        dt, ops, kind = ref_gemm_i8_rows(S, S, S, rows, nt)
        if i >= args.warmup:
            vals.append(ops / dt / 1e12)
    v = statistics.mean(vals)
    return {
        "impl": "reference", "metric": "int8 GEMM TOPS", "value": v, "unit": "TOPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": f"gemm_i8 C+=A.B M=N=K={S}", "M": S, "N": S, "K": S},
        "cpu_baseline": {"value": v, "unit": "TOPS", "cores": nt, "kind": kind,
                         "sample": f"each step: gemm_ref_i8 (reference src/gemm_ref.c) on {2 * nt} rows of "
                                   f"the {S}^3 problem, row-sliced over {nt} host threads"},
        "e2e": {"value": v, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---- full decode step ---------------------------------------------------------------------
DEC = dict(d=2048, n_heads=32, n_kv_heads=4, head_dim=128, vocab=151936, n_exp=128, n_act=8, moe_ffn=768,
           attn_qtype=8, expert_qtype=11, lm_qtype=8, ctx=4096, rope_base=1e6, eps=1e-6)


def bench_decode(args, dist, peaks, peak_src):
    """a 48-layer Qwen3-30B-A3B-shaped decode step (GQA
    32/4 heads of 128, RMSNorm, QK-norm, NEOX RoPE 1e6, Q8_0 attention, fp32
    router, top-8 of 128 Q3_K SwiGLU experts of 768, Q8_0 lm_head over 151936
    tokens), `batch` sequences each attending over a 4096-position fp16 KV
    cache (positions 0..4094 random, the step's token at 4095).  All weights
    random-init on the device.  One step = embed + 48 layers + head for every
    sequence; expert parallel over N GPUs (each rank holds 128/N experts and
    sums the experts' outputs with an NCCL all-reduce per layer)."""
    import numpy as np
    import torch
    import x100b
    B, NL = args.batch, args.layers
    world, rank = dist.world, dist.rank
    c = dict(DEC)
    d, qd, kvd, E, F, V = c["d"], c["n_heads"] * 128, c["n_kv_heads"] * 128, c["n_exp"], c["moe_ffn"], c["vocab"]
    lo, hi = shard.expert_slice(E, world, rank)
    m = x100b.Model(n_layers=NL, max_batch=B, expert_lo=lo, expert_hi=hi, **c)
    gen = torch.Generator(device="cuda").manual_seed(55)
    blk = lambda qt, n: wellformed_blocks_dev(qt, n, gen, on_device=True)   # noqa: E731
    nrm = lambda n: (1 + 0.1 * torch.randn(n, device="cuda", generator=gen)).contiguous()   # noqa: E731
    host_layers = []
    for li in range(NL):
        lw = dict(attn_norm=nrm(d), wq=blk(8, qd * d // 32), wk=blk(8, kvd * d // 32), wv=blk(8, kvd * d // 32),
                  q_norm=nrm(128), k_norm=nrm(128), wo=blk(8, d * qd // 32), ffn_norm=nrm(d),
                  router=(0.02 * torch.randn((E, d), device="cuda", generator=gen)).contiguous(),
                  gate=blk(11, E * F * d // 256), up=blk(11, E * F * d // 256), down=blk(11, E * d * F // 256))
        m.set_layer(li, *(lw[k] for k in ("attn_norm", "wq", "wk", "wv", "q_norm", "k_norm", "wo", "ffn_norm",
                                          "router", "gate", "up", "down")))
        if li < 2 and world == 1:
            host_layers.append({k: v.cpu().numpy() for k, v in lw.items()})
        del lw
    emb = torch.randn((V, d), device="cuda", generator=gen)
    out_norm = nrm(d)
    lm = blk(8, V * d // 32)
    m.set_output(emb, out_norm, lm)
    # KV cache: random fp16 for positions 0..4094 of every layer and slot
    P = c["ctx"] - 1
    kvk = (torch.randn((c["n_kv_heads"], P, 128), device="cuda", generator=gen)).half()
    kvv = (torch.randn((c["n_kv_heads"], P, 128), device="cuda", generator=gen)).half()
    for li in range(NL):
        for sl in range(B):
            m.kv_write(li, sl, 0, kvk, kvv)
    torch.cuda.synchronize()
    toks = torch.randint(0, V, (B,), dtype=torch.int32, device="cuda", generator=gen)
    pos = torch.full((B,), P, dtype=torch.int32, device="cuda")
    h = torch.empty((B, d), device="cuda")
    logits = torch.empty((B, V), device="cuda")
    eout = torch.empty((B, d), device="cuda")
    stream = torch.cuda.Stream()
    ep = dist.ep_group(B * d) if world > 1 and args.combine == "p2p" else None
    # launches per step: embed; per layer the q/k/v GEMV, attention and the
    # merge of its splits, the Wo GEMV (two launches above 8 tokens: the
    # 4096-wide activations of 16 tokens exceed one CTA's shared memory, so
    # the row is taken in two K pieces; its activations are prepared by the
    # attention merge), the MoE kernels (2 fused at batch 1; 6 grouped: router,
    # grouping, gate/up, h preparation, down, combine); above one token the
    # q/k/v and lm_head tensor-core GEMV calls add their activation-preparation
    # kernel -- in the one-process step (forward_dev) only layer 0's q/k/v, the
    # others and the lm_head's being prepared by the MoE combine before them;
    # the lm_head
    prep = 0 if B == 1 else 1
    chained = world == 1
    launches = (1 + NL * (1 + 2 + (1 if B <= 8 else 2) + (2 if B == 1 else 6) + (1 if ep is not None else 0))
                + prep * (1 if chained else NL) + 1 + (0 if chained else prep))

    def step():
        if world == 1:
            m.forward_dev(toks, h, pos, logits, B)
            return
        m.embed_dev(toks, h, B)
        for li in range(NL):
            m.layer_dev(li, h, pos, B, eout=eout)
            if ep is not None:
                ep.allreduce_dev(eout, h, B * d, accum=True)   # h += sum of the experts' shares
            else:
                dist.pg.all_reduce(eout)
                h.add_(eout)
        m.head_dev(h, logits, B)

    # routing of one step (per-layer expert unions for the algorithmic bytes)
    with torch.cuda.stream(stream):
        sel = torch.empty((NL, B, c["n_act"]), dtype=torch.int32, device="cuda")
        m.embed_dev(toks, h, B)
        for li in range(NL):
            if world == 1:
                m.layer_dev(li, h, pos, B, sel=sel[li])
            else:
                m.layer_dev(li, h, pos, B, eout=eout, sel=sel[li])
                if ep is not None:
                    ep.allreduce_dev(eout, h, B * d, accum=True)
                else:
                    dist.pg.all_reduce(eout)
                    h.add_(eout)
        torch.cuda.synchronize()
    selh = sel.cpu().numpy()
    union = [len(set(int(e) for e in selh[li].reshape(-1) if lo <= e < hi)) for li in range(NL)]
    attn_b = (qd + 2 * kvd) * d // 32 * 34 + d * qd // 32 * 34
    exp_b = 3 * F * d // 256 * 110
    kv_b = B * (P + 1) * kvd * 2 * 2
    norms_b = (2 * d + 2 * 128) * 4
    step_bytes = sum(attn_b + E * d * 4 + u * exp_b + kv_b + norms_b for u in union) + V * d // 32 * 34 + d * 4 + \
        B * d * 4
    with torch.cuda.stream(stream):
        ms, clocks = timed_graph(step, args.steps, args.warmup, dist, stream)
    step_ms = ms / args.steps
    tok_s = B / (step_ms / 1e3)
    gbs = step_bytes / (step_ms / 1e3) / 1e9
    err = None
    cpu = None
    if world == 1:
        import py_oracle as po   # checker only
        nt = cpu_threads()
        kvk_h = kvk.cpu().numpy().view(np.uint16)
        kvv_h = kvv.cpu().numpy().view(np.uint16)
        ocfg = dict(c, ctx=c["ctx"])

        def oracle_cache():
            kc = np.zeros((c["n_kv_heads"], c["ctx"], 128), np.uint16)
            vc = np.zeros_like(kc)
            kc[:, :P], vc[:, :P] = kvk_h, kvv_h
            return kc, vc
        # parity: layer 0 of slot 0 on the GPU against the oracle
        with torch.cuda.stream(stream):
            m.embed_dev(toks, h, B)
            h0 = h[0].cpu().numpy().copy()
            m.layer_dev(0, h, pos, B)
            torch.cuda.synchronize()
        kc, vc = oracle_cache()
        href = h0.copy()
        po.decode_layer(ocfg, host_layers[0], kc, vc, href, P, nthreads=nt)
        err = po.rel_l2(h[0].cpu().numpy(), href)
        assert err <= 1e-3, err
        if not args.no_cpu_baseline:
            hh = h0.copy()
            t0 = time.perf_counter()
            for li in range(2):
                kc, vc = oracle_cache()
                po.decode_layer(ocfg, host_layers[li], kc, vc, hh, P, nthreads=nt)
            t_layers = time.perf_counter() - t0
            lm_h = lm.cpu().numpy()
            t0 = time.perf_counter()
            po.decode_head(dict(c), out_norm.cpu().numpy(), lm_h, hh, nthreads=nt)
            t_head = time.perf_counter() - t0
            t_tok = t_layers / 2 * NL + t_head
            cpu = {"value": round(1.0 / t_tok, 4), "unit": "tokens/s", "cores": nt, "kind": "port",
                   "sample": f"oracle forward() restatement (qwen_moe_q3k.c:1842-1983) for one token: 2 of the "
                             f"{NL} layers ({t_layers:.2f} s) + output norm and lm_head ({t_head:.2f} s), "
                             f"scaled to {NL} layers; GEMV rows over {nt} threads"}
    # e2e: the synchronous host call (tokens, pos on the host -> logits on the host)
    e2e = None
    if world == 1:
        tok_p = toks.cpu().numpy()
        pos_p = pos.cpu().numpy()
        m.forward(tok_p, pos_p)
        n_e2e = 10
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            m.forward(tok_p, pos_p)
        dt = time.perf_counter() - t0
        e2e = {"value": round(n_e2e * B / dt, 2), "unit": "tokens/s", "h2d_bytes_per_step": 8 * B,
               "d2h_bytes_per_step": 4 * B * V,
               "api": "x100q_model_forward(model, tokens, pos, logits, batch) with host tokens/pos/logits"}
    # per-bucket step times (x100q_model_timing: the reference's decode buckets,
    # qwen_moe_q3k.c:910-941), from a few eager steps after the timed ones
    buckets = None
    if world == 1:
        m.timing(True)
        with torch.cuda.stream(stream):
            for _ in range(3):
                step()
            torch.cuda.synchronize()
        tms, tsteps = m.timing_read()
        m.timing(False)
        buckets = {k: round(v / tsteps, 4) for k, v in tms.items()}
        buckets["sum"] = round(sum(tms.values()) / tsteps, 4)
    return {
        "metric": "decode tokens/s (48-layer Qwen3-30B-A3B-shaped step)", "value": round(tok_s, 2),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "q8_0/q3_k weights, fp32 activations, fp16 KV",
        "data": "synthetic: random well-formed Q8_0 / Q3_K blocks, fp32 router N(0,0.02), norms 1+N(0,0.1), "
                "embeddings N(0,1), KV cache N(0,1) fp16",
        "config": {"workload": f"decode step {NL} layers, batch {B}, context 4096, GQA 32/4x128, "
                               f"Q8_0 attention, 128 Q3_K experts top-8 ffn 768, Q8_0 lm_head 151936",
                   "batch": B, "layers": NL, "context": P + 1,
                   "expert_parallel": f"{E // world} experts per GPU",
                   "l2": f"weights {step_bytes / 2**30:.2f} GiB per step (> L2)",
                   "graph": "one CUDA graph per step" + ("" if world == 1 else
                                                          f" ({args.combine} sum of the experts' output per layer inside)")},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": None,
                     "peak_source": f"hbm_gbs ({peak_src} MEASURED_PEAKS.json)",
                     "kernel": "whole step (qgemv, attn_decode, router, moe kernels)",
                     "algorithmic_bytes_per_step": step_bytes,
                     "expert_union_mean": round(float(np.mean(union)), 2), "parity_rel_l2_layer0": err},
        "buckets_ms_per_step": buckets,
        "buckets_note": "x100q_model_timing over 3 eager steps (events at bucket boundaries serialise the "
                        "kernels around them, so the sum exceeds ms_per_step slightly)",
        "clocks": clocks,
        "e2e": e2e,
        "gpu_launches": launches * args.steps,
        "cpu_baseline": cpu,
    }


def prefill_launches(n, NL, chunk=1024, max_batch=16, ctx=4096, kc=64):
    """Kernel launches of one x100q_model_prefill of n tokens at positions 0 ..
    n-1 without logits (decode.cu prefill_chunk_tc): per chunk the embedding,
    and per layer the q/k/v linear (split + GEMM), the k/v cache write, the
    attention groups (attention + split merge each; groups sized as the
    library sizes them), the Wo linear (split + GEMM) and the MoE (split,
    router, count, scatter, gate/up GEMM, swiglu split, down GEMM, combine)."""
    cap = max_batch * ((ctx + kc - 1) // kc)
    total = 0
    for c0 in range(0, n, chunk):
        T = min(chunk, n - c0)
        attn, g0 = 0, 0
        while g0 < T:
            gb = T - g0
            nsp = (c0 + g0 + gb - 1 + kc) // kc
            while gb > 1 and gb * nsp > cap:
                gb = max(1, cap // nsp if cap // nsp < gb else gb - 1)
                nsp = (c0 + g0 + gb - 1 + kc) // kc
            attn += 1 + (1 if nsp > 1 else 0)
            g0 += gb
        total += 1 + NL * (2 + 1 + attn + 2 + 8)
    return total


def bench_prefill(args, dist, peaks, peak_src):
    """Prefill of a prompt into one sequence of the config-5 model (48 layers,
    Q8_0 attention, 128 Q3_K experts, fp16 KV cache of 4096): x100q_model_prefill
    with n tokens > max_batch, the chunked tensor-core path (chunks of 1024
    tokens: the q/k/v, Wo and expert linears as tcgen05 dequant GEMMs, the
    experts grouped by the chunk's routing).  One step = one prefill of the
    whole prompt at positions 0 .. n-1 of slot 0, without logits (a prompt's
    logits are not needed).  1 GPU; the host call is synchronous, so the step
    is timed on the host clock around it."""
    import numpy as np
    import torch
    import x100b
    if dist.world > 1:
        raise SystemExit("prefill workload: 1 GPU (the prefill path does not shard)")
    NL, n = args.layers, args.tokens
    c = dict(DEC)
    d, qd, kvd, E, F, V = c["d"], c["n_heads"] * 128, c["n_kv_heads"] * 128, c["n_exp"], c["moe_ffn"], c["vocab"]
    m = x100b.Model(n_layers=NL, max_batch=16, expert_lo=0, expert_hi=E, **c)
    gen = torch.Generator(device="cuda").manual_seed(56)
    blk = lambda qt, k: wellformed_blocks_dev(qt, k, gen, on_device=True)   # noqa: E731
    nrm = lambda k: (1 + 0.1 * torch.randn(k, device="cuda", generator=gen)).contiguous()   # noqa: E731
    for li in range(NL):
        lw = dict(attn_norm=nrm(d), wq=blk(8, qd * d // 32), wk=blk(8, kvd * d // 32), wv=blk(8, kvd * d // 32),
                  q_norm=nrm(128), k_norm=nrm(128), wo=blk(8, d * qd // 32), ffn_norm=nrm(d),
                  router=(0.02 * torch.randn((E, d), device="cuda", generator=gen)).contiguous(),
                  gate=blk(11, E * F * d // 256), up=blk(11, E * F * d // 256), down=blk(11, E * d * F // 256))
        m.set_layer(li, *(lw[k] for k in ("attn_norm", "wq", "wk", "wv", "q_norm", "k_norm", "wo", "ffn_norm",
                                          "router", "gate", "up", "down")))
        del lw
    m.set_output(torch.randn((V, d), device="cuda", generator=gen), nrm(d), blk(8, V * d // 32))
    torch.cuda.synchronize()
    toks = np.random.default_rng(3).integers(0, V, size=n).astype(np.int32)
    toks_p = torch.from_numpy(toks).pin_memory()
    for _ in range(args.warmup):
        m.prefill(0, toks_p.numpy(), 0, logits=False)
    clk = ClockSampler(dist.physical_gpu())
    clk.start()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        m.prefill(0, toks_p.numpy(), 0, logits=False)
    dt = time.perf_counter() - t0
    clocks = clk.stop()
    step_ms = dt * 1e3 / args.steps
    tok_s = n / (step_ms / 1e3)
    # algorithmic work of one prompt: 2 flops per weight per token (q/k/v, Wo,
    # the token's 8 experts), the single product (the kernel issues three to
    # carry 22-bit operands); attention over the causal prefix
    params_tok = (qd + 2 * kvd) * d + d * qd + c["n_act"] * 3 * F * d
    flops = 2.0 * n * NL * params_tok + NL * 4.0 * c["n_heads"] * 128 * n * (n + 1) / 2
    tflops = flops / (step_ms / 1e3) / 1e12
    peak = peaks["bf16_tflops"]
    return {
        "metric": "prefill tokens/s (config-5 model)", "value": round(tok_s, 1), "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 3),
        "higher_is_better": True, "scaling": "none", "vs_baseline": None,
        "dtype": "q8_0 / q3_k weights, fp16 hi+lo operands on kind::f16, fp32 accumulate",
        "data": "synthetic: random well-formed blocks, fp32 router N(0,0.02), random token ids",
        "config": {"workload": f"prefill {n} tokens into one sequence, {NL} layers, Q8_0 attention, 128 Q3_K "
                               f"experts top-8, chunks of 256 tokens", "tokens": n, "layers": NL,
                   "timing": "host clock around the synchronous x100q_model_prefill call (syncs per chunk)",
                   "l2": f"weights {NL * ((qd + 2 * kvd) * d + d * qd) * 34 / 32 / 2**30 + NL * E * 3 * F * d * 110 / 256 / 2**30:.1f} GiB per prompt (> L2)"},
        "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(tflops / peak, 4), "traffic": None,
                     "peak_source": f"bf16_tflops ({peak_src} MEASURED_PEAKS.json)",
                     "kernel": "whole prefill (algorithmic flops: one product per weight and token; the dequant "
                               "GEMM issues three kind::f16 products)",
                     "algorithmic_flops_per_step": flops},
        "clocks": clocks,
        "e2e": {"value": round(tok_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": 4 * n, "d2h_bytes_per_step": 0,
                "api": "x100q_model_prefill(model, slot, tokens, n, pos0, NULL) with pinned host tokens"},
        "gpu_launches": prefill_launches(n, NL) * args.steps,
        "cpu_baseline": None,
    }


def main():
    args = parse()
    if args.impl == "reference":
        line = bench_reference(args)
        if line:
            print(json.dumps(line))
        return
    dist = Dist(args.gpus)
    dist.init()
    peaks, src = load_peaks()
    try:
        if args.workload.startswith("gemm"):
            line = bench_gemm(args, dist, peaks, src)
        elif args.workload == "q4gemv":
            line = bench_q4gemv(args, dist, peaks, src)
        elif args.workload == "decode":
            line = bench_decode(args, dist, peaks, src)
        elif args.workload == "prefill":
            line = bench_prefill(args, dist, peaks, src)
        else:
            line = bench_moe(args, dist, peaks, src)
    finally:
        dist.close()
    if dist.rank == 0:
        print(json.dumps(line))


if __name__ == "__main__":
    main()
