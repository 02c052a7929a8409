#!/usr/bin/env python
"""Benchmark of the batched slogpf / slogdet path on 1..8 B200s.

Default workload (the headline configuration): slogpf forward + VJP of logabs, float32,
batch 4096 of skew-symmetric S = A - A^T, A 128x128 iid N(0,1), prec="tf32x3". One step
is one pass over the batch: sign, logabs and the gradient S^-T/2 of sum(logabs) from one
fused launch through the C ABI (fermix_slogpf_grad). Scaling is weak: each rank
factorises its own batch, no collective on the data path; the timed region is bracketed
by barriers and the max over ranks is reported.

    python bench.py [--gpus N --steps K --warmup W]
    python bench.py --impl reference ...   # the reference's CPU path (the oracle port)

Prints one JSON line on rank 0.
"""

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "slogdet/slogpf matrices/sec fwd & fwd+bwd at 1-8 B200; % of roofline"
SMALL_KERNEL = {"slogpf": "pf_small_kernel", "slogdet": "lu_small_kernel"}
TC_KERNEL = {"slogpf": "pf_tc_kernel", "slogdet": "lu_tc_kernel"}


def kernel_name(a):
    """The dominant kernel of this workload: the tensor-memory kernels for float32 (slogpf
    8 <= n <= 128, even n; slogdet 8 <= n <= 256; both precisions: tcgen05 block updates
    under tf32x3, FMA ones under ieee), the register-panel kernels otherwise up to n = 256,
    and above that the blocked engines' trailing update (tcgen05 for float32 / complex64
    under tf32x3, DMMA for complex128, FMA tiles otherwise)."""
    if a.dtype == "f32" and a.n >= 8:
        if a.op == "slogpf" and a.n <= 128 and a.n % 2 == 0:
            return TC_KERNEL[a.op]
        if a.op == "slogdet" and a.n <= 256:
            return TC_KERNEL[a.op]
    if a.n <= 256:
        return SMALL_KERNEL[a.op]
    if a.dtype in ("f32", "c64") and a.prec == "tf32x3":
        return "lg_tc_update_kernel"
    return "lg_dmma_update_kernel" if a.dtype == "c128" else "lg_update_kernel"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="fermix_b200", choices=["fermix_b200", "reference"])
    ap.add_argument("--op", default="slogpf", choices=["slogpf", "slogdet"])
    ap.add_argument("--fwd-only", action="store_true", help="forward only (default: forward + VJP)")
    ap.add_argument("--batch", type=int, default=4096, help="matrices per GPU")
    ap.add_argument("--n", type=int, default=128)
    ap.add_argument("--dtype", default="f32", choices=["f32", "f64", "c64", "c128"])
    ap.add_argument("--prec", default="tf32x3", choices=["tf32x3", "ieee"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-sample", type=int, default=1536,
                    help="matrices in the CPU baseline sample (about 10-20 s of host work at the default workload)")
    ap.add_argument("--ref-step", type=int, default=16, help="matrices per step of the reference arm")
    ap.add_argument("--gather", type=int, default=0, metavar="SITES",
                    help="slogdet only: matrices are rows of a shared (SITES x n) phi picked by random occupations "
                         "(fermix_slogdet_gather, configuration 3's caller step); L2 flushed between timed steps")
    ap.add_argument("--move", type=int, default=0, metavar="K",
                    help="time a move instead: --op slogdet: fermix_slogdet_update (k-row ratio + in-place Woodbury "
                         "update of G = A^-T); --op slogpf (K = 1): fermix_slogpf_update (one-index Pfaffian move on "
                         "G = S^-T / 2). G stays resident; e2e copies only the new rows / indices in and the ratio out")
    ap.add_argument("--planar", action="store_true",
                    help="complex dtypes: inputs and gradients as split real / imaginary planes (fermix_*_planar)")
    ap.add_argument("--cpu-n", type=int, default=0,
                    help="time the CPU baseline at this n instead (for sizes where the restatement takes minutes)")
    ap.add_argument("--per-config", default="auto", choices=["auto", "on", "off"],
                    help="add a per_config array (every BASELINE configuration) to the line; auto: on for the "
                         "default workload at N = 1")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-launch-count", action="store_true",
                    help="skip counting kernel launches with the CUDA profiler (for runs under ncu)")
    a = ap.parse_args()
    d = ap.parse_args([])
    a.is_default = all(getattr(a, k) == getattr(d, k) for k in
                       ("op", "fwd_only", "batch", "n", "dtype", "prec", "gather", "move", "planar"))
    return a


def workload_name(a):
    what = "fwd" if a.fwd_only else "fwd+VJP(logabs)"
    g = f" gathered from phi {a.gather}x{a.n}" if a.gather else ""
    p = " planar" if getattr(a, "planar", False) and a.dtype in ("c64", "c128") else ""
    return f"{a.op} {what} {a.dtype}{p} B={a.batch}/GPU n={a.n} prec={a.prec}{g}"


def flops_bytes(a):
    """Algorithmic work per matrix (complex = 4 real flops per multiply-add pair)."""
    n = a.n
    s = {"f32": 4, "f64": 8, "c64": 8, "c128": 16}[a.dtype]
    cx = 4 if a.dtype in ("c64", "c128") else 1
    if a.op == "slogdet":
        fl = (2.0 / 3.0 if a.fwd_only else 2.0) * n**3
    else:
        fl = (1.0 / 3.0 if a.fwd_only else 5.0 / 3.0) * n**3
    by = (1 if a.fwd_only else 2) * n * n * s
    if a.gather:
        # the shared phi once per launch, the occupations, and the gradient written
        by = a.gather * n * s / a.batch + n * 4 + (0 if a.fwd_only else n * n * s)
    return fl * cx, by


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_from_profiles(a):
    """DRAM bytes per launch of the dominant kernel: the committed ncu summary's line
    'traffic_bytes_per_matrix: X' for this workload, times the batch; else None."""
    ieee = "_ieee" if a.prec == "ieee" and a.dtype in ("f32", "c64") else ""
    name = f"{kernel_name(a)}_{a.dtype}_n{a.n}{ieee}_{'fwd' if a.fwd_only else 'fwdbwd'}.md"
    p = os.path.join(ROOT, "profiles", name)
    if a.gather or not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("traffic_bytes_per_matrix:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0]) * a.batch
            except ValueError:
                return None
    return None


# --------------------------------------------------------------- clocks sampler
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-i", str(self.idx),
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------- CPU (oracle) timing
def cpu_rate(a, count, threads):
    """Matrices/s of the oracle (the numpy / LAPACK restatement of the reference's
    generic path) on `count` matrices of the workload."""
    import numpy as np
    from threadpoolctl import threadpool_limits

    from oracle import fallback as F

    gen = np.random.default_rng(a.seed + 12345)
    npdt = {"f32": np.float32, "f64": np.float64, "c64": np.complex64, "c128": np.complex128}[a.dtype]
    A = gen.standard_normal((count, a.n, a.n))
    if a.dtype in ("c64", "c128"):
        A = A + 1j * gen.standard_normal((count, a.n, a.n))
    A = A.astype(npdt)
    with threadpool_limits(limits=threads):
        t0 = time.perf_counter()
        if a.op == "slogpf":
            S = A - np.swapaxes(A, -1, -2)
            if a.fwd_only:
                F.slogpf(S)
            else:
                F.pf_parts(S, False)  # one factor-keeping Parlett-Reid: (sign, logabs, S^-1)
        else:
            if a.fwd_only:
                F.slogdet(A)
            else:
                F.lu_parts(A, True)
        dt = time.perf_counter() - t0
    return count / dt, dt


def run_reference(a, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    # warm-up and timed steps, each a bounded sample of the workload
    for _ in range(max(a.warmup, 0)):
        cpu_rate(a, max(1, a.ref_step // 4), threads)
    total_m, total_t = 0, 0.0
    for _ in range(a.steps):
        r, dt = cpu_rate(a, a.ref_step, threads)
        total_m += a.ref_step
        total_t += dt
    v = total_m / total_t
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": v,
        "unit": "matrices/s",
        "n_gpus": a.gpus,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": 1e3 * total_t / a.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": a.dtype,
        "data": "synthetic (seeded iid N(0,1))",
        "config": {"workload": workload_name(a), "op": a.op, "batch_per_gpu": a.batch, "n": a.n, "prec": a.prec},
        "cpu_baseline": {
            "value": v,
            "unit": "matrices/s",
            "cores": threads,
            "kind": "port",
            "sample": f"{a.ref_step} matrices per step x {a.steps} steps of the same workload (numpy/LAPACK "
                      "restatement of the reference's generic path; the reference itself needs jax, absent here)",
        },
        "e2e": {"value": v, "unit": "matrices/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- k-row moves
def run_move(a, rank, world, local):
    """--move K: one step = one fermix_slogdet_update call (the ratio kernel, then the
    in-place row update of every G = A^-T in the batch; every move accepted). HBM-bound:
    the algorithmic bytes per matrix are one read and one write of G plus the k new rows."""
    import numpy as np
    import torch

    from fermix_b200 import _lib

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    L = _lib.lib()
    tdt = {"f32": torch.float32, "f64": torch.float64, "c64": torch.complex64, "c128": torch.complex128}[a.dtype]
    rdt = torch.float32 if a.dtype in ("f32", "c64") else torch.float64
    kind = {"f32": 0, "f64": 1, "c64": 2, "c128": 3}[a.dtype]
    B, n, k = a.batch, a.n, a.move
    pfm = a.op == "slogpf"
    if pfm and n % 2:
        raise SystemExit("Pfaffian moves (--op slogpf) need an even n")
    pfk = pfm and k > 1  # k-index Pfaffian move (three passes over G)
    gen = torch.Generator(device=dev)
    gen.manual_seed(a.seed + 1000 * rank)
    # G of a well-conditioned matrix (identity-shifted A, or a skew S shifted by pair blocks
    # [[0, 2], [-2, 0]]); the moves replace random rows by random rows near them, so every
    # ratio stays O(1) while G is updated step after step
    A = torch.randn((B, n, n), generator=gen, device=dev, dtype=tdt) / n**0.5
    if pfm:
        J = torch.zeros((n, n), device=dev, dtype=tdt)
        r = torch.arange(0, n, 2, device=dev)
        J[r, r + 1], J[r + 1, r] = 2.0, -2.0
        A = A - A.transpose(-1, -2) + J
        G = (0.5 * torch.linalg.inv(A).transpose(-1, -2)).contiguous()
        IDX = torch.rand((B, n), generator=gen, device=dev).argsort(dim=1)[:, :k].to(torch.int32).contiguous()
    else:
        A = A + 2 * torch.eye(n, device=dev)
        G = torch.linalg.inv(A).transpose(-1, -2).contiguous()
        IDX = torch.rand((B, n), generator=gen, device=dev).argsort(dim=1)[:, :k].to(torch.int32).contiguous()
    U = (torch.gather(A, 1, IDX.long()[:, :, None].expand(B, k, n)) +
         0.1 * torch.randn((B, k, n), generator=gen, device=dev, dtype=tdt) / n**0.5).contiguous()
    del A
    sign = torch.empty(B, dtype=tdt, device=dev)
    logabs = torch.empty(B, dtype=rdt, device=dev)
    wsb = (L.fermix_slogpf_move_k_workspace_bytes(kind, B, n, k) if pfk else
           L.fermix_slogpf_update_workspace_bytes(kind, B, n) if pfm else
           L.fermix_slogdet_update_workspace_bytes(kind, B, n, k))
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def call(Ud, Id):
        if pfk:
            _lib.check(L.fermix_slogpf_update_k(sp, kind, B, n, k, G.data_ptr(), Ud.data_ptr(), Id.data_ptr(), None,
                                                sign.data_ptr(), logabs.data_ptr(), ws.data_ptr(), wsb))
            return
        if pfm:
            _lib.check(L.fermix_slogpf_update(sp, kind, B, n, G.data_ptr(), Ud.data_ptr(), Id.data_ptr(), None,
                                              sign.data_ptr(), logabs.data_ptr(), ws.data_ptr(), wsb))
            return
        _lib.check(L.fermix_slogdet_update(sp, kind, B, n, k, G.data_ptr(), Ud.data_ptr(), Id.data_ptr(), None,
                                           sign.data_ptr(), logabs.data_ptr(), ws.data_ptr(), wsb))

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(a.warmup):
        call(U, IDX)
    barrier()
    clocks = Clocks(local if "CUDA_VISIBLE_DEVICES" not in os.environ else
                    os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])
    clocks.start()
    time.sleep(0.2)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(a.steps):
        call(U, IDX)
    e1.record(stream)
    barrier()
    t_dev = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    ck = clocks.stop()
    s = G.element_size()
    # G read + written (k-index Pfaffian move: read twice), the new rows, the indices
    by = (3 if pfk else 2) * n * n * s + k * n * s + k * 4
    launch_s = t_dev / a.steps  # both kernels of the call: an upper bound on the row kernel's time
    hbm, peak_kind = peaks()
    achieved = B * by / launch_s / 1e9
    e2e = None
    if not a.no_e2e:
        hU = torch.empty(U.shape, dtype=tdt, pin_memory=True)
        hU.copy_(U)
        hI = torch.empty(IDX.shape, dtype=torch.int32, pin_memory=True)
        hI.copy_(IDX)
        dU, dI = torch.empty_like(U), torch.empty_like(IDX)
        hS = torch.empty(B, dtype=tdt, pin_memory=True)
        hL = torch.empty(B, dtype=rdt, pin_memory=True)
        ke = max(3, min(a.steps, 50))

        def e2e_step():
            dU.copy_(hU, non_blocking=True)
            dI.copy_(hI, non_blocking=True)
            call(dU, dI)
            hS.copy_(sign, non_blocking=True)
            hL.copy_(logabs, non_blocking=True)

        for _ in range(2):
            e2e_step()
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(ke):
            e2e_step()
        f1.record(stream)
        barrier()
        t_e2e = max_over_ranks(f0.elapsed_time(f1) / 1e3)
        e2e = {"value": world * B * ke / t_e2e, "unit": "moves/s",
               "h2d_bytes_per_step": hU.numel() * hU.element_size() + hI.numel() * 4,
               "d2h_bytes_per_step": hS.numel() * hS.element_size() + hL.numel() * hL.element_size(), "steps": ke}
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:
        from threadpoolctl import threadpool_limits

        from oracle import moves

        cnt = min(B, a.cpu_sample)
        Gh, Uh, Ih = G[:cnt].cpu().numpy(), U[:cnt].cpu().numpy(), IDX[:cnt].cpu().numpy()
        threads = os.cpu_count() or 1
        with threadpool_limits(limits=threads):
            t0 = time.perf_counter()
            if pfk:
                moves.pf_update_woodbury_k(Gh, Uh, Ih)
            elif pfm:
                moves.pf_update_woodbury(Gh, Uh[:, 0], Ih[:, 0])
            else:
                moves.ratio_woodbury(Gh, Uh, Ih)
                moves.update_woodbury(Gh, Uh, Ih)
            dt = time.perf_counter() - t0
        cpu = {"value": cnt / dt, "unit": "moves/s", "cores": threads, "kind": "port",
               "sample": f"{cnt} moves of the same workload ({dt:.2f} s; numpy Woodbury ratio + update in float64)"}
    if rank == 0:
        line = {
            "metric": (f"{k}-index Pfaffian moves/sec (ratio + in-place gradient update)" if pfk else
                       "one-index Pfaffian moves/sec (ratio + in-place gradient update)" if pfm else
                       "k-row determinant moves/sec (ratio + in-place inverse update)"),
            "value": world * B * a.steps / t_dev,
            "unit": "moves/s",
            "n_gpus": world,
            "steps": a.steps,
            "warmup": a.warmup,
            "ms_per_step": 1e3 * t_dev / a.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": a.dtype,
            "data": "synthetic (seeded G = inv(A)^T of A ~ N(0, 1/n) + 2I, new rows near the replaced ones)",
            "config": {"workload": (f"slogpf {k}-index move {a.dtype} B={B}/GPU n={n}" if pfk else
                                    f"slogpf one-index move {a.dtype} B={B}/GPU n={n}" if pfm else
                                    f"slogdet {k}-row move {a.dtype} B={B}/GPU n={n}"),
                       "op": "slogpf_update" if pfm else "slogdet_update",
                       "batch_per_gpu": B, "n": n, "k": k, "parallelism": f"batch sharded x{world}, no collective",
                       "l2": "G exceeds L2 (no flush needed)" if B * n * n * s > 126e6 else "G fits L2"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "traffic": None, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "kernel": "pfk_rows_kernel" if pfk else "pfm_rows_kernel" if pfm else "upd_rows_vec_kernel",
                         "timing": "the whole call (ratio kernel + row kernel): an upper bound on the row kernel's time",
                         "algorithmic_bytes_per_launch": B * by},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": a.steps * (3 if pfm else 2),  # pfk: v, prep, rows; pfm: ratio, v, rows
            "clocks": ck,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------- measured pipe peaks
_PIPES = {}


def pipe_peaks(dev):
    """Arithmetic peaks measured on this GPU (TFLOP/s), once per process: the FP32 / FP64
    FMA pipes with the library's FMA-throughput probe (fermix_selftest_fma_rate: 148 x 8
    blocks of 256 threads, 8 independent chains each), and TF32 tensor throughput as
    cuBLAS fp32 matmul with TF32 enabled (8192^3, best of 5)."""
    if _PIPES:
        return _PIPES
    import torch

    from fermix_b200 import _lib

    L = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    out = torch.empty(4096, dtype=torch.float64, device=dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    blocks, iters = sms * 8, 1 << 14
    for name, kind in (("ffma", _lib.FX_F32), ("dfma", _lib.FX_F64)):
        best = None
        for _ in range(4):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            _lib.check(L.fermix_selftest_fma_rate(stream.cuda_stream, kind, blocks, iters, out.data_ptr()))
            e1.record(stream)
            e1.synchronize()
            t = e0.elapsed_time(e1) / 1e3
            best = t if best is None else min(best, t)
        _PIPES[name] = blocks * 256 * 16.0 * iters / best / 1e12
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        a = torch.randn((8192, 8192), device=dev)
        b = torch.randn((8192, 8192), device=dev)
        torch.matmul(a, b)
        best = None
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            torch.matmul(a, b)
            e1.record(stream)
            e1.synchronize()
            t = e0.elapsed_time(e1) / 1e3
            best = t if best is None else min(best, t)
        _PIPES["tf32"] = 2 * 8192.0**3 / best / 1e12
        del a, b
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return _PIPES


def compute_roofline(a, flops_per_launch, launch_s, dev):
    """The arithmetic pipe that bounds this workload and the fraction of it achieved:
    the tensor cores for the tensor-memory kernels (measured TF32 throughput divided by
    the TF32 products per update: 4 for the LU, 3 for Parlett-Reid), the FP32 / FP64 FMA
    pipes otherwise -- all measured live on this GPU."""
    kern = kernel_name(a)
    pk = pipe_peaks(dev)
    achieved = flops_per_launch / launch_s / 1e12
    if (kern in TC_KERNEL.values() and a.prec == "tf32x3") or kern == "lg_tc_update_kernel":
        # the LU kernels and the blocked engines' update take 4 TF32 products, pf_tc 3
        products = 3 if kern == TC_KERNEL["slogpf"] else 4
        pipe, peak = f"tcgen05 kind::tf32, {products} products per update (measured TF32 / {products})", \
            pk["tf32"] / products
    elif a.dtype in ("f32", "c64"):
        pipe, peak = "fp32 FFMA (measured)", pk["ffma"]
    else:
        pipe, peak = "fp64 DFMA (measured)", pk["dfma"]
    return {"pipe": pipe, "achieved_tflops": achieved, "peak_tflops": peak, "frac": achieved / peak}


def count_launches(fn, reps=3):
    """Kernels launched by one call of fn: reps calls under the CUDA profiler (CUPTI),
    divided by reps; None when the profiler is unavailable or saw nothing."""
    import torch

    try:
        from torch.profiler import ProfilerActivity, profile

        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
            for _ in range(reps):
                fn()
                torch.cuda.synchronize()
        names = [e.name for e in prof.events() if e.device_type.name == "CUDA" and
                 not e.name.lower().startswith(("memcpy", "memset"))]
        if not names:
            return None, ["profiler recorded no kernels"]
        return round(len(names) / reps), sorted(set(names))
    except Exception as e:  # pragma: no cover - profiler not available
        return None, [f"profiler unavailable: {type(e).__name__}: {e}"]


# --------------------------------------------------------------- GPU arm
class Ctx:
    """Per-process state of the GPU arm: device, ranks, the process group."""

    def __init__(self, rank, world, local):
        import torch

        self.rank, self.world, self.local = rank, world, local
        torch.cuda.set_device(local)
        self.dev = torch.device("cuda", local)
        self.dist = None
        if world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.dev)
            self.dist = dist
        self.gpu_index = (local if "CUDA_VISIBLE_DEVICES" not in os.environ else
                          os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])

    def barrier(self):
        import torch

        if self.dist is not None:
            self.dist.barrier()
        torch.cuda.synchronize(self.dev)

    def max_over_ranks(self, x):
        import torch

        if self.dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.dist is not None:
            self.dist.barrier()
            self.dist.destroy_process_group()


def measure(a, ctx, cpu=True, e2e=True):
    """One workload on this rank's GPU: the device-resident throughput of K timed steps
    (max over ranks), the end-to-end rate through the C ABI with host buffers, the
    rooflines, the kernel launches of one step, the clocks and (rank 0, N = 1) the CPU
    baseline. For N > 1 every step also all-gathers the (sign, logabs) of the whole
    sharded batch (fermix_b200.sharded.all_gather_slog, the only collective)."""
    import torch

    from fermix_b200 import _lib

    dev, rank, world = ctx.dev, ctx.rank, ctx.world
    L = _lib.lib()
    tdt = {"f32": torch.float32, "f64": torch.float64, "c64": torch.complex64, "c128": torch.complex128}[a.dtype]
    rdt = torch.float32 if a.dtype in ("f32", "c64") else torch.float64
    kind = {"f32": 0, "f64": 1, "c64": 2, "c128": 3}[a.dtype]
    prec = {"tf32x3": 1, "ieee": 2}[a.prec]
    planar = bool(a.planar) and a.dtype in ("c64", "c128")
    B, n = a.batch, a.n
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed + 1000 * rank)
    PHI = None
    if a.gather:
        if a.op != "slogdet" or a.gather < n:
            raise SystemExit("--gather needs --op slogdet and SITES >= n")
        # configuration 3: phi iid N(0, 1/sqrt(n)), sorted random n-of-SITES occupations, a
        # duplicated row in 2 % of the samples
        PHI = (torch.randn((a.gather, n), generator=g, device=dev, dtype=tdt) / n**0.5).contiguous()
        OCC = torch.rand((B, a.gather), generator=g, device=dev).argsort(dim=1)[:, :n].sort(dim=1).values
        dup = torch.rand(B, generator=g, device=dev) < 0.02
        OCC[dup, 1] = OCC[dup, 0]
        inputs = [OCC.to(torch.int32).contiguous()]
    else:
        A = torch.randn((B, n, n), generator=g, device=dev, dtype=tdt)
        if a.op == "slogpf":
            A = (A - A.transpose(-1, -2)).contiguous()
        if planar:
            inputs = [A.real.contiguous(), A.imag.contiguous()]
            del A
        else:
            inputs = [A]
    sign = torch.empty(B, dtype=tdt, device=dev)
    logabs = torch.empty(B, dtype=rdt, device=dev)
    grads = [] if a.fwd_only else ([torch.empty((B, n, n), dtype=rdt, device=dev) for _ in range(2)] if planar
                                   else [torch.empty((B, n, n), dtype=tdt, device=dev)])
    op = _lib.FX_OP_SLOGPF if a.op == "slogpf" else _lib.FX_OP_SLOGDET
    grad = 0 if a.fwd_only else 1

    def ws_bytes(cnt):
        if a.gather:
            return L.fermix_slogdet_gather_workspace_bytes(kind, prec, cnt, n, grad)
        if planar:
            return L.fermix_workspace_bytes_planar(op, kind, cnt, n, grad)
        return L.fermix_workspace_bytes(op, kind, cnt, n, grad)

    wsb = ws_bytes(B)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)

    def call(b0, cnt, xs, gs, strm, wsp, wsz):
        """One C-ABI call on members [b0, b0 + cnt) of the input / gradient arrays."""
        e_in = xs[0].element_size()
        off = b0 * n * n
        x = [t.data_ptr() + off * e_in for t in xs]
        gp = [t.data_ptr() + off * t.element_size() for t in gs]
        sp = sign.data_ptr() + b0 * sign.element_size()
        lp = logabs.data_ptr() + b0 * logabs.element_size()
        if a.gather:
            st = L.fermix_slogdet_gather(strm, kind, prec, cnt, n, PHI.data_ptr(), a.gather, n,
                                         xs[0].data_ptr() + b0 * n * 4, None, 0, sp, lp, None,
                                         gp[0] if gp else None, wsp, wsz)
        elif planar and a.op == "slogpf":
            st = (L.fermix_slogpf_planar(strm, kind, prec, cnt, n, 1, x[0], x[1], sp, lp, None, wsp, wsz) if not gp else
                  L.fermix_slogpf_grad_planar(strm, kind, prec, cnt, n, 1, x[0], x[1], None, 0, 0, sp, lp, None,
                                              gp[0], gp[1], wsp, wsz))
        elif planar:
            st = (L.fermix_slogdet_planar(strm, kind, prec, cnt, n, x[0], x[1], sp, lp, None, wsp, wsz) if not gp else
                  L.fermix_slogdet_grad_planar(strm, kind, prec, cnt, n, x[0], x[1], None, 0, 0, sp, lp, None,
                                               gp[0], gp[1], wsp, wsz))
        elif a.op == "slogpf":
            st = (L.fermix_slogpf(strm, kind, prec, cnt, n, 1, x[0], sp, lp, None, wsp, wsz) if not gp else
                  L.fermix_slogpf_grad(strm, kind, prec, cnt, n, 1, x[0], None, 0, 0, sp, lp, None, gp[0], wsp, wsz))
        else:
            st = (L.fermix_slogdet(strm, kind, prec, cnt, n, x[0], sp, lp, None, wsp, wsz) if not gp else
                  L.fermix_slogdet_grad(strm, kind, prec, cnt, n, x[0], None, 0, 0, sp, lp, None, gp[0], wsp, wsz))
        _lib.check(st)

    stream = torch.cuda.current_stream(dev)
    gather_out = None
    if world > 1:
        from fermix_b200 import sharded

        def step():
            call(0, B, inputs, grads, stream.cuda_stream, ws.data_ptr(), wsb)
            # the sharded batch's (sign, logabs) on every rank: the only collective
            nonlocal gather_out
            gather_out = sharded.all_gather_slog(sign, logabs, B * world)
    else:
        def step():
            call(0, B, inputs, grads, stream.cuda_stream, ws.data_ptr(), wsb)

    # ---- device-resident timing
    for _ in range(a.warmup):
        step()
    ctx.barrier()
    clocks = Clocks(ctx.gpu_index)
    clocks.start()
    time.sleep(0.2)
    ctx.barrier()
    if a.gather:
        # the gathered inputs fit in L2: flush it (write 256 MB) before every step and time
        # each step's launch alone
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
        for f0, f1 in evs:
            flush.fill_(1)
            f0.record(stream)
            step()
            f1.record(stream)
        ctx.barrier()
        t_dev = sum(f0.elapsed_time(f1) for f0, f1 in evs) / 1e3
        del flush
    else:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(a.steps):
            step()
        e1.record(stream)
        ctx.barrier()
        t_dev = e0.elapsed_time(e1) / 1e3
    ck = clocks.stop()
    t_dev = ctx.max_over_ranks(t_dev)
    value = world * B * a.steps / t_dev
    fl, by = flops_bytes(a)
    launch_s = t_dev / a.steps
    hbm, peak_kind = peaks()
    achieved = B * by / launch_s / 1e9
    cr = compute_roofline(a, B * fl, launch_s, dev)
    t_hbm, t_pipe = B * by / (hbm * 1e9), B * fl / (cr["peak_tflops"] * 1e12)
    roofline = {
        "bound": "hbm",
        "achieved": achieved,
        "peak": hbm,
        "unit": "GB/s",
        "frac": achieved / hbm,
        "traffic": traffic_from_profiles(a),
        "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
        "kernel": kernel_name(a),
        "algorithmic_bytes_per_launch": B * by,
        "flops_per_launch": B * fl,
        "achieved_tflops": B * fl / launch_s / 1e12,
        "binding": "hbm" if t_hbm >= t_pipe else cr["pipe"],
        "binding_frac": max(t_hbm, t_pipe) / launch_s,
    }
    launches, kernels = (None, ["not counted (--no-launch-count)"]) if a.no_launch_count else count_launches(step)

    # ---- end to end through the C ABI with host buffers
    e2e_line = None
    if e2e:
        hin = []
        for t in inputs:
            h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            h.copy_(t)
            hin.append(h)
        din = [torch.empty_like(t) for t in inputs]
        hS = torch.empty(B, dtype=tdt, pin_memory=True)
        hL = torch.empty(B, dtype=rdt, pin_memory=True)
        hG = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in grads]
        hP = None
        if PHI is not None:
            hP = torch.empty(PHI.shape, dtype=tdt, pin_memory=True)
            hP.copy_(PHI)
        ke = max(3, min(a.steps, 20))
        # the step in CH chunks on three streams (copy in, compute, copy out), so that the
        # two copy directions and the compute overlap; every call goes through the C ABI
        CH = 1 if a.gather else min(8, B)
        s_in, s_cmp, s_out = (torch.cuda.Stream(dev) for _ in range(3))
        bounds = [(B * c // CH, B * (c + 1) // CH) for c in range(CH)]
        wmax = ws_bytes(max(e - b for b, e in bounds))
        wsc = torch.empty(max(wmax, 1), dtype=torch.uint8, device=dev)

        def e2e_step():
            start = torch.cuda.Event()
            start.record(stream)
            for s_ in (s_in, s_cmp, s_out):
                s_.wait_event(start)
            if hP is not None:
                with torch.cuda.stream(s_in):
                    PHI.copy_(hP, non_blocking=True)
            for b0, b1 in bounds:
                with torch.cuda.stream(s_in):
                    for d, h in zip(din, hin):
                        d[b0:b1].copy_(h[b0:b1], non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(s_in)
                s_cmp.wait_event(ev_in)
                call(b0, b1 - b0, din, grads, s_cmp.cuda_stream, wsc.data_ptr(), wmax)
                ev_c = torch.cuda.Event()
                ev_c.record(s_cmp)
                s_out.wait_event(ev_c)
                with torch.cuda.stream(s_out):
                    hS[b0:b1].copy_(sign[b0:b1], non_blocking=True)
                    hL[b0:b1].copy_(logabs[b0:b1], non_blocking=True)
                    for h, d in zip(hG, grads):
                        h[b0:b1].copy_(d[b0:b1], non_blocking=True)
            done = torch.cuda.Event()
            done.record(s_out)
            stream.wait_event(done)

        for _ in range(2):
            e2e_step()
        ctx.barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(ke):
            e2e_step()
        f1.record(stream)
        ctx.barrier()
        t_e2e = ctx.max_over_ranks(f0.elapsed_time(f1) / 1e3)
        h2d = sum(h.numel() * h.element_size() for h in hin) + (0 if hP is None else hP.numel() * hP.element_size())
        d2h = hS.numel() * hS.element_size() + hL.numel() * hL.element_size()
        d2h += sum(h.numel() * h.element_size() for h in hG)
        e2e_line = {"value": world * B * ke / t_e2e, "unit": "matrices/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": ke}
        del hin, din, hG, wsc

    cpu_line = None
    if cpu and rank == 0 and world == 1 and a.cpu_sample > 0:
        threads = os.cpu_count() or 1
        ca = argparse.Namespace(**vars(a))
        if a.cpu_n:
            ca.n = a.cpu_n
        r, dt = cpu_rate(ca, a.cpu_sample, threads)
        note = ""
        if a.cpu_n and a.cpu_n != a.n:
            note = (f"; timed at n = {a.cpu_n} because the restatement takes minutes per matrix at n = {a.n}: "
                    f"value is the n = {a.cpu_n} rate, est_value_at_n scales it by (n_sample / n)^3")
        cpu_line = {"value": r, "unit": "matrices/s", "cores": threads, "kind": "port",
                    "sample": f"{a.cpu_sample} matrices of the same workload ({dt:.1f} s; numpy/LAPACK restatement of "
                              f"the reference's generic path, all host threads){note}"}
        if note:
            cpu_line["n_sample"] = a.cpu_n
            cpu_line["est_value_at_n"] = r * (a.cpu_n / a.n) ** 3
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "matrices/s",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": 1e3 * t_dev / a.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": a.dtype,
        "data": ("synthetic (seeded iid N(0,1), S = A - A^T)" if a.op == "slogpf" else
                 "synthetic (seeded phi ~ N(0, 1/sqrt(n)), random sorted occupations, 2% duplicated rows)"
                 if a.gather else "synthetic (seeded iid N(0,1))") + (", split re/im planes" if planar else ""),
        "config": {
            "workload": workload_name(a),
            "op": a.op,
            "pass": "fwd" if a.fwd_only else "fwd+bwd",
            "batch_per_gpu": B,
            "n": n,
            "prec": a.prec,
            "layout": "planar (split re/im)" if planar else "interleaved",
            "parallelism": (f"batch sharded x{world}; (sign, logabs) all-gathered every step" if world > 1
                            else "one GPU"),
            "l2": ("L2 flushed before every timed step" if a.gather else
                   "inputs exceed L2 (no flush needed)" if B * n * n * inputs[0].element_size() * len(inputs) > 126e6
                   else "inputs fit L2"),
        },
        "roofline": roofline,
        "compute_roofline": cr,
        "cpu_baseline": cpu_line,
        "e2e": e2e_line,
        "gpu_launches": None if launches is None else launches * a.steps,
        "gpu_launches_per_step": launches,
        "kernels": kernels,
        "clocks": ck,
    }
    del inputs, grads, ws
    torch.cuda.empty_cache()
    return line


# the default run's per-configuration entries (C5 on bounded batch
# samples). Keys override the headline arguments.
PER_CONFIG = [
    ("C1 slogdet fwd", dict(op="slogdet", fwd_only=True)),
    ("C2 slogpf fwd tf32x3", dict(fwd_only=True, cpu_sample=128)),
    ("C2 slogpf fwd+bwd tf32x3", dict()),
    ("C2 slogpf fwd ieee", dict(fwd_only=True, prec="ieee", steps=10, cpu_sample=128)),
    ("C2 slogpf fwd+bwd ieee", dict(prec="ieee", steps=10, cpu_sample=128)),
    ("C3 slogdet fwd (materialised)", dict(op="slogdet", n=256, batch=16384, fwd_only=True, steps=10, cpu_sample=256)),
    ("C3 slogdet fwd+bwd (materialised)", dict(op="slogdet", n=256, batch=16384, steps=10, cpu_sample=128)),
    ("C3 slogdet fwd (gathered from phi)", dict(op="slogdet", n=256, batch=16384, gather=512, fwd_only=True, steps=10,
                                                cpu_sample=256)),
    ("C3 slogdet fwd+bwd (gathered from phi)", dict(op="slogdet", n=256, batch=16384, gather=512, steps=10,
                                                    cpu_sample=128)),
    ("C4 slogpf fwd c64 planar", dict(dtype="c64", n=512, batch=2048, fwd_only=True, planar=True, steps=5, warmup=3,
                                      cpu_sample=2, cpu_n=256)),
    ("C4 slogpf fwd+bwd c64 planar", dict(dtype="c64", n=512, batch=2048, planar=True, steps=5, warmup=3, cpu_sample=2,
                                          cpu_n=256)),
    ("C5a slogdet fwd f64 n4096 (B=16 sample)", dict(op="slogdet", dtype="f64", prec="ieee", n=4096, batch=16,
                                                     fwd_only=True, steps=3, warmup=3, cpu_sample=2)),
    ("C5a slogdet fwd+bwd f64 n4096 (B=16 sample)", dict(op="slogdet", dtype="f64", prec="ieee", n=4096, batch=16,
                                                         steps=3, warmup=3, cpu_sample=1)),
    ("C5b slogpf fwd c128 n4096 (B=4 sample)", dict(dtype="c128", prec="ieee", n=4096, batch=4, fwd_only=True, steps=3,
                                                    warmup=3, cpu_sample=1, cpu_n=512)),
    ("C5b slogpf fwd+bwd c128 n4096 (B=4 sample)", dict(dtype="c128", prec="ieee", n=4096, batch=4, steps=3, warmup=3,
                                                        cpu_sample=1, cpu_n=512)),
]

SLIM = ("value", "ms_per_step", "roofline", "compute_roofline", "cpu_baseline", "e2e", "gpu_launches_per_step",
        "clocks")


def per_config(a, ctx, headline):
    out = []
    for name, over in PER_CONFIG:
        if not over:
            line = headline
        else:
            b = argparse.Namespace(**vars(a))
            b.steps, b.warmup, b.cpu_sample = min(a.steps, 20), max(a.warmup, 3), 512
            for k, v in over.items():
                setattr(b, k, v)
            line = measure(b, ctx)
        entry = {"config": name, "workload": line["config"]["workload"], "pass": line["config"]["pass"],
                 "layout": line["config"]["layout"], "dtype": line["dtype"], "steps": line["steps"]}
        entry.update({k: line[k] for k in SLIM})
        if entry["roofline"]:
            entry["roofline"] = {k: entry["roofline"][k] for k in ("achieved", "peak", "frac", "kernel", "binding",
                                                                   "binding_frac", "achieved_tflops")}
        out.append(entry)
        if ctx.rank == 0:
            print(f"# {name}: {line['value']:.1f} mat/s", file=sys.stderr, flush=True)
    return out


def main():
    a = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        run_reference(a, rank)
        return
    if a.move:
        run_move(a, rank, world, local)
        return
    ctx = Ctx(rank, world, local)
    line = measure(a, ctx, cpu=not a.no_cpu, e2e=not a.no_e2e)
    pc = a.per_config == "on" or (a.per_config == "auto" and world == 1 and a.is_default)
    if pc:
        line["per_config"] = per_config(a, ctx, line)
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()


if __name__ == "__main__":
    main()
