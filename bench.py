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
    """The dominant kernel of this workload: the tensor-memory kernels for float32 /
    tf32x3 (slogpf 8 <= n <= 128, even n; slogdet 8 <= n <= 256), the register-panel
    kernels otherwise up to n = 256, and above that the blocked engines' tiled update."""
    if a.dtype == "f32" and a.prec == "tf32x3" and a.n >= 8:
        if a.op == "slogpf" and a.n <= 128 and a.n % 2 == 0:
            return TC_KERNEL[a.op]
        if a.op == "slogdet" and a.n <= 256:
            return TC_KERNEL[a.op]
    if a.n <= 256:
        return SMALL_KERNEL[a.op]
    return "lg_update_kernel"


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
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    return ap.parse_args()


def workload_name(a):
    what = "fwd" if a.fwd_only else "fwd+VJP(logabs)"
    g = f" gathered from phi {a.gather}x{a.n}" if a.gather else ""
    return f"{a.op} {what} {a.dtype} B={a.batch}/GPU n={a.n} prec={a.prec}{g}"


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


# FMA-pipe peaks measured on this pool's B200s at 1965 MHz (8 independent FMA chains per
# thread, 148 x 8 blocks of 256 threads, CUDA events)
FFMA_TFLOPS = 72.6
DFMA_TFLOPS = 34.1


def compute_roofline(a, flops_per_launch, launch_s):
    """The arithmetic pipe that bounds this workload and the fraction of it achieved:
    the tensor cores for the tensor-memory kernels (TF32 at half the measured bf16 rate,
    divided by the TF32 products per update), the FP32 / FP64 FMA pipes otherwise."""
    kern = kernel_name(a)
    achieved = flops_per_launch / launch_s / 1e12
    if kern in TC_KERNEL.values():
        p = os.path.join(ROOT, "MEASURED_PEAKS.json")
        bf16 = float(json.load(open(p))["bf16_tflops"]) if os.path.exists(p) else 1590.0
        products = 4 if a.op == "slogdet" else 3
        pipe, peak = f"tcgen05 kind::tf32, {products} products per update", 0.5 * bf16 / products
    elif a.dtype in ("f32", "c64"):
        pipe, peak = "fp32 FFMA", FFMA_TFLOPS
    else:
        pipe, peak = "fp64 DFMA", DFMA_TFLOPS
    return {"pipe": pipe, "achieved_tflops": achieved, "peak_tflops": peak, "frac": achieved / peak}


def launches_per_call(a, sms=148):
    """Kernels one library call launches for this workload, mirroring the dispatch of
    fermix_b200/csrc/api.cu: one for n <= 256 (odd-n slogpf, the closed forms, the
    tensor-memory and register-panel kernels); for n > 256 the blocked engines' kernels per
    panel and per batch slice (a slice: at most SMs x 4 matrices and about 8 GiB)."""
    n, B = a.n, a.batch
    if n <= 256 or (a.op == "slogpf" and n % 2):
        return 1
    s = {"f32": 4, "f64": 8, "c64": 8, "c128": 16}[a.dtype]
    nb = 32 if s <= 8 else 16
    per_mat = n * n * s + 2 * n * nb * s + 3 * nb * nb * s + n * s + 3 * n * 4 + ((n + 511) // 512) * nb * 4
    bs = max(1, min(B, sms * 4, (8 << 30) // per_mat))
    slices = (B + bs - 1) // bs
    grad = not a.fwd_only

    def lu_engine():
        k = 0
        for k0 in range(0, n, nb):
            kw = min(nb, n - k0)
            k += (1 if (n - k0 + 511) // 512 > 1 else 0) + 3 + (1 if (grad or k0 + kw < n) else 0)
        return k + 1 + (2 if grad else 0)

    if a.op == "slogdet":
        return slices * lu_engine()
    # slogpf: the skew copy, per panel the panel kernel, two swaps and the update, the finish
    npair = (nb // 2) if n <= 512 else (8 if s <= 8 else 4)
    k = 1
    for k0 in range(0, n, 2 * npair):
        np_ = min(npair, (n - k0) // 2)
        k += 3 + (1 if k0 + 2 * np_ < n else 0)
    k += 1
    if grad:
        k += 1 + lu_engine()  # the skew copy of the gradient engine, then the LU engine
    return slices * k


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_from_profiles(a):
    """DRAM bytes per launch of the dominant kernel: the committed ncu summary's line
    'traffic_bytes_per_matrix: X' for this workload, times the batch; else None."""
    name = f"{kernel_name(a)}_{a.dtype}_n{a.n}_{'fwd' if a.fwd_only else 'fwdbwd'}.md"
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
    if pfm and (k != 1 or n % 2):
        raise SystemExit("Pfaffian moves (--op slogpf) need --move 1 and an even n")
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
        IDX = torch.randint(0, n, (B, 1), generator=gen, device=dev, dtype=torch.int32)
    else:
        A = A + 2 * torch.eye(n, device=dev)
        G = torch.linalg.inv(A).transpose(-1, -2).contiguous()
        IDX = torch.rand((B, n), generator=gen, device=dev).argsort(dim=1)[:, :k].to(torch.int32).contiguous()
    U = (torch.gather(A, 1, IDX.long()[:, :, None].expand(B, k, n)) +
         0.1 * torch.randn((B, k, n), generator=gen, device=dev, dtype=tdt) / n**0.5).contiguous()
    del A
    sign = torch.empty(B, dtype=tdt, device=dev)
    logabs = torch.empty(B, dtype=rdt, device=dev)
    wsb = (L.fermix_slogpf_update_workspace_bytes(kind, B, n) if pfm else
           L.fermix_slogdet_update_workspace_bytes(kind, B, n, k))
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def call(Ud, Id):
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
    by = 2 * n * n * s + k * n * s + k * 4  # G read + written, the new rows, the indices
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
            if pfm:
                moves.pf_update_woodbury(Gh, Uh[:, 0], Ih[:, 0])
            else:
                moves.ratio_woodbury(Gh, Uh, Ih)
                moves.update_woodbury(Gh, Uh, Ih)
            dt = time.perf_counter() - t0
        cpu = {"value": cnt / dt, "unit": "moves/s", "cores": threads, "kind": "port",
               "sample": f"{cnt} moves of the same workload ({dt:.2f} s; numpy Woodbury ratio + update in float64)"}
    if rank == 0:
        line = {
            "metric": ("one-index Pfaffian moves/sec (ratio + in-place gradient update)" if pfm else
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
            "config": {"workload": (f"slogpf one-index move {a.dtype} B={B}/GPU n={n}" if pfm else
                                    f"slogdet {k}-row move {a.dtype} B={B}/GPU n={n}"),
                       "op": "slogpf_update" if pfm else "slogdet_update",
                       "batch_per_gpu": B, "n": n, "k": k, "parallelism": f"batch sharded x{world}, no collective",
                       "l2": "G exceeds L2 (no flush needed)" if B * n * n * s > 126e6 else "G fits L2"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "traffic": None, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "kernel": "pfm_rows_kernel" if pfm else "upd_rows_vec_kernel",
                         "timing": "the whole call (ratio kernel + row kernel): an upper bound on the row kernel's time",
                         "algorithmic_bytes_per_launch": B * by},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": a.steps * (3 if pfm else 2),
            "clocks": ck,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------- GPU arm
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
    prec = {"tf32x3": 1, "ieee": 2}[a.prec]
    B, n = a.batch, a.n
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed + 1000 * rank)
    if a.gather:
        if a.op != "slogdet" or a.gather < n:
            raise SystemExit("--gather needs --op slogdet and SITES >= n")
        # configuration 3: phi iid N(0, 1/sqrt(n)), sorted random n-of-SITES occupations, a
        # duplicated row in 2 % of the samples
        PHI = (torch.randn((a.gather, n), generator=g, device=dev, dtype=tdt) / n**0.5).contiguous()
        OCC = torch.rand((B, a.gather), generator=g, device=dev).argsort(dim=1)[:, :n].sort(dim=1).values
        dup = torch.rand(B, generator=g, device=dev) < 0.02
        OCC[dup, 1] = OCC[dup, 0]
        OCC = OCC.to(torch.int32).contiguous()
        A = OCC  # the per-step device input
    else:
        A = torch.randn((B, n, n), generator=g, device=dev, dtype=tdt)
        if a.op == "slogpf":
            A = (A - A.transpose(-1, -2)).contiguous()
    sign = torch.empty(B, dtype=tdt, device=dev)
    logabs = torch.empty(B, dtype=rdt, device=dev)
    G = None if a.fwd_only else torch.empty((B, n, n), dtype=tdt, device=dev)
    op = _lib.FX_OP_SLOGPF if a.op == "slogpf" else _lib.FX_OP_SLOGDET
    if a.gather:
        wsb = L.fermix_slogdet_gather_workspace_bytes(kind, prec, B, n, 0 if a.fwd_only else 1)
    else:
        wsb = L.fermix_workspace_bytes(op, kind, B, n, 0 if a.fwd_only else 1)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def call(X, Gout):
        if a.gather:
            st = L.fermix_slogdet_gather(sp, kind, prec, B, n, PHI.data_ptr(), a.gather, n, X.data_ptr(), None, 0,
                                         sign.data_ptr(), logabs.data_ptr(), None,
                                         None if Gout is None else Gout.data_ptr(), ws.data_ptr(), wsb)
            _lib.check(st)
            return
        if a.op == "slogpf":
            if a.fwd_only:
                st = L.fermix_slogpf(sp, kind, prec, B, n, 1, X.data_ptr(), sign.data_ptr(), logabs.data_ptr(),
                                     None, ws.data_ptr(), wsb)
            else:
                st = L.fermix_slogpf_grad(sp, kind, prec, B, n, 1, X.data_ptr(), None, 0, 0, sign.data_ptr(),
                                          logabs.data_ptr(), None, Gout.data_ptr(), ws.data_ptr(), wsb)
        else:
            if a.fwd_only:
                st = L.fermix_slogdet(sp, kind, prec, B, n, X.data_ptr(), sign.data_ptr(), logabs.data_ptr(), None,
                                      ws.data_ptr(), wsb)
            else:
                st = L.fermix_slogdet_grad(sp, kind, prec, B, n, X.data_ptr(), None, 0, 0, sign.data_ptr(),
                                           logabs.data_ptr(), None, Gout.data_ptr(), ws.data_ptr(), wsb)
        _lib.check(st)

    def call_chunk(b0, cnt, X, Gout, strm):
        """One C-ABI call on matrices [b0, b0 + cnt) of X / Gout (the e2e pipeline's
        chunks), on stream strm."""
        es = X.element_size()
        off = b0 * n * n * es
        sgn_p = sign.data_ptr() + b0 * sign.element_size()
        la_p = logabs.data_ptr() + b0 * logabs.element_size()
        g_p = None if Gout is None else Gout.data_ptr() + off
        x_p = X.data_ptr() + off
        wsc = L.fermix_workspace_bytes(op, kind, cnt, n, 0 if a.fwd_only else 1)
        wsp = wsc_buf[strm].data_ptr() if wsc else None
        if a.op == "slogpf":
            if a.fwd_only:
                st = L.fermix_slogpf(strm, kind, prec, cnt, n, 1, x_p, sgn_p, la_p, None, wsp, wsc)
            else:
                st = L.fermix_slogpf_grad(strm, kind, prec, cnt, n, 1, x_p, None, 0, 0, sgn_p, la_p, None, g_p, wsp,
                                          wsc)
        else:
            if a.fwd_only:
                st = L.fermix_slogdet(strm, kind, prec, cnt, n, x_p, sgn_p, la_p, None, wsp, wsc)
            else:
                st = L.fermix_slogdet_grad(strm, kind, prec, cnt, n, x_p, None, 0, 0, sgn_p, la_p, None, g_p, wsp,
                                           wsc)
        _lib.check(st)

    wsc_buf = {}

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

    # ---- device-resident timing
    for _ in range(a.warmup):
        call(A, G)
    barrier()
    clocks = Clocks(local if "CUDA_VISIBLE_DEVICES" not in os.environ else
                    os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])
    clocks.start()
    time.sleep(0.2)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    if a.gather:
        # the gathered inputs fit in L2: flush it (write 256 MB) before every step and time
        # each step's launch alone
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
        for f0, f1 in evs:
            flush.fill_(1)
            f0.record(stream)
            call(A, G)
            f1.record(stream)
        barrier()
        t_dev = sum(f0.elapsed_time(f1) for f0, f1 in evs) / 1e3
    else:
        e0.record(stream)
        for _ in range(a.steps):
            call(A, G)
        e1.record(stream)
        barrier()
        t_dev = e0.elapsed_time(e1) / 1e3
    ck = clocks.stop()
    t_dev = max_over_ranks(t_dev)
    value = world * B * a.steps / t_dev
    ms_step = 1e3 * t_dev / a.steps
    fl, by = flops_bytes(a)
    launch_s = t_dev / a.steps  # one launch per step
    hbm, peak_kind = peaks()
    achieved = B * by / launch_s / 1e9
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
    }

    # ---- end to end through the C ABI with host buffers
    e2e = None
    if not a.no_e2e:
        hA = torch.empty(A.shape, dtype=A.dtype, pin_memory=True)
        hA.copy_(A)
        dA = torch.empty_like(A)
        hS = torch.empty(B, dtype=tdt, pin_memory=True)
        hL = torch.empty(B, dtype=rdt, pin_memory=True)
        hG = None if a.fwd_only else torch.empty((B, n, n), dtype=tdt, pin_memory=True)
        dG = None if a.fwd_only else torch.empty((B, n, n), dtype=tdt, device=dev)
        hP = None
        if a.gather:
            hP = torch.empty(PHI.shape, dtype=tdt, pin_memory=True)
            hP.copy_(PHI)
        ke = max(3, min(a.steps, 20))
        # the step in CH chunks on three streams (copy in, compute, copy out), so that the
        # two copy directions and the compute overlap; every call goes through the C ABI
        CH = 1 if a.gather else 8
        s_in, s_cmp, s_out = (torch.cuda.Stream(dev) for _ in range(3))
        bounds = [(B * c // CH, B * (c + 1) // CH) for c in range(CH)]
        if not a.gather:
            wmax = L.fermix_workspace_bytes(op, kind, max(e - b for b, e in bounds), n, 0 if a.fwd_only else 1)
            wsc_buf[s_cmp.cuda_stream] = torch.empty(max(wmax, 1), dtype=torch.uint8, device=dev)

        def e2e_step():
            if a.gather:
                if hP is not None:
                    PHI.copy_(hP, non_blocking=True)
                dA.copy_(hA, non_blocking=True)
                call(dA, dG)
                hS.copy_(sign, non_blocking=True)
                hL.copy_(logabs, non_blocking=True)
                if hG is not None:
                    hG.copy_(dG, non_blocking=True)
                return
            start = torch.cuda.Event()
            start.record(stream)
            for s_ in (s_in, s_cmp, s_out):
                s_.wait_event(start)
            for b0, b1 in bounds:
                with torch.cuda.stream(s_in):
                    dA[b0:b1].copy_(hA[b0:b1], non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(s_in)
                s_cmp.wait_event(ev_in)
                call_chunk(b0, b1 - b0, dA, dG, s_cmp.cuda_stream)
                ev_c = torch.cuda.Event()
                ev_c.record(s_cmp)
                s_out.wait_event(ev_c)
                with torch.cuda.stream(s_out):
                    hS[b0:b1].copy_(sign[b0:b1], non_blocking=True)
                    hL[b0:b1].copy_(logabs[b0:b1], non_blocking=True)
                    if hG is not None:
                        hG[b0:b1].copy_(dG[b0:b1], non_blocking=True)
            done = torch.cuda.Event()
            done.record(s_out)
            stream.wait_event(done)

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
        h2d = A.numel() * A.element_size() + (0 if hP is None else hP.numel() * hP.element_size())
        d2h = sign.numel() * sign.element_size() + logabs.numel() * logabs.element_size()
        if hG is not None:
            d2h += hG.numel() * hG.element_size()
        e2e = {"value": world * B * ke / t_e2e, "unit": "matrices/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "steps": ke}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:
        threads = os.cpu_count() or 1
        r, dt = cpu_rate(a, a.cpu_sample, threads)
        cpu = {"value": r, "unit": "matrices/s", "cores": threads, "kind": "port",
               "sample": f"{a.cpu_sample} matrices of the same workload ({dt:.1f} s; numpy/LAPACK restatement of "
                         "the reference's generic path, all host threads)"}

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "matrices/s",
            "n_gpus": world,
            "steps": a.steps,
            "warmup": a.warmup,
            "ms_per_step": ms_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": a.dtype,
            "data": ("synthetic (seeded iid N(0,1), S = A - A^T)" if a.op == "slogpf" else
                     "synthetic (seeded phi ~ N(0, 1/sqrt(n)), random sorted occupations, 2% duplicated rows)"
                     if a.gather else "synthetic (seeded iid N(0,1))"),
            "config": {
                "workload": workload_name(a),
                "op": a.op,
                "pass": "fwd" if a.fwd_only else "fwd+bwd",
                "batch_per_gpu": B,
                "n": n,
                "prec": a.prec,
                "parallelism": f"batch sharded x{world}, no collective",
                "l2": ("L2 flushed before every timed step" if a.gather else
                       "inputs exceed L2 (no flush needed)" if B * n * n * A.element_size() > 126e6 else "inputs fit L2"),
            },
            "roofline": roofline,
            "compute_roofline": compute_roofline(a, B * fl, launch_s),
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": a.steps * launches_per_call(a),
            "clocks": ck,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
