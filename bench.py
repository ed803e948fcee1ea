#!/usr/bin/env python
"""Leaf-operator replay benchmark on B200.

Workload (one step): 4096 independent leaves x 2048 rows, 768-d SQ8 codes
(per-row symmetric int8 as the reference quantizes them), all-pairs distances
with a bounded top-32 list per row -- the SQ8 leaf hot path of SHEAR's TESSA
replay (``tessa_operator_replay`` A2/A3 leaf stage).  Synthetic rows ~N(0,1),
L2-normalised, seed 0 (the Wiki/LAION datasets are not available here).

Arms:
  ours (default)   libtessa_sm100.so (tcgen05 leaf kernel) through its C ABI.
                   value = rows/s with inputs resident in HBM (device API);
                   e2e   = the same through the host-buffer API with pinned host
                           inputs/outputs copied inside the timed region.
  reference        the reference's leaf algorithm restated on the CPU
                   (oracle/, OpenMP over leaves, all host threads), bounded
                   sample per step.  The reference itself is Rust and cannot be
                   built in this image.

Multi-GPU (torchrun): every rank runs the full per-GPU workload on its own
device (weak scaling, leaves are independent; no collective on the data path).
Timing is device time between barriers, max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

NOMINAL_INT8_TOPS = 4500.0  # B200 dense int8, nominal
# The leaf workload measures leaf-operator rows (vectors) per second of the
# config-2 replay, not a whole build; the build is --workload build.
LEAF_METRIC = "leaf-replay vectors/sec (config 2 leaf operator)"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--leaves", type=int, default=4096)
    ap.add_argument("--leaf-rows", type=int, default=2048)
    ap.add_argument("--dim", type=int, default=768)
    ap.add_argument("--k", type=int, default=32)
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["build", "leaf", "d0", "edges", "assign"], default="build",
                    help="build = GPU-subtree index build, BASELINE config 3 (default) or 1 (--config 1); "
                         "leaf = the config-2 leaf-operator replay; d0 = global-D0 SQ8 staging; "
                         "edges = candidate-edge hashes + host expansion of the leaf lists")
    ap.add_argument("--config", type=int, choices=[1, 3, 4], default=3, help="build: BASELINE config")
    ap.add_argument("--rows", type=int, default=0, help="build: base rows (0 = the config's)")
    ap.add_argument("--queries", type=int, default=0, help="build: recall queries (0 = the config's)")
    ap.add_argument("--cpu-rows", type=int, default=0, help="build: rows of the CPU-baseline sample (0 = auto)")
    ap.add_argument("--no-recall", action="store_true")
    ap.add_argument("--hash-bits", type=int, default=12, help="edges: m_hash_bits (params.rs default 12)")
    ap.add_argument("--assign-leaders", type=int, default=16, help="assign: leaders per task (replay contract)")
    ap.add_argument("--assign-rh", type=int, default=2, help="assign: r_h (replay contract)")
    ap.add_argument("--assign-fp32", action="store_true", help="assign: raw f32 rows (mode A0) instead of SQ8")
    ap.add_argument("--d0-rows", type=int, default=1 << 20, help="D0: raw rows per GPU per step")
    ap.add_argument("--d0-leaders", type=int, default=1000, help="D0: global leaders (params.rs max_leaders)")
    ap.add_argument("--d0-fanout", type=int, default=10, help="D0: fanout_top (params.rs default)")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def workload_desc(a):
    return {
        "workload": f"leaf-operator replay (BASELINE config 2): {a.leaves} leaves x {a.leaf_rows} rows, "
                    f"{a.dim}-d SQ8, top-{a.k} per row",
        "leaves": a.leaves, "leaf_rows": a.leaf_rows, "dim": a.dim, "k": a.k,
        "sq8": "per-row symmetric int8 (reference scheme, dco_sq_int8.rs:1431-1466)",
        "l2": "inputs larger than L2 (codes %.1f GB per GPU); no flush" % (a.leaves * a.leaf_rows * a.dim / 1e9),
    }


# ----------------------------------------------------------------- workload

def make_workload(torch, dev, a, seed):
    """Synthetic SQ8 leaf batch generated and quantized on the device."""
    from shear_b200 import ops

    rows = a.leaves * a.leaf_rows
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    pd = ops.padded_dim(a.dim, 16)
    codes = torch.empty((rows, pd), dtype=torch.int8, device=dev)
    scales = torch.empty(rows, dtype=torch.float32, device=dev)
    norms = torch.empty(rows, dtype=torch.float32, device=dev)
    chunk = 1 << 20
    for r0 in range(0, rows, chunk):
        r1 = min(rows, r0 + chunk)
        x = torch.randn((r1 - r0, a.dim), generator=g, device=dev, dtype=torch.float32)
        x /= torch.linalg.vector_norm(x, dim=1, keepdim=True)
        c, s, n = ops.quantize_sq8(x)
        codes[r0:r1].copy_(c)
        scales[r0:r1].copy_(s)
        norms[r0:r1].copy_(n)
        del x, c, s, n
    gids = torch.randperm(rows, generator=g, device=dev).to(torch.int32)
    members = torch.arange(rows, dtype=torch.int32, device=dev)
    starts = np.arange(a.leaves, dtype=np.uint64) * np.uint64(a.leaf_rows)
    sizes = np.full(a.leaves, a.leaf_rows, dtype=np.uint64)
    torch.cuda.synchronize(dev)
    return dict(codes=codes, scales=scales, norms=norms, gids=gids, members=members, starts=starts, sizes=sizes)


# ----------------------------------------------------------------- clocks

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.proc = None
        self.dev = device_index

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.dev)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not getattr(self, "out", ""):
            return None
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.strip().splitlines():
            f = [v.strip() for v in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return None
        loaded = [v for v in sm if v > 0.5 * max(sm)] or sm
        return {"sm_mhz": float(np.median(loaded)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------- peaks

def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except Exception:
        return {}


def int8_peak_tops(torch, dev):
    """Burst int8 GEMM rate of cuBLAS (torch._int_mm, 8192^3) on this GPU, TOP/s."""
    try:
        n = 8192
        a = torch.randint(-127, 127, (n, n), dtype=torch.int8, device=dev)
        b = torch.randint(-127, 127, (n, n), dtype=torch.int8, device=dev).t().contiguous().t()
        for _ in range(3):
            torch._int_mm(a, b)
        best = None
        for _ in range(10):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch._int_mm(a, b)
            e.record()
            e.synchronize()
            t = s.elapsed_time(e) / 1e3
            best = t if best is None else min(best, t)
        return 2.0 * n ** 3 / best / 1e12
    except Exception:
        return None


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one config-2
# leaf step, from one ncu capture of the three leaf kernels (one launch each)
# on 256 leaves of the same shape (400 MB of codes, 3x the L2), scaled by
# 4096/256 leaves (the fallback's share scales with its rows, 289 per 256
# leaves in the capture, 4,471 per step in the bench):
#   python bench.py --workload leaf --leaves 256 --steps 1 --warmup 3 --no-e2e --no-cpu-baseline &&
#   ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum \
#       --clock-control none -k regex:"leaf_topk_split|leaf_finish|leaf_fallback" -s 9 -c 3 \
#       python bench.py --workload leaf --leaves 256 --steps 1 --warmup 3 --no-e2e --no-cpu-baseline
LEAF_STEP_TRAFFIC = {"leaf_topk_split_kernel": 16 * 647565312, "leaf_finish_kernel": 16 * 335143680,
                     "leaf_fallback_kernel": 16 * 289767168}

# DRAM bytes of the build's leaf stage per unit, from one ncu capture (one
# launch of each kernel, in the fourth build) of the same build family at
# 200k rows (5,348 leaves, 6.0M leaf rows, 1.19e13 int8 ops; the full
# config-3 build is too large for a multi-metric capture): the main kernel's
# 9.47 GB per 1.1913e13 ops (its B re-reads grow with the leaves' all-pairs
# work) and the finishing kernel's 0.38 GB per 6.0M leaf rows (kernels with
# the A tile copied by tcgen05.cp and ceil(k/4) planes of merged distances).
#   python bench.py --workload build --config 3 --rows 200000 --steps 1 --warmup 3 --no-e2e --no-cpu-baseline --no-recall &&
#   ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum --clock-control none \
#       -k regex:"leaf_topk_split|leaf_finish" -s 6 -c 2 \
#       python bench.py --workload build --config 3 --rows 200000 --steps 1 --warmup 3 --no-e2e --no-cpu-baseline --no-recall
LEAF_BUILD_BYTES_PER_OP = (9198426112 + 274606336) / 11913301266432
LEAF_BUILD_FINISH_BYTES_PER_ROW = (307059200 + 72790528) / 6000000


def host_oracle():
    """The CPU restatement (test infrastructure) with every host core: torchrun
    sets OMP_NUM_THREADS=1 in each rank, which would leave it one thread."""
    from oracle import oracle as O
    O.set_num_threads(os.cpu_count() or 1)
    return O


# ----------------------------------------------------------------- CPU legs

def cpu_leaf_sample(oracle_mod, host, a, seconds, max_leaves):
    """Time the CPU restatement on whole leaves until `seconds` pass; rows/s."""
    threads = oracle_mod.num_threads()
    n = a.leaf_rows
    done_rows, t0, leaves = 0, time.perf_counter(), 0
    batch = max(1, threads)
    while leaves < max_leaves:
        cnt = min(batch, max_leaves - leaves)
        lo, hi = leaves * n, (leaves + cnt) * n
        members = np.arange(hi - lo, dtype=np.uint32)
        starts = np.arange(cnt, dtype=np.uint64) * np.uint64(n)
        sizes = np.full(cnt, n, np.uint64)
        oracle_mod.leaf_topk_sq8(host["codes"][lo:hi], host["scales"][lo:hi], host["norms"][lo:hi],
                                 host["gids"][lo:hi], members, starts, sizes, a.k)
        done_rows += hi - lo
        leaves += cnt
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return done_rows / dt, threads, leaves, dt


def reference_gpu_leaf(torch, w, a, sample_leaves=128):
    """The reference's own leaf kernel (gpu_persistent_subtree_topk_only, s8-WMMA
    filter, staged column tasks, launched as its replay session launches it) on
    the first `sample_leaves` leaves of the same workload, same B200, after our
    timed region; per-step time extrapolated by leaf count (the kernel is a
    persistent queue of independent leaf tasks)."""
    try:
        from oracle import refkernel as RK
    except Exception:
        return None
    if not RK.available():
        return None
    n = min(sample_leaves, a.leaves)
    host = host_sample(torch, w, n, a)
    rows = n * a.leaf_rows
    members = np.arange(rows, dtype=np.uint32)
    starts = np.arange(n, dtype=np.uint64) * np.uint64(a.leaf_rows)
    sizes = np.full(n, a.leaf_rows, np.uint64)
    try:
        _, _, counters, ms = RK.leaf_replay(host["codes"], host["scales"], host["norms"], host["gids"], members,
                                            starts, sizes, a.k, 2)
    except Exception as e:  # noqa: BLE001 - reported, not fatal to our arm
        return {"error": str(e)}
    step_ms = ms * a.leaves / n
    return {"kernel": "reference gpu_persistent_subtree_topk_only, SQ8 s8-WMMA filter (replay mode A3)",
            "value": a.leaves * a.leaf_rows / (step_ms / 1e3), "unit": "vectors/s",
            "ms_per_step": step_ms, "sample": f"{n} of {a.leaves} leaves in one launch ({ms:.1f} ms), "
                                              f"scaled by leaf count", "safety_gate": RK.leaf_safety_gate(counters, 2)}


def host_sample(torch, w, leaves, a):
    rows = leaves * a.leaf_rows
    return dict(codes=w["codes"][:rows].cpu().numpy(), scales=w["scales"][:rows].cpu().numpy(),
                norms=w["norms"][:rows].cpu().numpy(), gids=w["gids"][:rows].cpu().numpy().view(np.uint32))


def run_reference(a):
    """CPU restatement of the reference leaf operator (oracle port), rank 0 only."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    O = host_oracle()

    threads = O.num_threads()
    rng = np.random.default_rng(0)
    per_step = max(threads, 1)
    rows = per_step * a.leaf_rows
    x = rng.standard_normal((rows, a.dim)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    codes, scales, norms = O.quantize_sq8(x)
    gids = rng.permutation(rows).astype(np.uint32)
    members = np.arange(rows, dtype=np.uint32)
    starts = np.arange(per_step, dtype=np.uint64) * np.uint64(a.leaf_rows)
    sizes = np.full(per_step, a.leaf_rows, np.uint64)
    times = []
    for i in range(a.warmup + a.steps):
        t0 = time.perf_counter()
        O.leaf_topk_sq8(codes, scales, norms, gids, members, starts, sizes, a.k)
        dt = time.perf_counter() - t0
        if i >= a.warmup:
            times.append(dt)
    mean = float(np.mean(times))
    value = rows / mean
    sample = f"{per_step} leaves x {a.leaf_rows} rows per step ({per_step / a.leaves:.4%} of the workload)"
    line = {
        "impl": "reference", "metric": LEAF_METRIC, "value": value, "unit": "vectors/s",
        "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": mean * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic: N(0,1) rows, L2-normalised, SQ8 per-row int8 (seed 0)",
        "config": workload_desc(a),
        "cpu_baseline": {"value": value, "unit": "vectors/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "vectors/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference is Rust+NVRTC (no cargo in this image); timed leg is its leaf algorithm "
                "restated in C (oracle/tessa_oracle.c) on all host threads",
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------- our arm

def run_ours(a):
    import torch

    from shear_b200 import ops

    world, rank, local = dist_env()
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = ops.context(dev.index)
    w = make_workload(torch, dev, a, seed=1234 + rank)
    rows = a.leaves * a.leaf_rows
    ids = torch.empty(rows * a.k, dtype=torch.int32, device=dev)
    dists = torch.empty(rows * a.k, dtype=torch.float32, device=dev)

    def step():
        ops.leaf_topk_sq8(w["codes"], w["scales"], w["norms"], w["gids"], w["members"], w["starts"],
                          w["sizes"], a.k, leaf_ordered_codes=w["codes"], out=(ids, dists), ctx=ctx)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    for _ in range(max(a.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    with ClockSampler(dev.index) as clk:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for s, e in evs:
            s.record(stream)
            step()
            e.record(stream)
        t_end.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    total_s = t_start.elapsed_time(t_end) / 1e3
    kern_s = float(np.mean([s.elapsed_time(e) for s, e in evs])) / 1e3
    if world > 1:
        import torch.distributed as dist
        tt = torch.tensor([total_s, kern_s], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_s, kern_s = float(tt[0]), float(tt[1])
    per_step = total_s / a.steps
    value = world * rows / per_step
    fb_rows = ops.leaf_last_fallback_rows(ctx)  # rows of the last step sent to the exact fallback
    pairs = a.leaves * a.leaf_rows * (a.leaf_rows - 1)
    ops_per_step = 2.0 * a.dim * a.leaf_rows * a.leaf_rows * a.leaves  # int8 MAC*2 incl. the diagonal tile

    # ------------------------------------------------------------- e2e
    e2e = None
    if not a.no_e2e and a.e2e_steps > 0:
        pin = lambda t: t.cpu().pin_memory()
        hc, hs, hn, hg = pin(w["codes"]), pin(w["scales"]), pin(w["norms"]), pin(w["gids"])
        hm = pin(w["members"])
        oi = torch.empty(rows * a.k, dtype=torch.int32).pin_memory()
        od = torch.empty(rows * a.k, dtype=torch.float32).pin_memory()
        nv = lambda t: t.numpy()
        args = (nv(hc), nv(hs), nv(hn), nv(hg).view(np.uint32), nv(hm).view(np.uint32), w["starts"],
                w["sizes"], a.k)
        ops.leaf_topk_sq8_host(*args, device=dev.index, out=(nv(oi).view(np.uint32), nv(od)))
        barrier()
        t0 = time.perf_counter()
        for _ in range(a.e2e_steps):
            ops.leaf_topk_sq8_host(*args, device=dev.index, out=(nv(oi).view(np.uint32), nv(od)))
        e2e_s = (time.perf_counter() - t0) / a.e2e_steps
        if world > 1:
            import torch.distributed as dist
            tt = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e2e_s = float(tt[0])
        h2d = hc.numel() + 4 * (hs.numel() + hn.numel() + hg.numel() + hm.numel())
        d2h = 8 * rows * a.k
        e2e = {"value": world * rows / e2e_s, "unit": "vectors/s", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_s * 1e3,
               "timing": "wall clock around the synchronous host-buffer C-ABI call, pinned host memory"}
        del hc, hs, hn, hg, hm, oi, od

    if rank != 0:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return 0

    peaks = measured_peaks()
    int8_peak = int8_peak_tops(torch, dev)
    achieved_tops = ops_per_step / kern_s / 1e12
    peak, src = (int8_peak, "measured in-run: cuBLAS int8 burst (torch._int_mm 8192^3)") if int8_peak else \
        (NOMINAL_INT8_TOPS, "nominal B200 dense int8 4.5 POPS (no measured int8 peak)")
    # The committed ncu figure is for the full config-2 launch only.
    full_cfg = (a.leaves, a.leaf_rows, a.dim, a.k) == (4096, 2048, 768, 32)
    traffic = sum(v for v in LEAF_STEP_TRAFFIC.values() if v) if full_cfg else None
    roofline = {"bound": "tensor", "achieved": achieved_tops, "peak": peak, "unit": "TOP/s",
                "frac": achieved_tops / peak, "traffic": traffic, "peak_source": src,
                "frac_of_nominal_4500": achieved_tops / NOMINAL_INT8_TOPS,
                "kernel": "tessa::leaf::split::leaf_topk_split_kernel<32> (+ leaf_finish_kernel)",
                "algorithmic_ops_per_launch": ops_per_step,
                "hbm_bytes_algorithmic": rows * (a.dim + 16) + rows * a.k * 8,
                "hbm_peak_gbs": peaks.get("hbm_gbs")}

    cpu = None
    if not a.no_cpu_baseline and world == 1:
        O = host_oracle()
        max_leaves = max(O.num_threads(), 1) * 32  # ~10 s of OpenMP work; the time limit ends it
        host = host_sample(torch, w, min(a.leaves, max_leaves), a)
        v, thr, nl, dt = cpu_leaf_sample(O, host, a, a.cpu_seconds, min(a.leaves, max_leaves))
        cpu = {"value": v, "unit": "vectors/s", "cores": thr, "kind": "port",
               "sample": f"{nl} of {a.leaves} leaves ({nl * a.leaf_rows} rows) in {dt:.1f} s, "
                         f"oracle/tessa_oracle.c OpenMP"}

    ref_gpu = reference_gpu_leaf(torch, w, a) if world == 1 else None

    line = {
        "metric": LEAF_METRIC, "value": value, "unit": "vectors/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic: N(0,1) rows, L2-normalised, SQ8 per-row int8 (seed 1234+rank)",
        "config": dict(workload_desc(a), parallelism=f"leaf-sharded x{world} (independent, no collective)"),
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": 3 * a.steps,  # column-split leaf kernel, finishing kernel, exact fallback per step
        "clocks": clk.summary(),
        "leaf_kernel_ms": kern_s * 1e3, "pairs_per_sec": world * pairs / per_step,
        "fallback_rows_per_step": fb_rows,
        "int8_tops": achieved_tops,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ----------------------------------------------------------------- global D0

def d0_desc(a):
    return {
        "workload": f"global-D0 SQ8 staging (quantize_sq8_and_assign_global_d0): {a.d0_rows} raw rows x "
                    f"{a.dim}-d f32 per GPU, {a.d0_leaders} leaders, fanout {a.d0_fanout}",
        "rows": a.d0_rows, "dim": a.dim, "leaders": a.d0_leaders, "fanout": a.d0_fanout,
        "l2": "inputs larger than L2 (raw rows %.1f GB per GPU); no flush" % (a.d0_rows * a.dim * 4 / 1e9),
    }


def make_d0_workload(torch, dev, a, seed):
    """Unit-normal rows on the device; leaders are rows of the batch (the
    reference samples its root leaders from the data)."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.empty((a.d0_rows, a.dim), dtype=torch.float32, device=dev)
    chunk = 1 << 18
    for r0 in range(0, a.d0_rows, chunk):
        r1 = min(a.d0_rows, r0 + chunk)
        y = torch.randn((r1 - r0, a.dim), generator=g, device=dev, dtype=torch.float32)
        x[r0:r1] = y / torch.linalg.vector_norm(y, dim=1, keepdim=True)
    pick = torch.randperm(a.d0_rows, generator=g, device=dev)[:a.d0_leaders]
    gids = (torch.arange(a.d0_rows, device=dev, dtype=torch.int64) + seed * a.d0_rows).to(torch.int32)
    lv = x[pick].contiguous()
    lids = gids[pick].contiguous()
    torch.cuda.synchronize(dev)
    return x, gids, lids, lv


def run_d0_reference(a):
    """CPU restatement of quantize_sq8_and_assign_global_d0_reference (oracle port), rank 0 only."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    O = host_oracle()

    threads = O.num_threads()
    rng = np.random.default_rng(0)
    rows = max(threads, 1) * 512
    x = rng.standard_normal((rows, a.dim)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    pick = rng.permutation(rows)[:a.d0_leaders]
    gids = np.arange(rows, dtype=np.uint32)
    times = []
    for i in range(a.warmup + a.steps):
        t0 = time.perf_counter()
        O.d0_assign(x, gids, gids[pick], x[pick], a.d0_fanout)
        dt = time.perf_counter() - t0
        if i >= a.warmup:
            times.append(dt)
    mean = float(np.mean(times))
    value = rows / mean
    line = {
        "impl": "reference", "metric": "D0 staging rows/sec", "value": value, "unit": "rows/s",
        "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": mean * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic: N(0,1) rows, L2-normalised (seed 0)", "config": d0_desc(a),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port",
                         "sample": f"{rows} rows per step ({rows / a.d0_rows:.2%} of the per-GPU batch)"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's quantize + D0 assignment restated in C (oracle/tessa_oracle.c), OpenMP",
    }
    print(json.dumps(line), flush=True)
    return 0


def run_d0(a):
    import torch

    from shear_b200 import ops

    world, rank, local = dist_env()
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = ops.context(dev.index)
    x, gids, lids, lv = make_d0_workload(torch, dev, a, seed=1 + rank)
    rows, f, L = a.d0_rows, a.d0_fanout, a.d0_leaders
    pd = ops.padded_dim(a.dim)
    out = (torch.empty((rows, pd), dtype=torch.int8, device=dev), torch.empty(rows, device=dev),
           torch.empty(rows, device=dev), torch.empty(rows * f, dtype=torch.int32, device=dev),
           torch.empty(rows * f, dtype=torch.int32, device=dev), torch.empty(rows * f, device=dev))
    assign_ms = []

    def step(record=False):
        ops.quantize_sq8_assign_d0(x, gids, lids, f, leader_vectors=lv, ctx=ctx, out=out)
        if record:
            assign_ms.append(ops.d0_last_profile(ctx)["assign_ms"])

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    for _ in range(max(a.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    with ClockSampler(dev.index) as clk:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for _ in range(a.steps):
            step(record=True)
        t_end.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    total_s = t_start.elapsed_time(t_end) / 1e3
    kern_s = float(np.mean(assign_ms)) / 1e3
    if world > 1:
        import torch.distributed as dist
        tt = torch.tensor([total_s, kern_s], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_s, kern_s = float(tt[0]), float(tt[1])
    per_step = total_s / a.steps
    value = world * rows / per_step
    ops_per_step = 2.0 * rows * L * pd
    prof = ops.d0_last_profile(ctx)  # phases of the last timed step (before the host-buffer calls)

    e2e = None
    if not a.no_e2e and a.e2e_steps > 0:
        pin = lambda t: t.cpu().pin_memory()
        hx, hg, hl, hv = pin(x), pin(gids), pin(lids), pin(lv)
        hout = tuple(torch.empty(t.shape, dtype=t.dtype).pin_memory().numpy() for t in out)
        hout = (hout[0], hout[1], hout[2], hout[3].view(np.uint32), hout[4].view(np.uint32), hout[5])
        args = (hx.numpy(), hg.numpy().view(np.uint32), hl.numpy().view(np.uint32), hv.numpy(), f)
        ops.quantize_sq8_and_assign_global_d0(*args, device=dev.index, out=hout)
        barrier()
        t0 = time.perf_counter()
        for _ in range(a.e2e_steps):
            ops.quantize_sq8_and_assign_global_d0(*args, device=dev.index, out=hout)
        e2e_s = (time.perf_counter() - t0) / a.e2e_steps
        if world > 1:
            import torch.distributed as dist
            tt = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e2e_s = float(tt[0])
        h2d = hx.numel() * 4 + hg.numel() * 4 + hl.numel() * 4 + hv.numel() * 4
        d2h = rows * pd + rows * 8 + rows * f * 12
        e2e = {"value": world * rows / e2e_s, "unit": "rows/s", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_s * 1e3,
               "timing": "wall clock around the synchronous host-buffer C-ABI call, pinned host memory"}
        del hx, hg, hl, hv, hout

    if rank != 0:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return 0

    int8_peak = int8_peak_tops(torch, dev)
    achieved = ops_per_step / kern_s / 1e12
    peak, src = (int8_peak, "measured in-run: cuBLAS int8 burst (torch._int_mm 8192^3)") if int8_peak else \
        (NOMINAL_INT8_TOPS, "nominal B200 dense int8 4.5 POPS (no measured int8 peak)")
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOP/s", "frac": achieved / peak,
                "traffic": None, "peak_source": src, "frac_of_nominal_4500": achieved / NOMINAL_INT8_TOPS,
                "kernel": f"tessa::leaf::leaf_topk_sq8_kernel<{next(v for v in (2, 4, 8, 16, 32) if f <= v)}, true>",
                "algorithmic_ops_per_launch": ops_per_step, "kernel_ms": kern_s * 1e3}

    cpu = None
    if not a.no_cpu_baseline and world == 1:
        O = host_oracle()
        hx = x[: min(rows, 1 << 17)].cpu().numpy()
        hg = gids[: hx.shape[0]].cpu().numpy().view(np.uint32)
        hl, hv = lids.cpu().numpy().view(np.uint32), lv.cpu().numpy()
        done, t0, chunk = 0, time.perf_counter(), max(O.num_threads(), 1) * 256
        while done < hx.shape[0]:
            O.d0_assign(hx[done:done + chunk], hg[done:done + chunk], hl, hv, f)
            done += min(chunk, hx.shape[0] - done)
            if time.perf_counter() - t0 >= a.cpu_seconds:
                break
        dt = time.perf_counter() - t0
        cpu = {"value": done / dt, "unit": "rows/s", "cores": O.num_threads(), "kind": "port",
               "sample": f"{done} of {rows} rows in {dt:.1f} s (quantize + assign), oracle/tessa_oracle.c OpenMP"}

    line = {
        "metric": "D0 staging rows/sec", "value": value, "unit": "rows/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic: N(0,1) rows, L2-normalised, leaders drawn from the rows (seed 1+rank)",
        "config": dict(d0_desc(a), parallelism=f"row-sharded x{world} (independent, no collective)"),
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": 5 * a.steps,  # leader quantize, row quantize, assignment, fallback, fragments
        "clocks": clk.summary(),
        "profile_last_step": prof,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ----------------------------------------------------------------- candidate edges

def edges_desc(a):
    return {
        "workload": f"candidate edges of the leaf lists (flush_compact_topk_batch_into_edges): {a.leaves} leaves x "
                    f"{a.leaf_rows} rows, top-{a.k}, {a.hash_bits}-bit sketch hashes, both directions",
        "leaves": a.leaves, "leaf_rows": a.leaf_rows, "k": a.k, "hash_bits": a.hash_bits,
        "l2": "slot arrays larger than L2 (%.1f GB of ids); no flush" % (a.leaves * a.leaf_rows * a.k * 4 / 1e9),
    }


def edges_inputs(torch, dev, a, seed):
    """Leaf lists of the config-2 workload (one leaf-kernel run) and a sketch
    store over every global id (unit-normal sketches; sketch values do not
    change the hash cost)."""
    from shear_b200 import ops

    w = make_workload(torch, dev, a, seed)
    rows = a.leaves * a.leaf_rows
    ids = torch.empty(rows * a.k, dtype=torch.int32, device=dev)
    dists = torch.empty(rows * a.k, dtype=torch.float32, device=dev)
    ops.leaf_topk_sq8(w["codes"], w["scales"], w["norms"], w["gids"], w["members"], w["starts"], w["sizes"], a.k,
                      leaf_ordered_codes=w["codes"], out=(ids, dists))
    point_ids = w["gids"]  # members are the identity: leaf row r holds global id gids[r]
    g = torch.Generator(device=dev)
    g.manual_seed(seed + 7)
    sketches = torch.randn((rows, a.hash_bits), generator=g, device=dev, dtype=torch.float32)
    layout = (w["starts"], w["sizes"])
    del w
    torch.cuda.synchronize(dev)
    return point_ids, ids, dists, sketches, layout


def run_edges_reference(a):
    """The reference's flush (hash from sketches + edge expansion) restated in C, rank 0 only."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    from concurrent.futures import ThreadPoolExecutor

    O = host_oracle()

    threads = O.num_threads()
    rng = np.random.default_rng(0)
    per_step = max(threads, 1) * 4  # leaves per step
    rows = per_step * a.leaf_rows
    n_points = rows
    sk = rng.standard_normal((n_points, a.hash_bits)).astype(np.float32)
    pid = rng.permutation(n_points).astype(np.uint32)
    ids = rng.integers(0, n_points, rows * a.k).astype(np.uint32)
    ds = rng.uniform(0, 2, rows * a.k).astype(np.float32)

    def one(l):
        lo, hi = l * a.leaf_rows, (l + 1) * a.leaf_rows
        return O.flush_edges(pid[lo:hi], ids[lo * a.k:hi * a.k], ds[lo * a.k:hi * a.k], a.k, sk, a.hash_bits)[0].size

    times = []
    with ThreadPoolExecutor(max_workers=max(threads, 1)) as ex:
        for i in range(a.warmup + a.steps):
            t0 = time.perf_counter()
            n_edges = sum(ex.map(one, range(per_step)))
            dt = time.perf_counter() - t0
            if i >= a.warmup:
                times.append(dt)
    mean = float(np.mean(times))
    value = n_edges / mean
    line = {
        "impl": "reference", "metric": "candidate edges/sec", "value": value, "unit": "edges/s",
        "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": mean * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: random leaf lists and unit-normal sketches (seed 0)", "config": edges_desc(a),
        "cpu_baseline": {"value": value, "unit": "edges/s", "cores": threads, "kind": "port",
                         "sample": f"{per_step} leaves x {a.leaf_rows} rows x {a.k} slots per step"},
        "e2e": {"value": value, "unit": "edges/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference flush restated in C (oracle/tessa_oracle.c), one host thread per leaf batch",
    }
    print(json.dumps(line), flush=True)
    return 0


def run_edges(a):
    import torch

    from shear_b200 import ops

    world, rank, local = dist_env()
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = ops.context(dev.index)
    point_ids, ids, dists, sketches, layout = edges_inputs(torch, dev, a, seed=1234 + rank)
    rows = a.leaves * a.leaf_rows
    slots = rows * a.k
    hf = torch.empty(slots, dtype=torch.int16, device=dev)
    hr = torch.empty(slots, dtype=torch.int16, device=dev)
    n_valid = int((ids != -1).sum())

    def step():
        ops.edge_hashes(point_ids, ids, a.k, sketches, a.hash_bits, *layout, ctx=ctx, out=(hf, hr))

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    for _ in range(max(a.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    barrier()
    stream = torch.cuda.current_stream(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    with ClockSampler(dev.index) as clk:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for s_, e_ in evs:
            s_.record(stream)
            step()
            e_.record(stream)
        t_end.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    total_s = t_start.elapsed_time(t_end) / 1e3
    kern_s = float(np.mean([s_.elapsed_time(e_) for s_, e_ in evs])) / 1e3
    if world > 1:
        import torch.distributed as dist
        tt = torch.tensor([total_s, kern_s], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_s, kern_s = float(tt[0]), float(tt[1])
    per_step = total_s / a.steps
    value = world * 2 * n_valid / per_step

    # sketch kernel on 1M x 768 f32 rows (fill_sketch_row for the store)
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    xs = torch.randn((1 << 20, a.dim), generator=g, device=dev)
    planes = torch.rand((a.hash_bits, a.dim), generator=g, device=dev) * 2 - 1
    sk_out = torch.empty((1 << 20, a.hash_bits), device=dev)
    for _ in range(3):
        ops.sketch_rows(xs, planes, ctx=ctx, out=sk_out)
    torch.cuda.synchronize(dev)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(5):
        ops.sketch_rows(xs, planes, ctx=ctx, out=sk_out)
    s1.record(stream)
    torch.cuda.synchronize(dev)
    sketch_ms = s0.elapsed_time(s1) / 5
    del xs, sk_out

    e2e = None
    if not a.no_e2e and a.e2e_steps > 0:
        h_pid = point_ids.cpu().numpy().view(np.uint32)
        h_ids = torch.empty(slots, dtype=torch.int32).pin_memory()
        h_d = torch.empty(slots, dtype=torch.float32).pin_memory()
        h_hf = torch.empty(slots, dtype=torch.int16).pin_memory()
        h_hr = torch.empty(slots, dtype=torch.int16).pin_memory()

        def e2e_step():
            step()
            h_ids.copy_(ids, non_blocking=True)
            h_d.copy_(dists, non_blocking=True)
            h_hf.copy_(hf, non_blocking=True)
            h_hr.copy_(hr, non_blocking=True)
            torch.cuda.synchronize(dev)
            return ops.expand_edges(h_pid, h_ids.numpy(), h_d.numpy(), h_hf.numpy(), h_hr.numpy(), a.k)

        e2e_step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(a.e2e_steps):
            out = e2e_step()
        e2e_s = (time.perf_counter() - t0) / a.e2e_steps
        assert out[0].shape[0] == 2 * n_valid
        del out
        if world > 1:
            import torch.distributed as dist
            tt = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e2e_s = float(tt[0])
        e2e = {"value": world * 2 * n_valid / e2e_s, "unit": "edges/s", "h2d_bytes_per_step": 0,
               "d2h_bytes_per_step": int(slots * 12), "ms_per_step": e2e_s * 1e3,
               "timing": "wall clock: hash kernel, D2H of ids, distances and both hashes into pinned memory, "
                         "host expansion into edge arrays (all host threads)"}

    if rank != 0:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return 0

    peaks = measured_peaks()
    hbm = peaks.get("hbm_gbs") or 6650.0
    # algorithmic bytes per launch: ids in, both hashes out, each row's point id
    # and every global id's sketch once
    alg_bytes = slots * 4 + slots * 4 + rows * 4 + rows * a.hash_bits * 4
    achieved = alg_bytes / kern_s / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": None, "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks.get("hbm_gbs") else "fallback",
                "kernel": "tessa::edges::leaf_edge_hashes_kernel", "algorithmic_bytes_per_launch": alg_bytes,
                "kernel_ms": kern_s * 1e3}

    cpu = None
    if not a.no_cpu_baseline and world == 1:
        from concurrent.futures import ThreadPoolExecutor

        O = host_oracle()
        threads = O.num_threads()
        nl = min(a.leaves, max(threads, 1) * 16)
        h_sk = sketches.cpu().numpy()
        h_pid = point_ids[: nl * a.leaf_rows].cpu().numpy().view(np.uint32)
        h_ids = ids[: nl * a.leaf_rows * a.k].cpu().numpy().view(np.uint32)
        h_d = dists[: nl * a.leaf_rows * a.k].cpu().numpy()

        def one(l):
            lo, hi = l * a.leaf_rows, (l + 1) * a.leaf_rows
            return O.flush_edges(h_pid[lo:hi], h_ids[lo * a.k:hi * a.k], h_d[lo * a.k:hi * a.k], a.k, h_sk,
                                 a.hash_bits)[0].size

        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=max(threads, 1)) as ex:
            n_e = sum(ex.map(one, range(nl)))
        dt = time.perf_counter() - t0
        cpu = {"value": n_e / dt, "unit": "edges/s", "cores": threads, "kind": "port",
               "sample": f"{nl} of {a.leaves} leaves in {dt:.1f} s (hash from sketches + expansion), "
                         f"oracle/tessa_oracle.c, one thread per leaf"}

    line = {
        "metric": "candidate edges/sec", "value": value, "unit": "edges/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: config-2 leaf lists from the leaf kernel, unit-normal sketches (seed 1234+rank)",
        "config": dict(edges_desc(a), parallelism=f"leaf-sharded x{world} (independent, no collective)"),
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": a.steps, "clocks": clk.summary(),
        "edges_per_step": 2 * n_valid, "sketch_rows_per_sec": (1 << 20) / (sketch_ms / 1e3),
        "sketch_ms_1Mx768": sketch_ms,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ----------------------------------------------------------------- assignment

def assign_desc(a):
    src = "fp32 rows (A0)" if a.assign_fp32 else "SQ8 codes"
    return {
        "workload": f"TESSA assignment replay: {a.leaves} tasks x {a.leaf_rows} member rows, {a.dim}-d {src}, "
                    f"{a.assign_leaders} leaders per task, r_h = {a.assign_rh}",
        "tasks": a.leaves, "task_rows": a.leaf_rows, "dim": a.dim, "leaders": a.assign_leaders, "r_h": a.assign_rh,
        "source": src, "l2": "member rows larger than L2; no flush",
    }


def assign_tasks(a, rng):
    """Contiguous tasks of leaf_rows members; each task's leaders are members of it."""
    n = a.leaves * a.leaf_rows
    moff = (np.arange(a.leaves, dtype=np.uint64) * a.leaf_rows).astype(np.uint32)
    mcnt = np.full(a.leaves, a.leaf_rows, np.uint32)
    pick = np.stack([rng.choice(a.leaf_rows, a.assign_leaders, replace=False) for _ in range(a.leaves)])
    leaders = (pick + moff[:, None]).astype(np.uint32).reshape(-1)
    loff = (np.arange(a.leaves, dtype=np.uint64) * a.assign_leaders).astype(np.uint32)
    lcnt = np.full(a.leaves, a.assign_leaders, np.uint32)
    rh = np.full(a.leaves, a.assign_rh, np.uint32)
    outoff = (moff.astype(np.uint64) * a.assign_rh).astype(np.uint64)
    return n, leaders, moff, mcnt, loff, lcnt, rh, outoff


def run_assign_reference(a):
    """The reference's assignment replay restated in C (oracle port) on a task sample, rank 0 only."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    O = host_oracle()

    rng = np.random.default_rng(0)
    b = argparse.Namespace(**vars(a))
    b.leaves = max(O.num_threads(), 1) * 2
    n, leaders, moff, mcnt, loff, lcnt, rh, outoff = assign_tasks(b, rng)
    x = rng.standard_normal((n, a.dim)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    codes, scales, qn = O.quantize_sq8(x)
    norms = O.raw_norms(x) if a.assign_fp32 else qn
    mode = 0 if a.assign_fp32 else 3
    gids = np.arange(n, dtype=np.uint32)
    members = np.arange(n, dtype=np.uint32)
    times = []
    for i in range(a.warmup + a.steps):
        t0 = time.perf_counter()
        O.assign(mode, x, norms, codes, scales, gids, members, leaders, moff, mcnt, loff, lcnt, rh, outoff,
                 n * a.assign_rh)
        dt = time.perf_counter() - t0
        if i >= a.warmup:
            times.append(dt)
    mean = float(np.mean(times))
    value = n / mean
    line = {
        "impl": "reference", "metric": "assignment rows/sec", "value": value, "unit": "rows/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": mean * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32" if a.assign_fp32 else "int8",
        "data": "synthetic: N(0,1) rows, L2-normalised (seed 0)", "config": assign_desc(a),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": O.num_threads(), "kind": "port",
                         "sample": f"{b.leaves} tasks x {a.leaf_rows} rows per step"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "assignment replay restated in C (oracle/tessa_oracle.c), sequential per task",
    }
    print(json.dumps(line), flush=True)
    return 0


def run_assign(a):
    import torch

    from shear_b200 import _capi as CA, ops

    world, rank, local = dist_env()
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = ops.context(dev.index)
    rng = np.random.default_rng(1 + rank)
    n, leaders, moff, mcnt, loff, lcnt, rh, outoff = assign_tasks(a, rng)
    g = torch.Generator(device=dev)
    g.manual_seed(3 + rank)
    x = torch.empty((n, a.dim), dtype=torch.float32, device=dev)
    for r0 in range(0, n, 1 << 20):
        y = torch.randn((min(n, r0 + (1 << 20)) - r0, a.dim), generator=g, device=dev)
        x[r0:r0 + y.shape[0]] = y / torch.linalg.vector_norm(y, dim=1, keepdim=True)
    codes, scales, qn = ops.quantize_sq8(x)
    raw_norms = (x * x).sum(1) if a.assign_fp32 else None
    if not a.assign_fp32:
        del x
        x = None
    gids = torch.arange(n, dtype=torch.int32, device=dev)
    members = gids
    lead = torch.from_numpy(leaders.view(np.int32)).to(dev)
    torch.cuda.synchronize(dev)
    src = CA.ASSIGN_FP32 if a.assign_fp32 else CA.ASSIGN_SQ8

    def step():
        if a.assign_fp32:
            return ops.assign(src, x=x, raw_norms=raw_norms, global_ids=gids, members=members, leaders=lead,
                              task_member_offsets=moff, task_member_counts=mcnt, task_leader_offsets=loff,
                              task_leader_counts=lcnt, task_rh=rh, task_output_offsets=outoff,
                              output_len=n * a.assign_rh, ctx=ctx)
        return ops.assign(src, codes=codes, scales=scales, sq8_norms=qn, global_ids=gids, members=members,
                          leaders=lead, task_member_offsets=moff, task_member_counts=mcnt, task_leader_offsets=loff,
                          task_leader_counts=lcnt, task_rh=rh, task_output_offsets=outoff,
                          output_len=n * a.assign_rh, ctx=ctx)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    for _ in range(max(a.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    barrier()
    stream = torch.cuda.current_stream(dev)
    with ClockSampler(dev.index) as clk:
        t0e, t1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0e.record(stream)
        for _ in range(a.steps):
            step()
        t1e.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    total_s = t0e.elapsed_time(t1e) / 1e3
    if world > 1:
        import torch.distributed as dist
        tt = torch.tensor([total_s], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_s = float(tt[0])
    per_step = total_s / a.steps
    value = world * n / per_step
    if rank != 0:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return 0
    # ---- e2e: the step's rows from pinned host memory, tessa_assign, results back
    e2e = None
    if not a.no_e2e and a.e2e_steps > 0 and world == 1:
        if a.assign_fp32:
            hx, hn = x.cpu().pin_memory(), raw_norms.cpu().pin_memory()
            dx, dn = torch.empty_like(x), torch.empty_like(raw_norms)
            h2d = hx.numel() * 4 + hn.numel() * 4
        else:
            hc, hs, hq = codes.cpu().pin_memory(), scales.cpu().pin_memory(), qn.cpu().pin_memory()
            dc, ds_, dq = torch.empty_like(codes), torch.empty_like(scales), torch.empty_like(qn)
            h2d = hc.numel() + hs.numel() * 4 + hq.numel() * 4
        oi = torch.empty(n * a.assign_rh, dtype=torch.int32).pin_memory()
        od = torch.empty(n * a.assign_rh, dtype=torch.float32).pin_memory()

        def e2e_step():
            if a.assign_fp32:
                dx.copy_(hx, non_blocking=True)
                dn.copy_(hn, non_blocking=True)
                ids, dists = ops.assign(src, x=dx, raw_norms=dn, global_ids=gids, members=members, leaders=lead,
                                        task_member_offsets=moff, task_member_counts=mcnt, task_leader_offsets=loff,
                                        task_leader_counts=lcnt, task_rh=rh, task_output_offsets=outoff,
                                        output_len=n * a.assign_rh, ctx=ctx)
            else:
                dc.copy_(hc, non_blocking=True)
                ds_.copy_(hs, non_blocking=True)
                dq.copy_(hq, non_blocking=True)
                ids, dists = ops.assign(src, codes=dc, scales=ds_, sq8_norms=dq, global_ids=gids, members=members,
                                        leaders=lead, task_member_offsets=moff, task_member_counts=mcnt,
                                        task_leader_offsets=loff, task_leader_counts=lcnt, task_rh=rh,
                                        task_output_offsets=outoff, output_len=n * a.assign_rh, ctx=ctx)
            oi.copy_(ids, non_blocking=True)
            od.copy_(dists, non_blocking=True)
            torch.cuda.synchronize(dev)
        e2e_step()
        t0 = time.perf_counter()
        for _ in range(a.e2e_steps):
            e2e_step()
        e2e_s = (time.perf_counter() - t0) / a.e2e_steps
        e2e = {"value": n / e2e_s, "unit": "rows/s", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(n * a.assign_rh * 8), "ms_per_step": e2e_s * 1e3,
               "timing": "wall clock: pinned H2D of the rows, tessa_assign, D2H of ids and distances"}

    cpu = None
    if not a.no_cpu_baseline and world == 1:
        O = host_oracle()
        t_take = min(a.leaves, max(O.num_threads(), 1) * 8)
        sel = slice(0, t_take)
        rows_s = int(np.sum(mcnt[sel]))
        xs = (x[:rows_s].cpu().numpy() if a.assign_fp32 else np.zeros((rows_s, 1), np.float32))
        ns = (raw_norms if a.assign_fp32 else qn)[:rows_s].cpu().numpy()
        cs, ss = codes[:rows_s].cpu().numpy(), scales[:rows_s].cpu().numpy()
        g_s = np.arange(rows_s, dtype=np.uint32)
        lds = leaders[:int(np.sum(lcnt[sel]))]
        outs = np.asarray(outoff[sel], np.uint64)
        t0 = time.perf_counter()
        O.assign(0 if a.assign_fp32 else 3, xs, ns, cs, ss, g_s, g_s, lds, moff[sel], mcnt[sel], loff[sel],
                 lcnt[sel], rh[sel], outs, rows_s * a.assign_rh)
        dt = time.perf_counter() - t0
        cpu = {"value": rows_s / dt, "unit": "rows/s", "cores": O.num_threads(), "kind": "port",
               "sample": f"{t_take} of {a.leaves} tasks ({rows_s} rows) in {dt:.2f} s, oracle/tessa_oracle.c "
                         f"oracle_assign (OpenMP over rows)"}

    peaks = measured_peaks()
    hbm = peaks.get("hbm_gbs") or 6650.0
    row_bytes = a.dim * 4 + 4 if a.assign_fp32 else codes.shape[1] + 8
    # algorithmic bytes: every member row (and its norm / scale) once, leaders
    # once per task, the outputs (id + distance per r_h slot)
    alg = n * row_bytes + a.leaves * a.assign_leaders * row_bytes + n * a.assign_rh * 8
    achieved = alg / per_step / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": None,
                "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks.get("hbm_gbs") else "fallback",
                "kernel": ("tessa::assign::assign_kernel<false, LG> (FP32, SIMT)" if a.assign_fp32
                           else "tessa::assign::tc::assign_tc_kernel<NB> (SQ8, tcgen05)"),
                "algorithmic_bytes_per_launch": alg, "kernel_ms": per_step * 1e3,
                "note": "per-step time includes the host-side task table build and one host sync"}
    line = {
        "metric": "assignment rows/sec", "value": value, "unit": "rows/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32" if a.assign_fp32 else "int8",
        "data": "synthetic: N(0,1) rows, L2-normalised; leaders drawn from each task's members (seed 1+rank)",
        "config": dict(assign_desc(a), parallelism=f"task-sharded x{world} (independent, no collective)"),
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": a.steps,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ----------------------------------------------------------------- build (configs 1 and 3)

BUILD_METRIC = "build vectors/sec"
BUILD_CONFIGS = {
    # 200k x 128 GMM (64 components, centres N(0,1), isotropic sigma 0.3,
    # seed 0), L2, leaf size 1024, degree 64, recall@10 on 1,000 queries (seed 1)
    1: dict(rows=200_000, dim=128, comps=64, aniso=False, unit=False, sigma=0.3, queries=1000, c_max=1024),
    # 1M x 768 L2-normalised, 1,024-component anisotropic GMM (diagonal
    # sigma ~ U[0.05, 0.5]), inner product on unit vectors = L2 order, degree 64, 10,000 queries
    3: dict(rows=1_000_000, dim=768, comps=1024, aniso=True, unit=True, sigma=None, queries=10_000, c_max=2048),
    # 35M x 768, the config-3 family with 4,096 components, 1/2/4/8 GPUs; rows
    # drawn per 2^18-row chunk from the chunk's own seed, so each rank draws only its row range and every
    # GPU count builds the same dataset (107.5 GB of f32 rows in all)
    4: dict(rows=35_000_000, dim=768, comps=4096, aniso=True, unit=True, sigma=None, queries=10_000, c_max=2048,
            chunked=True),
}


def build_cfg(a):
    c = dict(BUILD_CONFIGS[a.config])
    if a.rows:
        c["rows"] = a.rows
    if a.queries:
        c["queries"] = a.queries
    return c


def build_desc(a, c):
    return {"workload": f"GPU-subtree index build, BASELINE config {a.config}: {c['rows']} x {c['dim']} "
                        f"{'L2-normalised ' if c['unit'] else ''}{c['comps']}-component "
                        f"{'anisotropic' if c['aniso'] else 'isotropic'} Gaussian mixture, leaf size "
                        f"{c['c_max']}, degree 64, recall@10 on {c['queries']} queries",
            "rows": c["rows"], "dim": c["dim"], "c_max": c["c_max"], "leaf_knn": 2, "l_max": 64,
            "fanout_top": 10, "fanout_second": 3,
            "l2": "inputs larger than L2 (%.2f GB of rows); no flush" % (c["rows"] * c["dim"] * 4 / 1e9)}


def make_mixture_np(n, c, seed, centre_seed=0):
    """The config's mixture on the host (numpy), same procedure as make_mixture."""
    rng = np.random.default_rng(centre_seed)
    centres = rng.standard_normal((c["comps"], c["dim"])).astype(np.float32)
    sig = (rng.random((c["comps"], c["dim"])) * 0.45 + 0.05).astype(np.float32) if c["aniso"] else None
    r2 = np.random.default_rng(seed)
    comp = r2.integers(0, c["comps"], n)
    noise = r2.standard_normal((n, c["dim"])).astype(np.float32)
    x = centres[comp] + (sig[comp] * noise if c["aniso"] else np.float32(c["sigma"]) * noise)
    if c["unit"]:
        x /= np.linalg.norm(x, axis=1, keepdims=True)
    return np.ascontiguousarray(x, np.float32)


def make_mixture(torch, dev, n, c, seed, centre_seed=0):
    """Synthetic stand-in for the config's dataset on the device (centres and
    per-component sigmas from centre_seed, draws from seed)."""
    g = torch.Generator(device=dev)
    g.manual_seed(centre_seed)
    centres = torch.randn((c["comps"], c["dim"]), generator=g, device=dev)
    sig = torch.rand((c["comps"], c["dim"]), generator=g, device=dev) * 0.45 + 0.05 if c["aniso"] else None
    g2 = torch.Generator(device=dev)
    g2.manual_seed(seed)
    x = torch.empty((n, c["dim"]), dtype=torch.float32, device=dev)
    for r0 in range(0, n, 1 << 18):
        r1 = min(n, r0 + (1 << 18))
        comp = torch.randint(0, c["comps"], (r1 - r0,), generator=g2, device=dev)
        noise = torch.randn((r1 - r0, c["dim"]), generator=g2, device=dev)
        y = centres[comp] + (sig[comp] * noise if c["aniso"] else c["sigma"] * noise)
        if c["unit"]:
            y /= torch.linalg.vector_norm(y, dim=1, keepdim=True)
        x[r0:r1] = y
    torch.cuda.synchronize(dev)
    return x


def make_mixture_range(torch, dev, c, seed, lo, hi, centre_seed=0):
    """Rows [lo, hi) of the config's mixture drawn chunk by chunk: chunk i
    (rows i * 2^18 ...) from its own generator (seed, i), so any row range
    is drawn alone and equals the same rows of the whole set."""
    g = torch.Generator(device=dev)
    g.manual_seed(centre_seed)
    centres = torch.randn((c["comps"], c["dim"]), generator=g, device=dev)
    sig = torch.rand((c["comps"], c["dim"]), generator=g, device=dev) * 0.45 + 0.05
    x = torch.empty((hi - lo, c["dim"]), dtype=torch.float32, device=dev)
    step = 1 << 18
    for ci in range(lo // step, (hi + step - 1) // step):
        r0, r1 = ci * step, min(c["rows"], (ci + 1) * step)
        g2 = torch.Generator(device=dev)
        g2.manual_seed(seed * 1_000_003 + ci)
        comp = torch.randint(0, c["comps"], (r1 - r0,), generator=g2, device=dev)
        noise = torch.randn((r1 - r0, c["dim"]), generator=g2, device=dev)
        y = centres[comp] + sig[comp] * noise
        y /= torch.linalg.vector_norm(y, dim=1, keepdim=True)
        a, b = max(r0, lo), min(r1, hi)
        if a < b:
            x[a - lo:b - lo] = y[a - r0:b - r0]
        del comp, noise, y
    torch.cuda.synchronize(dev)
    return x


def build_recall(torch, x, res, queries, ls=(50, 100, 200)):
    from shear_b200 import graph as G
    gt, _ = G.exact_knn(x, queries, 10)
    gt = gt.cpu().numpy()
    xh = x.cpu().numpy()
    qh = queries.cpu().numpy()
    out = {}
    for l in ls:
        ids, comps = G.search(xh, res.offsets, res.neighbors, res.entry_point, qh, 10, l)
        out[str(l)] = G.recall_at(ids, gt, 10)
    return out


def run_build(a):
    import torch

    from shear_b200 import ops
    from shear_b200.index import BuildParams, build_index
    from shear_b200.sharded_build import build_index_sharded, row_range

    world, rank, local = dist_env()
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    ctx = ops.context(dev.index)
    c = build_cfg(a)
    p = BuildParams(c_max=c["c_max"], reducer_threads=max(1, (os.cpu_count() or 1) // world))
    # one dataset of the config's size, split over the ranks (strong scaling): every rank draws the same
    # mixture (outside the timed region) and keeps its row range
    n = c["rows"]
    lo, hi, _ = row_range(n, world, rank)
    if c.get("chunked"):  # each rank draws its own range only; the whole set exists on one GPU alone
        xs = make_mixture_range(torch, dev, c, 1234, lo, hi)
        x = xs if world == 1 else None
    else:
        x = make_mixture(torch, dev, c["rows"], c, seed=1234)
        xs = x[lo:hi].contiguous()

    def build(inp):
        if world == 1:
            return build_index(inp, p, device=dev.index, ctx=ctx)
        return build_index_sharded(inp, n, p, device=dev.index, ctx=ctx)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    for _ in range(max(a.warmup, 3)):
        res = build(xs)
    torch.cuda.synchronize(dev)
    barrier()
    stream = torch.cuda.current_stream(dev)
    times, leaf_ms, step_phases = [], [], []
    with ClockSampler(dev.index) as clk:
        for _ in range(a.steps):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier()
            torch.cuda.synchronize(dev)
            s.record(stream)
            res = build(xs)
            e.record(stream)
            torch.cuda.synchronize(dev)
            times.append(s.elapsed_time(e) / 1e3)
            leaf_ms.append(res.timings["leaf_kernel_ms"])
            step_phases.append({k: round(v, 4) for k, v in res.timings.items() if k.startswith("partition")})
    barrier()
    if world > 1:  # each step's time is its slowest rank's
        import torch.distributed as dist
        tt = torch.tensor(times, device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        times = tt.cpu().tolist()
    per_step = float(np.mean(times))
    value = n / per_step

    # ---- e2e: host rows (pinned) -> graph on the host, through the public build call
    e2e = None
    if not a.no_e2e and a.e2e_steps > 0:
        xh = xs.cpu().pin_memory().numpy()
        build(xh)
        e2e_t, r2 = [], None
        for _ in range(a.e2e_steps):
            # the previous result's graph goes back to the pinned cache first (holding it
            # would make this build allocate new pinned blocks for its graph)
            r2 = None
            barrier()
            t0 = time.perf_counter()
            r2 = build(xh)
            e2e_t.append(time.perf_counter() - t0)
        if world > 1:  # each step's time is its slowest rank's
            import torch.distributed as dist
            tt = torch.tensor(e2e_t, device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e2e_t = tt.cpu().tolist()
        e2e_s = float(np.mean(e2e_t))
        d2h = torch.tensor([int(r2.stats["d2h_bytes"])], device=dev, dtype=torch.int64)
        if world > 1:
            import torch.distributed as dist
            dist.all_reduce(d2h)
        e2e = {"value": n / e2e_s, "unit": "vectors/s", "h2d_bytes_per_step": int(n * c["dim"] * 4),
               "d2h_bytes_per_step": int(d2h.item()), "ms_per_step": e2e_s * 1e3,
               "phases_s": {k_: round(v_, 4) for k_, v_ in r2.timings.items()},
               "timing": ("wall clock around build_index(host numpy rows): upload from pinned memory, GPU "
                          "stages, device HashPrune reservoirs, pinned D2H of the graph" if world == 1 else
                          "wall clock, slowest rank per step, around build_index_sharded(host numpy row range): "
                          "each rank uploads its rows from pinned memory; all-gather of D0 rows, partial "
                          "reservoirs exchanged by owner range, graph gathered on rank 0 and copied to its "
                          "pinned host memory")}
        del xh

    if rank != 0:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return 0

    recall = None
    if not a.no_recall and x is not None:
        q = make_mixture(torch, dev, c["queries"], c, seed=99991)
        recall = {"at": 10, "queries": c["queries"], "by_L": build_recall(torch, x, res, q),
                  "ground_truth": "exact f32 L2 top-10 on the GPU", "search": "greedy beam search restating "
                  "apps/search_shear_index (tessa_graph_search, host threads)"}
        del q

    peaks = measured_peaks()
    int8_peak = int8_peak_tops(torch, dev)
    leaf_s = float(np.mean(leaf_ms)) / 1e3
    achieved = res.stats["leaf_ops"] / leaf_s / 1e12
    peak, src = (int8_peak, "measured in-run: cuBLAS int8 burst (torch._int_mm 8192^3)") if int8_peak else \
        (NOMINAL_INT8_TOPS, "nominal B200 dense int8 4.5 POPS (no measured int8 peak)")
    traffic = int(LEAF_BUILD_BYTES_PER_OP * res.stats["leaf_ops"] +
                  LEAF_BUILD_FINISH_BYTES_PER_ROW * res.stats["leaf_rows"])
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOP/s", "frac": achieved / peak,
                "traffic": traffic, "peak_source": src,
                "traffic_source": "ncu DRAM bytes of the leaf kernels on the 200k-row build of the same family, "
                                  "scaled by leaf int8 ops (main kernel) and leaf rows (finishing kernel)",
                "kernel": "leaf stage of the build:tessa::leaf::split::leaf_topk_split_kernel<2> + finish "
                          "(CUDA events around tessa_leaf_topk_sq8)",
                "algorithmic_ops_per_launch": res.stats["leaf_ops"], "leaf_kernel_ms": leaf_s * 1e3,
                "hbm_bytes_algorithmic": int(res.stats["leaf_rows"] * ((res.stats["dim"] + 15) // 16 * 16 + 16) +
                                             res.stats["leaf_rows"] * res.stats["leaf_k"] * 8),
                "hbm_peak_gbs": peaks.get("hbm_gbs")}

    cpu = None
    parity = None
    if not a.no_cpu_baseline and world == 1 and x is not None:
        from oracle.cpu_build import build_index_cpu
        O = host_oracle()
        m = a.cpu_rows or min(n, 30000 if c["dim"] > 256 else 100000)
        xs = x[:m].contiguous()
        xsh = xs.cpu().numpy()
        g = build_index(xs, p, device=dev.index, ctx=ctx)
        t0 = time.perf_counter()
        offs, nb, entry, tm, _ = build_index_cpu(xsh, p, g.stats["root_leaders"], threads=os.cpu_count() or 1)
        dt = time.perf_counter() - t0
        cpu = {"value": m / dt, "unit": "vectors/s", "cores": O.num_threads(), "kind": "port",
               "sample": f"the CPU restatement of the same build (oracle/cpu_build.py: OpenMP C stages + the host "
                         f"reducer) on the first {m} of the {n} rows, {dt:.1f} s"}
        same = bool(np.array_equal(g.offsets, offs) and np.array_equal(g.neighbors, nb) and g.entry_point == entry)
        parity = {"rows": m, "graphs_identical": same}
        if not a.no_recall:
            q = make_mixture(torch, dev, min(1000, c["queries"]), c, seed=99991)
            from shear_b200.index import BuildResult
            parity["recall10_L100_gpu"] = build_recall(torch, xs, g, q, ls=(100,))["100"]
            parity["recall10_L100_cpu_restatement"] = build_recall(
                torch, xs, BuildResult(offs, nb, entry), q, ls=(100,))["100"]

    line = {
        "metric": BUILD_METRIC, "value": value, "unit": "vectors/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8",
        "data": f"synthetic stand-in for BASELINE config {a.config} (seeded Gaussian mixture on the device, seed "
                f"1234); random root leaders and sketch hyperplanes from seeded generators",
        "config": dict(build_desc(a, c), parallelism=(
            "one GPU" if world == 1 else f"one build over {world} GPUs: row ranges, D0 all-gather, child runs "
            f"by LPT, partial reservoirs all-to-all by owner range, graph gathered on rank 0 (NCCL)")),
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "recall": recall, "recall_parity": parity,
        "gpu_launches": res.stats["kernel_launches"] * a.steps,
        "clocks": clk.summary(),
        "phases_s": {k: round(v, 4) for k, v in res.timings.items()},
        "step_ms": [round(t * 1e3, 2) for t in times],
        "step_partition_s": step_phases,
        "build_stats": {k: v for k, v in res.stats.items() if k not in ("root_plan",)},
        "degree": res.degree_stats(),
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_build_reference(a):
    """The reference arm for the build: the CPU restatement of the same build
    (oracle/cpu_build.py) on all host cores, rank 0 only, on a bounded sample
    of the config's rows per step."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    from oracle.cpu_build import build_index_cpu
    from shear_b200.index import BuildParams, root_leader_count

    O = host_oracle()
    c = build_cfg(a)
    m = a.cpu_rows or min(c["rows"], 30000 if c["dim"] > 256 else 100000)
    x = make_mixture_np(m, c, seed=1234)
    p = BuildParams(c_max=c["c_max"])
    k0, _ = root_leader_count(m, c["dim"], p, 183_000_000_000)
    times = []
    for i in range(a.warmup + a.steps):
        t0 = time.perf_counter()
        build_index_cpu(x, p, k0, threads=os.cpu_count() or 1)
        if i >= a.warmup:
            times.append(time.perf_counter() - t0)
    mean = float(np.mean(times))
    value = m / mean
    line = {
        "impl": "reference", "metric": BUILD_METRIC, "value": value, "unit": "vectors/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": mean * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": f"synthetic stand-in for BASELINE config {a.config} (seeded Gaussian mixture, host)",
        "config": build_desc(a, c),
        "cpu_baseline": {"value": value, "unit": "vectors/s", "cores": O.num_threads(), "kind": "port",
                         "sample": f"{m} of the config's {c['rows']} rows per step"},
        "e2e": {"value": value, "unit": "vectors/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference is Rust + NVRTC (no cargo in this image); the timed arm is its build restated on "
                "the CPU (oracle/, OpenMP) with the host HashPrune reducer, all host cores",
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    a = parse_args()
    if a.workload == "build":
        return run_build_reference(a) if a.impl == "reference" else run_build(a)
    if a.workload == "assign":
        return run_assign_reference(a) if a.impl == "reference" else run_assign(a)
    if a.workload == "edges":
        return run_edges_reference(a) if a.impl == "reference" else run_edges(a)
    if a.workload == "d0":
        return run_d0_reference(a) if a.impl == "reference" else run_d0(a)
    if a.impl == "reference":
        return run_reference(a)
    return run_ours(a)


if __name__ == "__main__":
    sys.exit(main())
