#!/usr/bin/env python
"""Benchmark: batched Householder QR (geqrf + Q formation) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

One step = one fused QR (``qr_b200.qr``: (H, tau) in torch.geqrf form plus the
explicit Q, i.e. 8/3 n^3 flops per matrix) of one batch of the configuration.
Default configuration: ``b32_n2048`` (32 i.i.d. N(0,1) 2048x2048 fp32 matrices,
the largest configuration; the tensor-core blocked path).  The other four
configurations are timed after it (fewer steps) and reported under
``extra_configs`` in the same JSON line.

Multi-GPU (torchrun, one process per GPU): the configuration's batch is split
into contiguous slices, rank r factoring matrices [r*B/N, (r+1)*B/N) of the same
seeded batch (strong scaling; uneven tails go to the later ranks).  There is no
collective on the data path, only a barrier and a max-reduction of the timings.
``value`` = B / max-over-ranks time.

Timing: per step, the L2 is flushed (256 MiB write, untimed, as the reference
harness's clear_l2_cache does) and the step is bracketed by CUDA events on the
launching stream; ms_per_step is the mean of the K step durations, max over ranks.
A second pass of the same K steps runs with the library's per-launch CUDA-event
timing on (``qrb_kernel_timing``); its per-kernel totals give the dominant kernel
and its roofline.

``--impl reference``: the reference arm -- CPU ``torch.linalg.qr`` (the
comparator the reference names) on all host cores, rank 0 only, on the full batch
of the configuration every step.  It imports nothing that loads the repo's
libraries.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "linalg-gpu-comp_b200"
for _p in (str(ROOT), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = json.loads((ROOT / "BASELINE.json").read_text())["metric"] if (ROOT / "BASELINE.json").exists() \
    else "batched QR matrices/s"
DEFAULT_CONFIG = "b32_n2048"


def flops_per_matrix(n: int) -> float:
    return 8.0 / 3.0 * n ** 3


def bytes_per_matrix(n: int) -> int:
    """Algorithmic HBM bytes of the fused QR: read A, write H, tau and Q."""
    return 12 * n * n + 4 * n


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def shard(batch: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous slice [lo, hi) of a batch of ``batch`` matrices owned by ``rank`` of
    ``world`` ranks; sizes differ by at most one, the larger slices last."""
    return rank * batch // world, (rank + 1) * batch // world


def load_traffic(config: str) -> dict:
    """Per-kernel DRAM traffic of a configuration from the committed ncu summaries: either
    bytes per launch, or DRAM bytes per algorithmic byte measured on a smaller case of the
    same kernel (scaled by the run's algorithmic bytes per launch)."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        return json.loads(p.read_text()).get(config) or {}
    return {}


def traffic_for(traffic: dict, kernel: str, bytes_per_launch: float):
    e = (traffic or {}).get(kernel)
    if not e:
        return None
    if "dram_bytes_per_launch" in e:
        return e["dram_bytes_per_launch"]
    return e["dram_per_algorithmic"] * bytes_per_launch


# ---------------------------------------------------------------------------
# clocks (read-only NVML sampling during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        0x0000000000000004: "sw_power_cap", 0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown", 0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000080: "hw_power_brake_slowdown", 0x0000000000000002: "applications_clocks_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.02):
        self.samples, self.reasons, self.ok = [], set(), False
        self.max_mhz = None
        self._stop = threading.Event()
        self._period = period_s
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self._period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_init(gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        # NCCL may print its version banner on the C-level stdout when the communicator
        # comes up; keep stdout for the one JSON line by sending that to stderr.
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
            dist.barrier(device_ids=[local])
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
        return dist, rank, world, local
    return None, 0, 1, 0


def reduce_max(dist, x: float, device) -> float:
    if dist is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist, device):
    if dist is not None:
        dist.barrier(device_ids=[device.index])
    torch.cuda.synchronize(device)


# ---------------------------------------------------------------------------
# CPU legs
# ---------------------------------------------------------------------------
def cpu_sample(config: str, seed: int, target_s: float):
    """Bounded sample of the workload on the host: (matrices, A_cpu)."""
    from qr_b200.inputs import CONFIGS, config_input
    batch, n, _ = CONFIGS[config]
    from oracle import cpu_ref
    probe = config_input(config, seed=seed, device="cpu", batch=min(batch, 8))
    cpu_ref.cpu_qr(probe)
    t0 = time.perf_counter()
    cpu_ref.cpu_qr(probe)
    per = max((time.perf_counter() - t0) / probe.shape[0], 1e-7)
    m = int(max(1, min(batch, target_s / per)))
    return m, config_input(config, seed=seed, device="cpu", batch=m)


def cpu_baseline(config: str, seed: int, budget_s: float = 12.0) -> dict:
    from oracle import cpu_ref
    threads = cpu_ref.set_threads()
    m, A = cpu_sample(config, seed, budget_s / 6)
    sec = cpu_ref.time_cpu_qr(A, min_seconds=budget_s * 0.8, max_iters=10_000)
    return {"value": m / sec, "unit": "matrices/s", "cores": threads, "kind": "reference",
            "sample": f"torch.linalg.qr (LAPACK sgeqrf+sorgqr, fp32) on {m} of the {config} matrices, "
                      f"repeated for ~{budget_s * 0.8:.0f} s on {threads} host threads"}


def run_reference(args) -> dict | None:
    """CPU torch.linalg.qr on the full batch of the configuration, every step.

    Rank 0 only; the other torchrun ranks exit without work.  No process group is
    needed (nothing is exchanged), CUDA is never touched, and only ``qr_b200.inputs``
    (plain torch generators) is imported from the package -- no repo library loads."""
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    from oracle import cpu_ref
    from qr_b200.inputs import CONFIGS, config_input
    batch, n, _ = CONFIGS[args.config]
    threads = cpu_ref.set_threads()
    A = config_input(args.config, seed=args.seed, device="cpu")
    warm = max(1, min(args.warmup, 3))
    for _ in range(warm):
        cpu_ref.cpu_qr(A)
    t = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu_ref.cpu_qr(A)
        t.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.mean(t)
    value = batch / (ms / 1e3)
    sample = (f"torch.linalg.qr (LAPACK sgeqrf+sorgqr, fp32) on the full batch of {batch} {args.config} "
              f"matrices per step, {threads} host threads, {warm} untimed warm-up call(s)")
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "matrices/s",
        "gflops": value * flops_per_matrix(n) / 1e9, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": warm, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic i.i.d. N(0,1), seeded (CPU generator)",
        "config": {"workload": args.config, "batch": batch, "n": n, "sample_matrices": batch},
        "cpu_baseline": {"value": value, "unit": "matrices/s", "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": value, "unit": "matrices/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def time_steps(step, steps: int, stream, flush, dist, dev, clocks=None) -> float:
    """Mean CUDA-event duration of ``steps`` calls of ``step`` (L2 flushed before each,
    outside the events), max over ranks."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    barrier(dist, dev)
    for i in range(steps):
        flush.fill_(42)
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    barrier(dist, dev)
    times = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    return reduce_max(dist, statistics.mean(times), dev)


def kernel_profile(step, steps: int, stream, flush, dist, dev) -> dict:
    """Per-kernel CUDA-event totals over ``steps`` more steps, with the library's launch
    timing on (events on each kernel's launching stream)."""
    import qr_b200
    from qr_b200._lib import kernel_timing_report
    lib = qr_b200.lib()
    kernel_timing_report()            # drop anything logged earlier
    barrier(dist, dev)
    lib.qrb_kernel_timing(1)
    try:
        for _ in range(steps):
            flush.fill_(7)
            step()
        torch.cuda.synchronize(dev)
    finally:
        lib.qrb_kernel_timing(0)
    return kernel_timing_report()


def roofline_from_profile(prof: dict, steps: int, step_ms: float, n: int, batch: int, peaks: dict,
                          traffic) -> dict | None:
    if not prof:
        return None
    total = sum(v["ms"] for v in prof.values())
    name, d = max(prof.items(), key=lambda kv: kv[1]["ms"])
    per_launch_ms = d["ms"] / d["launches"]
    bytes_per_launch = d["bytes"] / d["launches"]
    gbs = d["bytes"] / (d["ms"] / 1e3) / 1e9
    tf32_peak = peaks["bf16_tflops_sustained"] / 2.0
    # 3xTF32: the tensor-core kernels issue three tf32 products per useful multiply-add.
    tensor_kernel = name in ("wpart_kernel", "update_kernel", "ygemm_kernel", "wupdate_kernel", "w2tc_kernel")
    k_tflops = (3.0 if tensor_kernel else 1.0) * d["flops"] / (d["ms"] / 1e3) / 1e12
    step_tflops = batch * flops_per_matrix(n) / (step_ms / 1e3) / 1e12
    return {
        "bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
        "frac": gbs / peaks["hbm_gbs"], "traffic": traffic_for(traffic, name, bytes_per_launch), "kernel": name,
        "launches_per_step": d["launches"] / steps, "ms_per_launch": per_launch_ms,
        "algorithmic_bytes_per_launch": bytes_per_launch,
        "share_of_kernel_time": d["ms"] / total if total > 0 else None,
        "peak_source": f"{peaks['source']} hbm_gbs (MEASURED_PEAKS.json), 'of measured'",
        "tensor": {"kernel_tflops_issued": k_tflops, "step_tflops_useful": step_tflops,
                   "peak_tf32_derived": tf32_peak,
                   "kernel_frac": k_tflops / tf32_peak if tensor_kernel else None,
                   "step_frac": step_tflops / tf32_peak,
                   "note": "tf32 peak derived as bf16_tflops_sustained / 2 (no tf32 GEMM is measured); "
                           "kernel figure counts the three tf32 products of 3xTF32"},
        "kernels": {k: {"launches_per_step": v["launches"] / steps, "ms_per_step": v["ms"] / steps,
                        "share": v["ms"] / total if total > 0 else None,
                        "gbs": v["bytes"] / (v["ms"] / 1e3) / 1e9 if v["ms"] > 0 else None}
                    for k, v in sorted(prof.items(), key=lambda kv: -kv[1]["ms"])},
    }


def bench_config(config: str, args, dist, rank: int, world: int, dev, steps: int, warmup: int,
                 flush, clocks=None) -> dict:
    """Time one configuration with this rank's slice of its batch; returns the numbers."""
    import qr_b200
    from qr_b200.inputs import CONFIGS, config_input
    batch, n, _ = CONFIGS[config]
    if config == args.config and args.batch is not None:
        batch = args.batch
    lo, hi = shard(batch, rank, world)
    full = config_input(config, seed=args.seed, device=dev, batch=batch)
    A = full[lo:hi].contiguous()
    del full
    H = torch.empty_like(A)
    tau = torch.empty(A.shape[0], n, device=dev)
    Q = torch.empty_like(A)
    stream = torch.cuda.current_stream(dev)

    geqrf_only = args.op == "geqrf" and config == args.config

    def step():
        if A.shape[0] > 0:
            if geqrf_only:
                qr_b200.geqrf(A, out=(H, tau))
            else:
                qr_b200.qr(A, out=(H, tau, Q))

    for _ in range(max(warmup, 3)):
        step()
    if clocks is not None:
        with clocks:
            ms = time_steps(step, steps, stream, flush, dist, dev)
    else:
        ms = time_steps(step, steps, stream, flush, dist, dev)
    prof = kernel_profile(step, steps, stream, flush, dist, dev)
    return {"batch": batch, "n": n, "lo": lo, "hi": hi, "ms": ms, "prof": prof, "A": A, "H": H, "tau": tau,
            "Q": Q, "step": step}


def run_ours(args) -> dict | None:
    import qr_b200

    dist, rank, world, local = dist_init(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    flush = torch.empty(256 * 1024 * 1024 // 8, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)
    peaks = load_peaks()

    clocks = ClockSampler(dev.index)
    main = bench_config(args.config, args, dist, rank, world, dev, args.steps, args.warmup, flush, clocks)
    batch, n, ms = main["batch"], main["n"], main["ms"]
    A, H, tau, Q = main["A"], main["H"], main["tau"], main["Q"]
    roof = roofline_from_profile(main["prof"], args.steps, ms, n, main["hi"] - main["lo"], peaks,
                                 load_traffic(args.config))
    launches = sum(v["launches"] for v in main["prof"].values())

    # end to end through the public API: pinned host A -> device, QR, H/tau/Q -> pinned host
    e2e = None
    if not args.no_e2e:
        A_h = A.cpu().pin_memory()
        H_h = torch.empty(H.shape, dtype=H.dtype).pin_memory()
        t_h = torch.empty(tau.shape, dtype=tau.dtype).pin_memory()
        Q_h = torch.empty(Q.shape, dtype=Q.dtype).pin_memory()

        def e2e_step():
            # one library call: chunked host->device copy, QR, device->host copies
            if A_h.shape[0] > 0:
                qr_b200.qr_host(A_h, out=(H_h, t_h, Q_h), device=dev)

        for _ in range(2):
            e2e_step()
        barrier(dist, dev)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k_e2e = max(3, min(args.steps, 20))
        ev0.record(stream)
        for _ in range(k_e2e):
            e2e_step()
        ev1.record(stream)
        barrier(dist, dev)
        ms_e2e = reduce_max(dist, ev0.elapsed_time(ev1) / k_e2e, dev)
        h2d = A.numel() * 4
        d2h = (H.numel() + tau.numel() + Q.numel()) * 4
        e2e = {"value": batch / (ms_e2e / 1e3), "unit": "matrices/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e,
               "steps": k_e2e, "api": "qr_b200.qr_host (C ABI qrb_qr_f32_host, pinned host buffers)"}
        del A_h, H_h, t_h, Q_h
    del main, A, H, tau, Q

    extras = {}
    if not args.no_extra:
        from qr_b200.inputs import CONFIGS
        for name in CONFIGS:
            if name == args.config:
                continue
            r = bench_config(name, args, dist, rank, world, dev, max(3, min(args.steps, 10)), 3, flush)
            extras[name] = {
                "ms_per_step": r["ms"], "matrices_per_s": r["batch"] / (r["ms"] / 1e3),
                "gflops": r["batch"] * flops_per_matrix(r["n"]) / (r["ms"] / 1e3) / 1e9,
                "steps": max(3, min(args.steps, 10)),
                "roofline": roofline_from_profile(r["prof"], max(3, min(args.steps, 10)), r["ms"], r["n"],
                                                  r["hi"] - r["lo"], peaks, load_traffic(name)),
            }
            del r

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(args.config, args.seed)

    if rank != 0:
        return None
    value = batch / (ms / 1e3)
    return {
        "metric": METRIC, "value": value, "unit": "matrices/s",
        "gflops": value * flops_per_matrix(n) / 1e9, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic i.i.d. N(0,1), seeded; one batch split across ranks",
        "config": {"workload": args.config, "global_batch": batch, "n": n,
                   "batch_per_gpu": [shard(batch, r, world)[1] - shard(batch, r, world)[0] for r in range(world)],
                   "parallelism": f"batch split over {world} GPU(s), no collective",
                   "l2": "flushed between steps (256 MiB write)", "op": "geqrf + orgqr (qrb_qr_f32)"},
        "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": int(round(launches)),
        "gpu_launches_note": "kernels the library launched in the K timed-pass steps, counted by its launch log",
        "clocks": clocks.summary(),
        "extra_configs": extras,
    }


# ---------------------------------------------------------------------------
# the reference task's own benchmark shapes (drop-in path: custom_kernel -> (H, tau))
# ---------------------------------------------------------------------------
# reference_repo/task.yml:93-100, with the reference's best published B200 time per shape
# (ms per custom_kernel call, as its eval.py measures it).
GPUMODE_SHAPES = [
    (20, 32, 1, 43214, 0.0269, "v19, bench_history.json:109"),
    (40, 176, 1, 423011, 0.634, "v19, bench_history.json:110"),
    (40, 352, 1, 123456, 1.634, "v19, bench_history.json:111"),
    (640, 512, 2, 1029, 12.15, "v24 = submission.py, RESUME.md:183"),
    (60, 1024, 2, 75342, 10.72, "v24 = submission.py, RESUME.md:183"),
    (8, 2048, 1, 224466, 73.5, "v24 = submission.py, RESUME.md:183"),
    (2, 4096, 1, 32412, 50.55, "v24 = submission.py, RESUME.md:183"),
]


def run_gpumode(args) -> None:
    """Time ``custom_kernel`` the way the reference harness does (eval.py:178-224).

    Per shape: up to 50 inputs of the shape (256 MiB of input in total, seeds
    seed + 42·i, eval.py:158-175), each output checked with the device restatement
    of the reference's gate; then repeated timed passes over all inputs, each after
    an L2 flush, CUDA events around the pass, duration / number of inputs; mean over
    the passes.  One JSON line per shape plus a geometric-mean summary line.
    """
    import math
    from qr_b200 import custom_kernel
    from qr_b200.checker import check_implementation
    from qr_b200.inputs import task_input
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    flush = torch.empty(256 * 1024 * 1024 // 8, dtype=torch.int64, device=dev)
    logs = []
    for batch, n, cond, seed, ref_ms, ref_src in GPUMODE_SHAPES:
        count = max(1, min(50, (256 * 1024 * 1024) // (batch * n * n * 4)))
        data = [task_input(batch, n, cond, seed + 42 * (i + 1), "dense", device=dev) for i in range(count)]
        outs = [custom_kernel(d) for d in data]
        checks = [check_implementation(d, o) for d, o in zip(data, outs)]
        ok = all(c[0] for c in checks)
        del outs
        durations = []
        t_start = time.perf_counter()
        for i in range(max(args.steps, 3)):
            torch.cuda.synchronize()
            flush.fill_(i)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            outs = [custom_kernel(d) for d in data]
            e1.record()
            torch.cuda.synchronize()
            durations.append(e0.elapsed_time(e1) / len(data))
            del outs
            if i >= 2 and time.perf_counter() - t_start > 10.0:
                break
        ms = statistics.mean(durations)
        line = {"suite": "gpumode", "shape": f"b{batch}_n{n}_c{cond}", "ms": ms, "runs": len(durations),
                "inputs": count, "check": "pass" if ok else f"FAIL: {[c[1] for c in checks if not c[0]][:1]}",
                "reference_ms": ref_ms, "reference": ref_src, "speedup_vs_reference": ref_ms / ms,
                "example_check": checks[0][1]}
        logs.append((ms, ref_ms))
        print(json.dumps(line), flush=True)
        del data
    geo = math.exp(sum(math.log(m) for m, _ in logs) / len(logs))
    geo_ref = math.exp(sum(math.log(r) for _, r in logs) / len(logs))
    print(json.dumps({"suite": "gpumode", "summary": "geometric mean over the task's benchmark shapes "
                      "(the leaderboard's ranking_by: geom)", "ms": geo, "reference_ms": geo_ref,
                      "speedup_vs_reference": geo_ref / geo}), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", default=DEFAULT_CONFIG)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the other configurations")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the configuration's batch (profiling captures on a small case)")
    ap.add_argument("--op", choices=["qr", "geqrf"], default="qr",
                    help="geqrf: time the factorisation alone (profiling); the metric is defined on qr")
    ap.add_argument("--suite", choices=["gpumode"], default=None,
                    help="gpumode: custom_kernel on the reference task's benchmark shapes (one line each)")
    args = ap.parse_args(argv)
    if args.suite == "gpumode":
        run_gpumode(args)
        return
    out = run_reference(args) if args.impl == "reference" else run_ours(args)
    if out is not None:
        print(json.dumps(out), flush=True)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
