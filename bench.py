#!/usr/bin/env python3
"""Benchmark of the pn_fir_tau attention operator (forward + backward).

Headline (BASELINE metric): flash_pn_fir_tau_attention fwd+bwd TFLOP/s at
N=4096 (config 3: B=8, H=8, N=4096, d=64, bf16, half of the 64-row query
blocks scaled by 0.05), algorithmic FLOPs 7*B*H*N^2*d per step (causal = half
of dense QK^T + PV forward and the five backward products; skipped silent
tiles still count). Alongside: the 6-layer pn_fir_tau LM training step in
tokens/s (config 4), the end-to-end number through the public API with host
buffers, the dominant kernel's roofline, a bounded CPU-oracle baseline and
the SM clocks seen during the timed region.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (one rank per GPU)

Also: config 3's tau sweep {-0.5, 0, +0.5} with the silent-tile skips the
kernels took, and config 5 (B8 H16 N16384 d128) with its 128 heads sharded
over the ranks.

Multi-GPU: every rank runs its own config-3-sized shard of batch x heads
(weak scaling, no collective on the operator's data path); the shared tau
gradient is summed across ranks with one fp64 all-reduce per backward on a side
stream (TauGradReducer: no step waits for the other ranks; the sum is collected
at the end of the timed region). The LM is data parallel: its headline step is
captured in one CUDA graph per rank with the gradient average (one NCCL
all-reduce) inside it; the eager comparison uses DDP.
``--impl reference`` times the reference's eager algorithm on the host cores
on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "pn_fir_tau attn fwd+bwd TFLOP/s (% tensor peak) at N=4096; 6-layer LM tokens/s"
WORKLOADS = {
    "c3": dict(B=8, H=8, N=4096, D=64, quiet_frac=0.5,
               desc="flash_pn_fir_tau_attention fwd+bwd, B8 H8 N4096 d64 bf16, 50% of 64-row q blocks x0.05"),
    "c2": dict(B=16, H=4, N=512, D=64, quiet_frac=0.0, desc="flash_pn_fir_tau_attention fwd+bwd, B16 H4 N512 d64 bf16"),
    "c5": dict(B=8, H=16, N=16384, D=128, quiet_frac=0.0,
               desc="flash_pn_fir_tau_attention fwd+bwd, B8 H16 N16384 d128 bf16"),
}
L2_BYTES = 126 * 2**20
FALLBACK_PEAK_TFLOPS = 1590.0
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c3")
    ap.add_argument("--tau", type=float, default=0.0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--lm-steps", type=int, default=10)
    ap.add_argument("--no-lm", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-fir", action="store_true")
    ap.add_argument("--no-lm-kernels", action="store_true", help="skip timing the LM step's kernels alone")
    ap.add_argument("--lm-kernels-only", action="store_true",
                    help="only the LM step's kernels, one call each then timed (the profiling command)")
    ap.add_argument("--lm-kernel-rows", type=int, default=16352, help="logit rows of the cross-entropy timing")
    ap.add_argument("--no-sweep", action="store_true", help="skip the config-3 tau sweep")
    ap.add_argument("--no-c5", action="store_true", help="skip the config-5 measurement")
    ap.add_argument("--no-triton", action="store_true",
                    help="reference arm: skip timing the reference's Triton kernels on the GPU")
    ap.add_argument("--sweep-steps", type=int, default=10)
    ap.add_argument("--c5-steps", type=int, default=4)
    ap.add_argument("--e2e-chunks", type=int, default=4,
                    help="pipeline chunks of the e2e step (whole heads each; 1 = one call per step)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--generic", action="store_true", help="force the generic SIMT kernels")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.active = self.world > 1
        self.tau_group = None  # NCCL group of the per-backward tau all-reduce (init)

    def init(self, backend: str):
        if self.active:
            import torch.distributed as dist

            opts = None
            if backend == "nccl":
                # NCCL's kernels on a high-priority stream: the per-backward tau
                # all-reduce then takes the next free SM slot instead of queueing
                # behind the attention kernels that fill every SM
                opts = dist.ProcessGroupNCCL.Options()
                opts.is_high_priority_stream = True
            dist.init_process_group(backend, timeout=timedelta(seconds=180), pg_options=opts,
                                    device_id=torch.device("cuda", self.local_rank) if backend == "nccl" else None)
            if backend == "nccl":
                # the 8-byte tau all-reduce of every backward on its own communicator
                # whose kernel takes one CTA: it runs beside the next step's
                # attention kernels and takes one SM slot from them, not several
                topts = dist.ProcessGroupNCCL.Options()
                topts.is_high_priority_stream = True
                topts.config.min_ctas = 1
                topts.config.max_ctas = 1
                self.tau_group = dist.new_group(backend="nccl", pg_options=topts, timeout=timedelta(seconds=180))

    def barrier(self):
        if self.active:
            import torch.distributed as dist

            dist.barrier()

    def max(self, x: float, device) -> float:
        if not self.active:
            return x
        import torch.distributed as dist

        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.active:
            import torch.distributed as dist

            dist.destroy_process_group()


# ---------------------------------------------------------------------------
# clocks (NVML reads only; nothing is ever set)
# ---------------------------------------------------------------------------


class ClockSampler:
    """Samples SM clock and clock-event reasons of one GPU every `period` s."""

    REASONS = {
        0x0000000000000008: "hw_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000004: "sw_power_cap",
        0x0000000000000080: "hw_power_brake_slowdown",
        0x0000000000000001: "gpu_idle",
        0x0000000000000002: "applications_clocks_setting",
        0x0000000000000100: "display_clock_setting",
    }

    def __init__(self, device: torch.device, period: float = 0.005):
        self.period = period
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self.error = None
        self._stop = threading.Event()
        self._thread = None
        self.handle = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(h)
                u = u.decode() if isinstance(u, bytes) else u
                if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                    self.handle = h
                    break
            if self.handle is None:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(device.index or 0)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001 - clocks are reported as unavailable
            self.error = f"{type(e).__name__}: {e}"

    def _run(self):
        nv = self.nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                try:
                    reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                except AttributeError:
                    reasons = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle)
                self.samples.append((mhz, int(reasons)))
            except Exception as e:  # noqa: BLE001
                self.error = f"{type(e).__name__}: {e}"
                return
            self._stop.wait(self.period)

    def __enter__(self):
        if self.handle is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "error": self.error or "no samples"}
        mhz = [m for m, _ in self.samples]
        seen = 0
        for _, r in self.samples:
            seen |= r
        reasons = [name for bit, name in self.REASONS.items() if seen & bit and name != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "sm_min_mhz": min(mhz),
                "reasons": reasons, "samples": len(mhz)}


# ---------------------------------------------------------------------------
# peaks and profile figures
# ---------------------------------------------------------------------------


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16_tflops": float(d["bf16_tflops"]), "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", 0)),
                "hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"bf16_tflops": FALLBACK_PEAK_TFLOPS, "bf16_tflops_sustained": 1400.0, "hbm_gbs": FALLBACK_HBM_GBS,
            "source": "fallback"}


def profile_traffic(kernel_key: str) -> float | None:
    """DRAM bytes per launch of `kernel_key` from the committed ncu summary
    (a line `traffic_bytes_per_launch[<key>]: <bytes>` under profiles/)."""
    for p in sorted((ROOT / "profiles").glob("*.md")):
        m = re.search(rf"traffic_bytes_per_launch\[{re.escape(kernel_key)}\]:\s*([0-9.eE+]+)", p.read_text())
        if m:
            return float(m.group(1))
    return None


def profile_traffic_source(kernel_key: str) -> str | None:
    """Which committed ncu summary the traffic figure comes from (it is a recorded
    capture, not measured in this run)."""
    for p in sorted((ROOT / "profiles").glob("*.md")):
        if re.search(rf"traffic_bytes_per_launch\[{re.escape(kernel_key)}\]", p.read_text()):
            return f"recorded ncu capture, profiles/{p.name} (not measured in this run)"
    return None


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------


def make_inputs(w: dict, seed: int, device, dtype=torch.bfloat16):
    """Seeded config inputs: q,k,v,dO ~ N(0,1); with quiet_frac > 0 a seeded
    random fraction of the 64-row query blocks of every (b,h) is scaled by 0.05."""
    B, H, N, D = w["B"], w["H"], w["N"], w["D"]
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(B, H, N, D, generator=g, device=device, dtype=torch.float32)
    if w["quiet_frac"] > 0:
        nb = (N + 63) // 64
        quiet = torch.rand(B, H, nb, generator=g, device=device) < w["quiet_frac"]
        fac = torch.where(quiet, 0.05, 1.0).repeat_interleave(64, dim=-1)[..., :N]
        q = q * fac[..., None]
    k = torch.randn(B, H, N, D, generator=g, device=device)
    v = torch.randn(B, H, N, D, generator=g, device=device)
    do = torch.randn(B, H, N, D, generator=g, device=device)
    return [t.to(dtype) for t in (q, k, v, do)]


def flops_fwd_bwd(w: dict) -> float:
    return 7.0 * w["B"] * w["H"] * w["N"] ** 2 * w["D"]


def reference_package():
    """The reference's own package (src.triton_pnfirtau, src.pnfirtau_attention)
    as staged unchanged into oracle/_ref by oracle/stage_ref.py, or None when it
    was not staged. Used only by the CPU-baseline legs and the reference arm."""
    from oracle import stage_ref

    d = stage_ref.staged()
    if d is None:
        return None
    if str(d) not in sys.path:
        sys.path.insert(0, str(d))
    import src.pnfirtau_attention as A
    import src.triton_pnfirtau as R

    return R, A


def cpu_oracle_sample(w: dict, seconds: float, seed: int, steps: int | None = None):
    """Times the reference's CPU path of the operator on whole (b,h) slices of
    the workload, fp32 fwd+bwd: raw = q k^T, the reference's own
    triton_pn_fir_tau_scores (on CPU tensors it runs its eager fallback,
    power_norm_peak_gate, src/triton_pnfirtau.py:797-811), then @ v. Without the
    staged reference package, the oracle's restatement of the same algorithm.
    Returns (TFLOP/s, threads, slices, seconds, kind, what)."""
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    N, D = w["N"], w["D"]
    scale = 1.0 / math.sqrt(D)
    flops_slice = 7.0 * N * N * D
    g = torch.Generator().manual_seed(seed)
    ref = reference_package()
    if ref is not None:
        R = ref[0]
        kind, what = "reference", "the reference's own triton_pn_fir_tau_scores CPU path (oracle/_ref, unchanged)"

        def attn(q, k, v, tau):
            return torch.matmul(R.triton_pn_fir_tau_scores(torch.matmul(q, k.transpose(-2, -1)), tau, scale), v)
    else:
        from oracle import pnfirtau_oracle as O

        kind, what = "port", "oracle/pnfirtau_oracle.py, the reference's eager algorithm restated"

        def attn(q, k, v, tau):
            return O.pn_fir_tau_attention(q, k, v, tau, scale)

    def one():
        q, k, v, do = (torch.randn(1, 1, N, D, generator=g) for _ in range(4))
        q.requires_grad_(True), k.requires_grad_(True), v.requires_grad_(True)
        tau = torch.tensor(0.0, requires_grad=True)
        out = attn(q, k, v, tau)
        torch.autograd.grad(out, (q, k, v, tau), do)

    one()  # warm-up
    t0 = time.perf_counter()
    n = 0
    while True:
        one()
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (steps is None and el >= seconds):
            break
    return flops_slice * n / el / 1e12, torch.get_num_threads(), n, el, kind, what


def reference_triton_b200(args, w: dict) -> dict:
    """The reference's own Triton Flash kernels (flash_pn_fir_tau_attention,
    src/triton_pnfirtau.py:971-983, unchanged, from oracle/_ref) timed fwd+bwd on
    one B200 on this workload's shape and inputs, at the config-3 tau sweep
    {-0.5, 0, +0.5} (the first value is the headline tau). CUDA events, after
    Triton's JIT warm-up."""
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device in this process"}
    ref = reference_package()
    if ref is None:
        return {"unavailable": "the reference package was not staged into oracle/_ref (oracle/stage_ref.py)"}
    R = ref[0]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    q, k, v, do = make_inputs(w, args.seed, dev)
    leaves = [t.detach().requires_grad_(True) for t in (q, k, v)]
    flops = flops_fwd_bwd(w)
    res = {"impl": "src/triton_pnfirtau.py flash_pn_fir_tau_attention (reference Triton, unchanged)",
           "triton": __import__("triton").__version__}
    taus = [args.tau] + [t for t in (-0.5, 0.0, 0.5) if t != args.tau]
    try:
        for tau0 in taus:
            tau = torch.tensor(tau0, device=dev, requires_grad=True)

            def one(ev=None):
                if ev is not None:
                    ev[0].record()
                out = R.flash_pn_fir_tau_attention(*leaves, tau)
                if ev is not None:
                    ev[1].record()
                torch.autograd.grad(out, (*leaves, tau), do)
                if ev is not None:
                    ev[2].record()

            for _ in range(max(3, args.warmup)):
                one()
            torch.cuda.synchronize()
            steps = max(5, min(args.steps, 20))
            evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for i in range(steps):
                one(evs[i])
            e.record()
            torch.cuda.synchronize()
            ms = s.elapsed_time(e) / steps
            res[f"{tau0:+.1f}"] = {
                "tau": tau0, "ms_per_step": round(ms, 4), "value": round(flops / (ms / 1e3) / 1e12, 2),
                "unit": "TFLOP/s", "steps": steps,
                "fwd_ms": round(statistics.mean(x[0].elapsed_time(x[1]) for x in evs), 4),
                "bwd_ms": round(statistics.mean(x[1].elapsed_time(x[2]) for x in evs), 4)}
    except Exception as exc:  # the reference's kernels may not compile or run on this GPU: report why
        res["unavailable"] = f"{type(exc).__name__}: {exc}"[:400]
    return res


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------


def bench_ours(args, dist_: Dist) -> dict:
    import paper_01_anti_decoy_pnfirtau_b200 as P
    from paper_01_anti_decoy_pnfirtau_b200 import _lib, pnfirtau_ops
    from paper_01_anti_decoy_pnfirtau_b200.sharding import TauGradReducer, sharded_flash_pn_fir_tau_attention

    dev = torch.device("cuda", dist_.local_rank)
    torch.cuda.set_device(dev)
    dist_.init("nccl")
    if args.generic:
        pnfirtau_ops._FORCE_GENERIC = True
    w = WORKLOADS[args.workload]
    q, k, v, do = make_inputs(w, args.seed + 1000 * dist_.rank, dev)
    tau = torch.tensor(args.tau, device=dev, requires_grad=True)
    leaves = [t.requires_grad_(True) for t in (q, k, v)]
    path = P.flash_kernel_path(q, k, v)
    flops = flops_fwd_bwd(w)
    # tau's gradient: this rank's partial is summed over the ranks in fp64 on a side
    # stream (TauGradReducer), so no step waits for the other ranks; the sum is
    # collected once, by the consumer of tau's gradient, at the end of the timed region
    reducer = TauGradReducer(dist_.tau_group)

    def step(evs=None):
        if evs is not None:
            evs[0].record()
        # this rank's B*H shard
        out = sharded_flash_pn_fir_tau_attention(*leaves, tau, reducer=reducer)
        if evs is not None:
            evs[1].record()
        grads = torch.autograd.grad(out, (*leaves, tau), do, allow_unused=True)
        if evs is not None:
            evs[2].record()
        return out, grads

    for _ in range(args.warmup):
        step()
    reducer.result()
    torch.cuda.synchronize()
    P.check_device_status(dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps_done = torch.cuda.Event(enable_timing=True)
    dist_.barrier()
    torch.cuda.synchronize()
    n0 = _lib.launch_count()
    with ClockSampler(dev) as clocks:
        start.record()
        for i in range(args.steps):
            step(evs[i])
        steps_done.record()
        dtau_sum = reducer.result()  # the tau-gradient consumer waits for the last all-reduce
        end.record()
        torch.cuda.synchronize()
    launches = _lib.launch_count() - n0
    dist_.barrier()
    P.check_device_status(dev)
    ms_local = start.elapsed_time(end)
    ms = dist_.max(ms_local, dev)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    collective_wait_ms = steps_done.elapsed_time(end)
    ms_per_step = ms / args.steps
    value = dist_.world * flops * args.steps / (ms / 1e3) / 1e12
    peaks = measured_peaks()

    B, H, N, D = w["B"], w["H"], w["N"], w["D"]
    if bwd_ms >= fwd_ms:
        kname, kflops, kms = "flash_bwd", 5.0 * B * H * N * N * D, bwd_ms
    else:
        kname, kflops, kms = "flash_fwd", 2.0 * B * H * N * N * D, fwd_ms
    achieved = kflops / (kms / 1e3) / 1e12
    traffic = profile_traffic(f"{kname}:{args.workload}")
    traffic_src = profile_traffic_source(f"{kname}:{args.workload}")
    roofline = {
        "bound": "tensor", "kernel": kname, "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"],
        "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4), "traffic": traffic,
        "traffic_source": traffic_src,
        "peak_source": f"{peaks['source']} bf16 burst (sustained {peaks['bf16_tflops_sustained']})",
        "flops_per_launch": kflops, "ms_per_launch": round(kms, 4),
        "note": "flash_bwd time includes its per-row prep, dQ cast and tau-sum launches",
    }
    result = {
        "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": dist_.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{args.workload}: {w['desc']}", "B": B, "H": H, "N": N, "d": D, "tau": args.tau,
                   "kernel_path": path, "per_rank_shard": "each rank runs its own B*H shard of this size",
                   "l2": f"inputs {4 * B * H * N * D * 2 / 2**20:.0f} MiB > 126 MiB L2 (no flush)",
                   "parallelism": f"bh-shard x{dist_.world}" if dist_.world > 1 else "single GPU",
                   "flops_per_step_per_gpu": flops},
        "pct_of_peak": round(100.0 * value / dist_.world / peaks["bf16_tflops"], 2),
        "fwd_ms": round(fwd_ms, 4), "bwd_ms": round(bwd_ms, 4),
        "tau_grad": {"allreduce": "fp64 on a side stream per backward (no per-step rank lock-step)" if dist_.active
                     else "single GPU: no collective", "pushes": reducer.pushes,
                     "exposed_wait_ms": round(collective_wait_ms, 4),
                     "value": float(dtau_sum) if dtau_sum is not None else None},
        "roofline": roofline, "gpu_launches": int(launches), "clocks": clocks.summary(),
    }

    del q, k, v, do, leaves
    if not args.no_sweep and args.workload == "c3":
        result["tau_sweep"] = bench_tau_sweep(args, dist_, w, dev)
    if not args.no_sweep:
        result["deterministic"] = bench_deterministic(args, dist_, w, dev)
    if not args.no_c5 and args.workload == "c3":
        result["c5"] = bench_c5(args, dist_, dev)
    if not args.no_e2e:
        result["e2e"] = bench_e2e(args, dist_, w, dev, flops, P)
    if not args.no_lm:
        result["lm"] = bench_lm(args, dist_, dev)
    if not args.no_fir:
        result["fir"] = bench_fir(args, dist_, dev)
    if not args.no_lm_kernels:
        result["lm_kernels"] = bench_lm_kernels(args, dev)
    if dist_.rank == 0 and dist_.world == 1 and not args.no_cpu:
        tf, cores, n, el, kind, what = cpu_oracle_sample(w, args.cpu_seconds, args.seed)
        result["cpu_baseline"] = {"value": round(tf, 6), "unit": "TFLOP/s", "cores": cores, "kind": kind,
                                  "sample": f"{n} (b,h) slices of [1,1,{N},{D}] fp32 fwd+bwd in {el:.1f} s "
                                            f"({what}, torch CPU eager)"}
    return result


def _time_fwd_bwd(q, k, v, do, tau, steps: int, warmup: int, reducer, attention=None):
    """(total ms, mean fwd ms, mean bwd ms) of `steps` fwd+bwd calls of this rank's
    shard through the public API; tau's gradient through `reducer`."""
    from paper_01_anti_decoy_pnfirtau_b200.sharding import sharded_flash_pn_fir_tau_attention

    leaves = [t.detach().requires_grad_(True) for t in (q, k, v)]

    def one(ev=None):
        if ev is not None:
            ev[0].record()
        out = sharded_flash_pn_fir_tau_attention(*leaves, tau, reducer=reducer, attention=attention)
        if ev is not None:
            ev[1].record()
        torch.autograd.grad(out, (*leaves, tau), do, allow_unused=True)
        if ev is not None:
            ev[2].record()

    for _ in range(warmup):
        one()
    reducer.result()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for i in range(steps):
        one(evs[i])
    reducer.result()
    e.record()
    torch.cuda.synchronize()
    return (s.elapsed_time(e), statistics.mean(x[0].elapsed_time(x[1]) for x in evs),
            statistics.mean(x[1].elapsed_time(x[2]) for x in evs))


def bench_tau_sweep(args, dist_: Dist, w: dict, dev) -> dict:
    """Config 3's tau sweep {-0.5, 0, +0.5} on the same inputs (50% of the 64-row
    query blocks scaled by 0.05): fwd+bwd time and algorithmic TFLOP/s (silent
    tiles still counted), with the skip decisions the kernels took, read back from
    the forward's per-64x64-tile record:
      tiles_silent_frac   causal 64x64 tiles with no u > 0: their elementwise work
                          (u^10, P) is skipped (per 32-row warp) and they are the
                          reference's silent tiles (exp4b definition; the tests
                          check the decisions against the oracle on every head);
      pv_skipped_frac     causal 64x64 tiles whose PV MMA was not issued: the
                          forward's PV unit is 128 query rows x 64 keys, skipped
                          when both of its 64-row halves are silent;
      bwd_qtiles_skipped_frac  64-row query tiles with every row silent, which the
                          backward skips entirely (the reference's `max(peak) > 0`)."""
    from paper_01_anti_decoy_pnfirtau_b200 import TauGradReducer
    from paper_01_anti_decoy_pnfirtau_b200.pnfirtau_ops import flash_pn_fir_tau_forward_stats

    q, k, v, do = make_inputs(w, args.seed + 1000 * dist_.rank, dev)
    B, H, N, D = w["B"], w["H"], w["N"], w["D"]
    flops = flops_fwd_bwd(w)
    nT = (N + 63) // 64
    causal = torch.tril(torch.ones(nT, nT, dtype=torch.bool, device=dev))
    out = {}
    for tau0 in (-0.5, 0.0, 0.5):
        tau = torch.tensor(tau0, device=dev, requires_grad=True)
        ms, fwd, bwd = _time_fwd_bwd(q, k, v, do, tau, args.sweep_steps, 3, TauGradReducer(dist_.tau_group))
        ms = dist_.max(ms, dev)
        _, M, _, _, live = flash_pn_fir_tau_forward_stats(q, k, v, tau.detach())
        ncausal = float(causal.sum()) * B * H
        silent = (~live) & causal
        # PV unit = query tiles (2p, 2p+1): skipped iff both halves are silent
        lp = torch.nn.functional.pad(live, (0, 0, 0, nT % 2))
        pair_live = (lp[:, :, 0::2] | lp[:, :, 1::2]).repeat_interleave(2, dim=2)[:, :, :nT]
        pv_skip = (~pair_live) & causal
        qt_dead = ~(torch.nn.functional.pad(M, (0, nT * 64 - N)).reshape(B, H, nT, 64) > 0).any(-1)
        out[f"{tau0:+.1f}"] = {
            "tau": tau0, "ms_per_step": round(ms / args.sweep_steps, 4),
            "value": round(dist_.world * flops * args.sweep_steps / (ms / 1e3) / 1e12, 2), "unit": "TFLOP/s",
            "fwd_ms": round(fwd, 4), "bwd_ms": round(bwd, 4),
            "tiles_silent_frac": round(float(silent.sum()) / ncausal, 4),
            "pv_skipped_frac": round(float(pv_skip.sum()) / ncausal, 4),
            "bwd_qtiles_skipped_frac": round(float(qt_dead.float().mean()), 4),
            "rows_silent_frac": round(float((M <= 0).float().mean()), 4),
        }
    out["note"] = ("algorithmic FLOPs 7*B*H*N^2*d per step at every tau (skipped tiles counted); this rank's "
                   "shard; fractions over causal 64x64 tiles")
    return out


def bench_deterministic(args, dist_: Dist, w: dict, dev) -> dict:
    """The same fwd+bwd with the ordered (bitwise reproducible) dQ accumulation
    (flash_pn_fir_tau_attention(..., deterministic=True))."""
    import functools

    from paper_01_anti_decoy_pnfirtau_b200 import TauGradReducer
    from paper_01_anti_decoy_pnfirtau_b200.pnfirtau_ops import flash_pn_fir_tau_attention

    q, k, v, do = make_inputs(w, args.seed + 1000 * dist_.rank, dev)
    tau = torch.tensor(args.tau, device=dev, requires_grad=True)
    attn = functools.partial(flash_pn_fir_tau_attention, deterministic=True)
    ms, fwd, bwd = _time_fwd_bwd(q, k, v, do, tau, args.sweep_steps, 3, TauGradReducer(dist_.tau_group), attention=attn)
    ms = dist_.max(ms, dev)
    return {"ms_per_step": round(ms / args.sweep_steps, 4),
            "value": round(dist_.world * flops_fwd_bwd(w) * args.sweep_steps / (ms / 1e3) / 1e12, 2),
            "unit": "TFLOP/s", "fwd_ms": round(fwd, 4), "bwd_ms": round(bwd, 4), "tau": args.tau,
            "note": "dQ contributions added in key order (turn counters): bitwise reproducible gradients"}


def bench_c5(args, dist_: Dist, dev) -> dict:
    """Config 5 (B8 H16 N16384 d128 bf16, fwd+bwd) with batch x heads sharded
    over the ranks (strong scaling of the fixed 128 heads): each rank runs its
    contiguous block of heads; reported value = total FLOPs / max-over-ranks time."""
    from paper_01_anti_decoy_pnfirtau_b200 import TauGradReducer, bh_range

    w = WORKLOADS["c5"]
    B, H, N, D = w["B"], w["H"], w["N"], w["D"]
    lo, hi = bh_range(B, H, dist_.rank, dist_.world)
    ws = dict(w, B=1, H=hi - lo)
    q, k, v, do = make_inputs(ws, args.seed + 50 + lo, dev)
    tau = torch.tensor(0.0, device=dev, requires_grad=True)
    ms, fwd, bwd = _time_fwd_bwd(q, k, v, do, tau, args.c5_steps, 2, TauGradReducer(dist_.tau_group))
    ms = dist_.max(ms, dev)
    total = flops_fwd_bwd(w)
    mine = flops_fwd_bwd(ws)
    peaks = measured_peaks()
    bwd_tf = 5.0 * ws["B"] * ws["H"] * N * N * D / (bwd / 1e3) / 1e12
    return {
        "workload": w["desc"], "heads_per_rank": hi - lo, "steps": args.c5_steps, "scaling": "strong",
        "ms_per_step": round(ms / args.c5_steps, 3),
        "value": round(total * args.c5_steps / (ms / 1e3) / 1e12, 2), "unit": "TFLOP/s",
        "fwd_ms": round(fwd, 3), "bwd_ms": round(bwd, 3),
        "roofline": {"bound": "tensor", "kernel": "flash_bwd", "achieved": round(bwd_tf, 2),
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": round(bwd_tf / peaks["bf16_tflops"], 4),
                     "flops_per_launch": 5.0 * ws["B"] * ws["H"] * N * N * D, "ms_per_launch": round(bwd, 3),
                     "traffic": (profile_traffic("flash_bwd:c5") or 0) * (hi - lo) / (B * H) or None,
                     "traffic_source": profile_traffic_source("flash_bwd:c5")},
        "rank0_fwd_tflops": round(2.0 * ws["B"] * ws["H"] * N * N * D / (fwd / 1e3) / 1e12, 2),
        "flops_per_step_per_rank": mine,
    }


def bench_e2e(args, dist_: Dist, w: dict, dev, flops: float, P) -> dict:
    """Same op through the public API with pinned host inputs and host outputs:
    every step copies q,k,v,dO host->device and out,dq,dk,dv,dtau device->host.

    The step is pipelined over chunks of whole heads (--e2e-chunks, default 4: two
    batch elements each for config 3; one call of the public API per chunk; each
    call and its copies cost ~0.4 ms of host time, so 8 chunks are host-bound), as a
    caller streaming host data would run it: the host->device copies of chunk i+1,
    the attention fwd+bwd of chunk i and the device->host copies of chunk i-1 run
    on three streams, so the two PCIe directions and the kernels overlap, and so do
    consecutive steps (step s+1's first uploads start once step s's compute has
    read those device buffers, not after its last download; the timed region ends
    when the last step's results are in host memory). Every byte of the serial
    version is still copied every step; dtau is the sum over chunks (all-reduced
    over ranks). `host_link` times the same copies alone."""
    from paper_01_anti_decoy_pnfirtau_b200.pnfirtau_ops import flash_pn_fir_tau_attention

    hq, hk, hv, hdo = (t.detach().cpu().pin_memory() for t in make_inputs(w, args.seed + 7, dev))
    outs = [torch.empty_like(hq).pin_memory() for _ in range(4)]
    htau = torch.empty((), dtype=torch.float32).pin_memory()
    tau = torch.tensor(args.tau, device=dev, requires_grad=True)
    # chunks of whole heads: (b, h0, h1) blocks, each contiguous in the host buffers
    B, H = hq.shape[0], hq.shape[1]
    want = max(1, args.e2e_chunks)
    if want <= B:  # whole batch elements
        bounds = [(B * i // want, B * (i + 1) // want, 0, H) for i in range(want)]
    else:  # every batch element split into head groups
        hsplit = min(H, (want + B - 1) // B)
        bounds = [(b, b + 1, H * j // hsplit, H * (j + 1) // hsplit) for b in range(B) for j in range(hsplit)]
    nchunk = len(bounds)
    gq_, gk_, gv_, gdo_ = (torch.empty(t.shape, device=dev, dtype=t.dtype) for t in (hq, hk, hv, hdo))  # device inputs
    s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    from paper_01_anti_decoy_pnfirtau_b200 import TauGradReducer

    reducer = TauGradReducer(dist_.tau_group)
    done_cmp = [None] * nchunk  # compute of chunk i finished reading its device inputs (previous step)

    def step():
        total = None
        for i, (b0, b1, h0, h1) in enumerate(bounds):
            sl = (slice(b0, b1), slice(h0, h1))
            with torch.cuda.stream(s_in):
                if done_cmp[i] is not None:
                    s_in.wait_event(done_cmp[i])
                for d, h in zip((gq_, gk_, gv_, gdo_), (hq, hk, hv, hdo)):
                    d[sl].copy_(h[sl], non_blocking=True)
                landed = torch.cuda.Event()
                landed.record(s_in)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(landed)
                q, k, v = (t[sl].detach().requires_grad_(True) for t in (gq_, gk_, gv_))
                out = flash_pn_fir_tau_attention(q, k, v, tau)
                gq, gk, gv, gt = torch.autograd.grad(out, (q, k, v, tau), gdo_[sl])
                total = gt if total is None else total + gt
                ev = torch.cuda.Event()
                ev.record(s_cmp)
                done_cmp[i] = ev
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev)
                for h, d in zip(outs, (out, gq, gk, gv)):
                    d.record_stream(s_out)
                    h[sl].copy_(d, non_blocking=True)
        with torch.cuda.stream(s_cmp):
            total.record_stream(s_out)
            if dist_.world > 1:
                reducer.push(total)  # fp64 all-reduce on the reducer's side stream
            fin = torch.cuda.Event()
            fin.record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(fin)
            summed = reducer.result() if dist_.world > 1 else total  # s_out waits for the all-reduce
            htau.copy_(summed, non_blocking=True)

    main = torch.cuda.current_stream(dev)
    for _ in range(max(2, min(args.warmup, 3))):
        step()
    torch.cuda.synchronize()
    steps = args.steps
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist_.barrier()
    torch.cuda.synchronize()
    s.record(main)
    for st_ in (s_in, s_cmp, s_out):
        st_.wait_event(s)
    for _ in range(steps):
        step()
    for st_ in (s_in, s_cmp, s_out):
        main.wait_stream(st_)
    e.record(main)
    torch.cuda.synchronize()
    ms = dist_.max(s.elapsed_time(e), dev)
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hdo))
    d2h = sum(t.numel() * t.element_size() for t in outs) + htau.element_size()
    link = _host_link_floor(dist_, dev, (hq, hk, hv, hdo), (gq_, gk_, gv_, gdo_), outs)
    per_step = ms / steps
    return {"value": round(dist_.world * flops * steps / (ms / 1e3) / 1e12, 3), "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(per_step, 4),
            "steps": steps, "chunks": nchunk,
            "api": "flash_pn_fir_tau_attention + torch.autograd.grad per batch chunk, pinned host buffers, "
                   "H2D / compute / D2H on three streams",
            "host_link": dict(link, frac=round(link["both_ms"] / per_step, 3))}


def _host_link_floor(dist_: Dist, dev, hin, din, hout, reps: int = 3) -> dict:
    """The copies of one e2e step alone: every input host->device and every output
    device->host, first one direction at a time, then both at once on two streams
    (the floor of a step whose copies overlap its kernels perfectly). Pinned host
    buffers, one copy call per tensor, max over ranks (all ranks copy at once, as
    in the step, so they share the host's memory and PCIe switches). The downloads
    read their own device buffers, not the ones being uploaded."""
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    dsrc = [torch.zeros_like(h, device=dev) for h in hout]

    def run(h2d: bool, d2h: bool) -> float:
        torch.cuda.synchronize()
        dist_.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        main = torch.cuda.current_stream(dev)
        a.record(main)
        s_in.wait_event(a)
        s_out.wait_event(a)
        for _ in range(reps):
            if h2d:
                with torch.cuda.stream(s_in):
                    for d, h in zip(din, hin):
                        d.copy_(h, non_blocking=True)
            if d2h:
                with torch.cuda.stream(s_out):
                    for h, d in zip(hout, dsrc):
                        h.copy_(d, non_blocking=True)
        main.wait_stream(s_in)
        main.wait_stream(s_out)
        b.record(main)
        torch.cuda.synchronize()
        return dist_.max(a.elapsed_time(b), dev) / reps

    run(True, True)  # warm-up
    nin = sum(t.numel() * t.element_size() for t in hin)
    nout = sum(t.numel() * t.element_size() for t in hout)
    t_in, t_out, t_both = run(True, False), run(False, True), run(True, True)
    return {"h2d_ms": round(t_in, 4), "d2h_ms": round(t_out, 4), "both_ms": round(t_both, 4),
            "h2d_gbs": round(nin / t_in / 1e6, 1), "d2h_gbs": round(nout / t_out / 1e6, 1),
            "note": "the step's copies alone (no kernels); frac = both_ms / e2e ms_per_step"}


def bench_lm_kernels(args, dev, iters: int = 10) -> dict:
    """The LM step's own kernels (csrc/lm_step.cu) alone at config 4's shapes:
    the head cross-entropy over `--lm-kernel-rows` x 33280 bf16 logits (one
    pass: logits read, gradient written), the residual add + LayerNorm forward
    and backward over [16384, 256], and the MLP's GELU forward and GELU backward
    + bias gradient over [16384, 1024]. Each entry point is called once first
    (the order an ncu capture sees), then timed with CUDA events; three operand
    sets rotate so every pass reads more than L2 holds. GB/s counts the
    algorithmic bytes (each operand read or written once). The timed loop
    launches back to back from the host; the weight-gradient GEMMs are timed
    from a replayed CUDA graph of the same calls (their host-side setup, two
    tensor-map encodes per call, would otherwise be timed)."""
    from paper_01_anti_decoy_pnfirtau_b200 import _lib

    L = _lib.lib()
    st = torch.cuda.current_stream(dev).cuda_stream
    g = torch.Generator(device=dev).manual_seed(args.seed + 7)
    BF, F32 = _lib.DTYPE_BF16, _lib.DTYPE_F32
    M1, V, ld = args.lm_kernel_rows, 33278, 33280
    M, C, H = 16384, 256, 1024
    logits = (torch.randn(M1, ld, generator=g, device=dev) * 3).to(torch.bfloat16)
    tgt = torch.randint(0, V, (M1,), generator=g, device=dev)
    row_loss = torch.empty(M1, device=dev)
    gtab = torch.empty(_lib.GELU_TABLE_FLOATS, device=dev)
    _lib.check(L.pnft_gelu_table(gtab.data_ptr(), st), "pnft_gelu_table")
    lnb = L.pnft_layernorm_bwd_workspace_size(M, C)
    cb = L.pnft_colsum_workspace_size(M, H)
    w, b = torch.ones(C, device=dev), torch.zeros(C, device=dev)
    dw, db, db1 = torch.empty(C, device=dev), torch.empty(C, device=dev), torch.empty(H, device=dev)
    wg1, wg2 = torch.empty(H, C, device=dev), torch.empty(C, C, device=dev)
    wgb = max(L.pnft_gemm_at_b_workspace_size(M, H, C), L.pnft_gemm_at_b_workspace_size(M, C, C))
    wgws = torch.empty(max(wgb, 16), dtype=torch.uint8, device=dev)
    sets = []
    for _ in range(3):
        o = {"x": torch.randn(M, C, generator=g, device=dev),
             "r": torch.randn(M, C, generator=g, device=dev).to(torch.bfloat16),
             "s": torch.empty(M, C, device=dev), "y": torch.empty(M, C, device=dev, dtype=torch.bfloat16),
             "mean": torch.empty(M, device=dev), "rstd": torch.empty(M, device=dev),
             "gy": torch.randn(M, C, generator=g, device=dev).to(torch.bfloat16),
             "gs": torch.randn(M, C, generator=g, device=dev), "dx": torch.empty(M, C, device=dev),
             "dr": torch.empty(M, C, device=dev, dtype=torch.bfloat16),
             "lnws": torch.empty(lnb, dtype=torch.uint8, device=dev),
             "dh": torch.randn(M, H, generator=g, device=dev).to(torch.bfloat16),
             "a0": torch.randn(M, H, generator=g, device=dev).to(torch.bfloat16),
             "da": torch.empty(M, H, device=dev, dtype=torch.bfloat16),
             "cws": torch.empty(cb, dtype=torch.uint8, device=dev)}
        sets.append(o)
    calls = {
        "head_xent": (lambda o, st: L.pnft_lm_xent(logits.data_ptr(), ld, tgt.data_ptr(), -100, row_loss.data_ptr(),
                                               M1, V, 1.0, None, None, st), 2 * M1 * ld * 2,
                      f"[{M1}, {ld}] bf16 logits -> loss + gradient in place"),
        "add_layernorm_fwd": (lambda o, st: L.pnft_add_layernorm_fwd(
            o["x"].data_ptr(), C, o["r"].data_ptr(), C, BF, o["s"].data_ptr(), C, w.data_ptr(), b.data_ptr(), 1e-5,
            o["y"].data_ptr(), C, o["mean"].data_ptr(), o["rstd"].data_ptr(), M, C, F32, BF, st),
            M * C * (4 + 2 + 4 + 2), f"[{M}, {C}]: x f32 + r bf16 -> s f32, y bf16"),
        "add_layernorm_bwd": (lambda o, st: L.pnft_add_layernorm_bwd(
            o["gy"].data_ptr(), C, o["gs"].data_ptr(), C, o["s"].data_ptr(), C, w.data_ptr(), o["mean"].data_ptr(),
            o["rstd"].data_ptr(), o["dx"].data_ptr(), C, o["dr"].data_ptr(), C, BF, dw.data_ptr(), db.data_ptr(),
            o["lnws"].data_ptr(), lnb, M, C, BF, F32, st),
            M * C * (2 + 4 + 4 + 4 + 2), f"[{M}, {C}]: dy bf16, s f32, gs f32 -> dx f32, dr bf16, dgamma, dbeta"),
        "gelu_bwd_colsum": (lambda o, st: L.pnft_gelu_bwd_colsum(
            o["dh"].data_ptr(), H, o["a0"].data_ptr(), H, o["da"].data_ptr(), H, db1.data_ptr(), o["cws"].data_ptr(),
            cb, M, H, BF, gtab.data_ptr(), st), M * H * 6, f"[{M}, {H}] bf16: dh, a -> da, bias gradient"),
        "gelu_fwd": (lambda o, st: L.pnft_gelu_fwd(o["a0"].data_ptr(), H, o["da"].data_ptr(), H, M, H, BF,
                                              gtab.data_ptr(), st), M * H * 4, f"[{M}, {H}] bf16"),
        # weight gradients dW = dY^T X of the MLP's first layer ([1024, 256] over 16384 tokens) and of the
        # attention's output projection ([256, 256])
        "weight_grad_fc1": (lambda o, st: L.pnft_gemm_at_b(o["da"].data_ptr(), H, o["gy"].data_ptr(), C,
                                                       wg1.data_ptr(), C, wgws.data_ptr(), wgb, M, H, C, BF, None,
                                                       st), (M * H + M * C) * 2 + H * C * 4,
                            f"[{M}, {H}]^T x [{M}, {C}] bf16 -> [{H}, {C}] fp32, split-K tcgen05"),
        "weight_grad_out": (lambda o, st: L.pnft_gemm_at_b(o["gy"].data_ptr(), C, o["r"].data_ptr(), C,
                                                       wg2.data_ptr(), C, wgws.data_ptr(), wgb, M, C, C, BF, None,
                                                       st), (M * C + M * C) * 2 + C * C * 4,
                            f"[{M}, {C}]^T x [{M}, {C}] bf16 -> [{C}, {C}] fp32, split-K tcgen05"),
    }
    for name, (fn, _, _) in calls.items():
        _lib.check(fn(sets[0], st), name)
    torch.cuda.synchronize()
    peak = measured_peaks().get("hbm_gbs")
    res = {}
    s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for name, (fn, nbytes, what) in calls.items():
        for i in range(3):
            fn(sets[i % 3], st)
        if name.startswith("weight_grad"):
            # device time from a replayed graph of the calls (their host-side setup is not timed)
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                for i in range(iters):
                    _lib.check(fn(sets[i % 3], side.cuda_stream), name)
            torch.cuda.current_stream(dev).wait_stream(side)
            graph.replay()
            torch.cuda.synchronize()
            s_.record()
            graph.replay()
            e_.record()
            torch.cuda.synchronize()
            del graph
        else:
            s_.record()
            for i in range(iters):
                fn(sets[i % 3], st)
            e_.record()
            torch.cuda.synchronize()
        us = s_.elapsed_time(e_) / iters * 1e3
        gbs = nbytes / us / 1e3
        res[name] = {"us": round(us, 2), "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / peak, 3) if peak else None,
                     "what": what}
        if name.startswith("weight_grad"):
            mm = H if name.endswith("fc1") else C
            res[name]["TFLOP/s"] = round(2 * M * mm * C / us / 1e6, 1)
    res["note"] = ("each kernel alone, CUDA events, operands rotated over three sets (the cross-entropy's logits "
                   "exceed L2 on their own); the same kernels inside the LM step: profiles/lm_step_kernels.md")
    return res


def bench_fir(args, dist_: Dist, dev, iters: int = 20) -> dict:
    """Standalone causal FIR (triton_causal_fir, 7 Gaussian taps, bf16) as achieved
    HBM GB/s: bytes = one read of x + one write of y per pass (the 6-row halo
    re-reads are not counted). Shapes: the LM's keys [32, 512, 256] and the keys
    of config 5 viewed as [8, 16384, 16*128]. Buffers rotate so the inputs of
    consecutive passes together exceed the 126 MiB L2 (every pass reads DRAM).
    Three figures per shape: `GB/s` through the public API call by call (at the
    LM shape this is bound by the host's per-call overhead), `device_GB/s` from
    a CUDA graph of the same calls replayed (kernel time, no host overhead), and
    `dtaps_GB/s`, the tap gradient alone (torch.autograd.grad of the output with
    respect to the taps: one read of gy and one of x per pass)."""
    from paper_01_anti_decoy_pnfirtau_b200.pnfirtau_attention import causal_gaussian_taps
    from paper_01_anti_decoy_pnfirtau_b200.pnfirtau_ops import triton_causal_fir

    peak = measured_peaks().get("hbm_gbs")
    taps = causal_gaussian_taps(7, device=dev)
    g = torch.Generator(device=dev).manual_seed(args.seed + 11)
    res = {}

    def timed(fn, n):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        fn(n)
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / n

    for name, shape in (("lm_k_32x512x256", (32, 512, 256)), ("c5_k_8x16384x2048", (8, 16384, 2048))):
        nbytes = 2 * shape[0] * shape[1] * shape[2]
        nbuf = max(1, -(-2 * L2_BYTES // nbytes))
        xs = [torch.randn(shape, generator=g, device=dev).to(torch.bfloat16) for _ in range(nbuf)]
        for i in range(3):
            triton_causal_fir(xs[i % nbuf], taps)

        def calls(n):
            for i in range(n):
                triton_causal_fir(xs[i % nbuf], taps)

        ms = timed(calls, iters)
        # the same calls captured once in a CUDA graph and replayed: device time per call
        ncap = 2 * nbuf if nbytes < L2_BYTES else nbuf
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            calls(ncap)
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            calls(ncap)
        graph.replay()
        reps = max(1, iters // ncap)
        ms_dev = timed(lambda n: [graph.replay() for _ in range(reps)], 1) / (reps * ncap)
        del graph
        # tap gradient alone (gx not requested)
        th = taps.clone().requires_grad_(True)
        gys = [torch.randn(shape, generator=g, device=dev).to(torch.bfloat16) for _ in range(nbuf)]

        def dtaps_calls(n):
            for i in range(n):
                y = triton_causal_fir(xs[i % nbuf], th)
                torch.autograd.grad(y, th, gys[i % nbuf])

        dtaps_calls(2)
        ms_fwd_dt = timed(dtaps_calls, iters)  # includes the forward pass
        ms_dt = max(ms_fwd_dt - ms, 1e-6)
        gbs = 2 * nbytes / (ms / 1e3) / 1e9
        gbs_dev = 2 * nbytes / (ms_dev / 1e3) / 1e9
        gbs_dt = 2 * nbytes / (ms_dt / 1e3) / 1e9
        res[name] = {"ms": round(ms, 4), "bytes_per_pass": 2 * nbytes, "GB/s": round(gbs, 1),
                     "frac_of_hbm": round(gbs / peak, 3) if peak else None,
                     "device_ms": round(ms_dev, 4), "device_GB/s": round(gbs_dev, 1),
                     "device_frac_of_hbm": round(gbs_dev / peak, 3) if peak else None,
                     "dtaps_ms": round(ms_dt, 4), "dtaps_GB/s": round(gbs_dt, 1),
                     "dtaps_frac_of_hbm": round(gbs_dt / peak, 3) if peak else None}
        del xs, gys
    res["peak_GB/s"] = peak
    res["note"] = ("device_* from a replayed CUDA graph of the calls; dtaps_* = (forward + tap-gradient call) "
                   "minus the forward call, 2 reads of B*N*C bf16 per pass")
    return res


def bench_lm(args, dist_: Dist, dev) -> dict:
    """Config 4: 6-layer LM training step, bf16 autocast, AdamW, data parallel
    over NCCL at N > 1. Headline: the step captured in one CUDA graph
    (lm.GraphedTrainStep: forward, backward, one NCCL gradient average, clip,
    fused AdamW). Beside it the same step run eagerly (DDP at N > 1), which
    is bound by the host's per-op launch overhead."""
    import torch.distributed as dist

    from paper_01_anti_decoy_pnfirtau_b200.lm import GraphedTrainStep, LMConfig, PnFirLM, make_optimizer, train_step

    cfg = LMConfig()
    B, N = 32, cfg.max_seq
    g = torch.Generator(device=dev).manual_seed(args.seed + 17 * dist_.rank)
    batches = [torch.randint(0, cfg.vocab, (B, N), generator=g, device=dev) for _ in range(4)]
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(run_step) -> tuple[float, torch.Tensor]:
        for i in range(3):
            run_step(batches[i % 4])
        torch.cuda.synchronize()
        dist_.barrier()
        torch.cuda.synchronize()
        s.record()
        loss = None
        for i in range(args.lm_steps):
            loss = run_step(batches[i % 4])
        e.record()
        torch.cuda.synchronize()
        return dist_.max(s.elapsed_time(e), dev) / args.lm_steps, loss

    torch.manual_seed(args.seed)
    model = PnFirLM(cfg).to(dev)
    nparams = model.param_count()
    opt = make_optimizer(model, capturable=True)
    graphed = GraphedTrainStep(model, opt, batches[0], group=dist.group.WORLD if dist_.active else None)
    ms_g, loss_g = timed(graphed.step)
    loss_g = float(loss_g)
    graphed.close()
    del graphed, opt, model
    torch.cuda.synchronize()

    torch.manual_seed(args.seed)
    model = PnFirLM(cfg).to(dev)
    if dist_.active:
        model = torch.nn.parallel.DistributedDataParallel(model, device_ids=[dev.index])
    opt = make_optimizer(model)
    ms_e, loss_e = timed(lambda idx: train_step(model, opt, idx))
    tok = dist_.world * B * N
    return {"tokens_per_s": round(tok / (ms_g / 1e3), 1), "ms_per_step": round(ms_g, 3), "loss": round(loss_g, 4),
            "tokens_per_s_eager": round(tok / (ms_e / 1e3), 1), "ms_per_step_eager": round(ms_e, 3),
            "loss_eager": round(float(loss_e), 4), "steps": args.lm_steps, "global_batch": B * dist_.world,
            "seq_len": N, "params": nparams,
            "model": "6-layer Pre-LN pn_fir_tau LM, D256 H4 MLP4x V33278, bf16 autocast, AdamW",
            "step": "one CUDA graph per step: forward, backward, NCCL gradient average (N > 1), clip, fused AdamW; "
                    "eager: the same ops launched one by one (DDP at N > 1)",
            "step_ops": "library LayerNorm, MLP-backward and one-pass head cross-entropy kernels, fused AdamW",
            "parallelism": f"dp{dist_.world}" if dist_.world > 1 else "single GPU"}


# ---------------------------------------------------------------------------
# reference arm: the reference's eager algorithm on the host cores
# ---------------------------------------------------------------------------


def bench_reference(args, dist_: Dist) -> dict | None:
    """The reference arm: the reference's own CPU path of the operator on the
    host cores (see cpu_oracle_sample; one whole (b,h) slice per step), rank 0
    only. Alongside, as `triton_b200`, the reference's own Triton Flash kernels
    timed on GPU 0 (reference_triton_b200)."""
    if dist_.rank != 0:
        return None
    w = WORKLOADS[args.workload]
    for _ in range(args.warmup):
        cpu_oracle_sample(w, 0.0, args.seed, steps=1)
    tf, cores, n, el, kind, what = cpu_oracle_sample(w, 0.0, args.seed, steps=args.steps)
    sample = (f"each step = one (b,h) slice [1,1,{w['N']},{w['D']}] fp32 fwd+bwd of the {args.workload} workload "
              f"({what}), {cores} threads")
    res = {
        "impl": "reference", "metric": METRIC, "value": round(tf, 6), "unit": "TFLOP/s", "n_gpus": dist_.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * el / n, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.workload}: {w['desc']}", "B": w["B"], "H": w["H"], "N": w["N"], "d": w["D"]},
        "cpu_baseline": {"value": round(tf, 6), "unit": "TFLOP/s", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": round(tf, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_triton:
        res["triton_b200"] = reference_triton_b200(args, w)
    return res


def _claim_stdout():
    """Point file descriptor 1 at stderr for the run (NCCL and other native code
    print banners to stdout) and return a writer on the original stdout, which
    then carries exactly the one JSON line."""
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    return out


def main():
    out = _claim_stdout()
    args = parse_args()
    dist_ = Dist()
    if args.impl == "reference":
        res = bench_reference(args, dist_)
        if res is not None:
            print(json.dumps(res), file=out, flush=True)
        return
    if args.lm_kernels_only:
        dev = torch.device("cuda", dist_.local_rank)
        torch.cuda.set_device(dev)
        print(json.dumps({"lm_kernels": bench_lm_kernels(args, dev)}), file=out, flush=True)
        return
    res = bench_ours(args, dist_)
    if dist_.rank == 0:
        print(json.dumps(res), file=out, flush=True)
    dist_.close()


if __name__ == "__main__":
    main()
