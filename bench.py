#!/usr/bin/env python
"""Benchmark of the batched FP32 geqrf hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one factorization of one batch of the workload config. The default
workload is config 5 (b=8, n=4096, iid N(0,1), seed 4): the largest
single-GPU config of the metric. Scaling is strong by default: the config's
fixed global batch is sharded across the N ranks (``sharding.shard_range``;
config 5 gives one matrix per GPU at N=8), with no collective on the hot path;
``--scaling weak`` instead gives every rank a full batch of its own. Timing: W
untimed warm-up steps, then K steps, each bracketed by CUDA events on the
launching stream, with a 256 MiB write between steps to flush L2 (outside the
events). The timed region is bracketed by a barrier and
``torch.cuda.synchronize()``; the reported time is the MAX over ranks of the
summed step times. Rank 0 prints one JSON line. At N > 1 the line also carries
a strong-scaling sweep of configs 1-4 (``strong``); at N = 1 a per-config
sweep with gates, parity and CPU times (``per_config``).

``--impl reference`` times the reference's own CPU implementation of the path,
``torch.geqrf`` on the host cores (``src/qrbench/reference.py:18-20``), on the
same config and metric (rank 0 only; other ranks exit 0).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "median ms/batch + matrices/s of batched fp32 geqrf at 1/2/4/8 B200; % roofline"
UNIT = "matrices/s"
L2_FLUSH_BYTES = 256 << 20
FP32_FFMA_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # at clocks.max.sm


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", type=int, default=5, help="workload config index (1-5)")
    ap.add_argument("--scaling", choices=("strong", "weak"), default="strong",
                    help="strong: shard the config's batch over the ranks; weak: a batch per rank")
    ap.add_argument("--no-configs", action="store_true", help="skip the per-config sweeps")
    ap.add_argument("--no-cpu", action="store_true", help="skip CPU geqrf timings")
    ap.add_argument("--cpu-seconds", type=float, default=8.0, help="CPU baseline sample budget")
    ap.add_argument("--set", action="append", default=[], metavar="KEY=VALUE",
                    help="library test hook (qrb_set_config) applied before timing; repeatable")
    ap.add_argument("--chunks", type=int, default=0,
                    help="e2e pipeline depth for qrb_geqrf_f32_host (0 = automatic)")
    ap.add_argument("--batch", type=int, default=None,
                    help="global batch (default: the config's batch); for small profiling cases")
    ap.add_argument("--workload", choices=("geqrf", "gram"), default="geqrf",
                    help="gram: time the statistics step S = G G^T (b=--batch or 640, n=k=512)")
    ap.add_argument("--quick", action="store_true",
                    help="device-timed steps only: no gate, e2e, CPU baseline or sweep (profiling)")
    return ap.parse_args(argv)


def apply_hooks(items) -> dict:
    from gpumode_qr_b200 import _lib

    out = {}
    for it in items:
        key, _, val = it.partition("=")
        _lib.set_config(key.strip(), int(val))
        out[key.strip()] = int(val)
    return out


# ---------------------------------------------------------------------------
# clocks sampled during the timed region (NVML reads only)
# ---------------------------------------------------------------------------


class ClockSampler:
    REASONS = {
        0x0000000000000001: "gpu_idle",
        0x0000000000000002: "applications_clocks_setting",
        0x0000000000000004: "sw_power_cap",
        0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sync_boost",
        0x0000000000000040: "sw_thermal_slowdown",
        0x0000000000000080: "hw_thermal_slowdown",
        0x0000000000000100: "hw_power_brake_slowdown",
        0x0000000000000200: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.period = period_s
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.err = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = device_index
            if vis:
                ids = [v.strip() for v in vis.split(",") if v.strip()]
                if device_index < len(ids) and ids[device_index].isdigit():
                    idx = int(ids[device_index])
            self._h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001 - clocks are reported as unavailable
            self._nv = None
            self.err = repr(e)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, rs))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv is not None:
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
                    "note": self.err or "no samples"}
        mhz = [s for s, _ in self.samples]
        mask = 0
        for _, r in self.samples:
            mask |= r
        reasons = [name for bit, name in self.REASONS.items() if mask & bit and name != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}


def measured_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs"), "bf16_tflops": d.get("bf16_tflops"),
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def flop_peak(route: str, peaks: dict) -> tuple[float, str, str]:
    """(peak TFLOP/s, bound, derivation) of the pipe a large-n route computes on.

    The tensor-core routes run 3xTF32: three TF32 MMAs per FP32 product, and
    B200's dense TF32 rate is half its BF16 rate, so the effective peak is the
    BF16 figure / 6. The FFMA routes have no measured FP32 figure, so the
    nominal CUDA-core rate is used."""
    if "tcgen05" in route:
        bf16 = peaks["bf16_tflops"]
        return (bf16 / 6.0, "tensor",
                f"{peaks['source']} bf16 burst {bf16} TFLOP/s / 2 (tf32 rate) / 3 (3xTF32 products)")
    return (FP32_FFMA_NOMINAL_TFLOPS, "fp32_ffma",
            "nominal 148 SMs x 128 FFMA x 2 x 1965 MHz (no measured FP32 figure)")


def profile_record(workload: str):
    """Per-workload figures taken from committed ncu summaries under profiles/
    (DRAM traffic per launch of the dominant kernel, its share of the launch
    list), or None."""
    p = REPO / "profiles" / "roofline_traffic.json"
    if not p.exists():
        return None
    rec = json.loads(p.read_text()).get(workload)
    return rec if isinstance(rec, dict) else None


def config_dict(cfg, global_batch: int, scaling: str) -> dict:
    """The workload description, identical in both arms."""
    inp = ("iid N(0,1)" if cfg.kind == "iid" else
           f"U diag(logspace(0, {cfg.log10_cond:g}, n)) V^T, U and V Haar")
    return {"workload": f"cfg{cfg.index}_b{global_batch}_n{cfg.n}", "global_batch": global_batch,
            "n": cfg.n, "seed": cfg.seed, "inputs": inp, "scaling": scaling}


def global_batch_of(args, cfg, world: int) -> int:
    b = cfg.batch if args.batch is None else args.batch
    return b * world if args.scaling == "weak" else b


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own CPU path, torch.geqrf (LAPACK) on the host
# ---------------------------------------------------------------------------


def cpu_geqrf_rate(A_cpu, budget_s: float, min_reps: int = 2, max_reps: int = 200):
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    torch.geqrf(A_cpu[:1])  # warm-up (threads, MKL init)
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < max_reps and (len(times) < min_reps or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        torch.geqrf(A_cpu)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {
        "value": A_cpu.shape[0] / med,
        "unit": UNIT,
        "median_ms": med * 1e3,
        "reps": len(times),
        "cores": torch.get_num_threads(),
        "kind": "reference",
        "sample": (f"torch.geqrf on CPU (LAPACK sgeqrf; the reference's geqrf_reference, "
                   f"src/qrbench/reference.py:18-20), full batch of {A_cpu.shape[0]} x "
                   f"{A_cpu.shape[1]}x{A_cpu.shape[2]}, median of {len(times)} runs"),
        "cpu_model": _cpu_model(),
    }


def _cpu_model() -> str:
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args, info) -> int:
    """Reference arm: CPU torch.geqrf on this arm's config, rank 0 only."""
    from gpumode_qr_b200 import inputs

    if info.rank != 0:
        return 0
    import torch

    cfg = inputs.config(args.config)
    gb = global_batch_of(args, cfg, info.world)
    A = inputs.make_config_input(cfg, gb)
    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(max(1, min(args.warmup, 3))):
        torch.geqrf(A)
    steps = max(1, args.steps)
    # bound the run: cap the number of timed steps to ~60 s of CPU work
    t0 = time.perf_counter()
    torch.geqrf(A)
    est = time.perf_counter() - t0
    steps = max(1, min(steps, int(60.0 / max(est, 1e-6))))
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        torch.geqrf(A)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = gb * steps / total
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": total / steps * 1e3,
        "median_ms": statistics.median(times) * 1e3,
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded torch.Generator on CPU)",
        "config": config_dict(cfg, gb, args.scaling),
        "cpu_baseline": {
            "value": value,
            "unit": UNIT,
            "cores": torch.get_num_threads(),
            "kind": "reference",
            "sample": (f"torch.geqrf on CPU (the reference's geqrf_reference, "
                       f"src/qrbench/reference.py:18-20), {steps} steps of the full "
                       f"{gb}-matrix batch, all host threads"),
        },
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------


def time_device_steps(step, steps: int, warmup: int, flush_buf, stream):
    """Per-step CUDA-event times (ms) with an L2 flush between steps."""
    import torch

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for k in range(steps):
        flush_buf.fill_(k & 0x7F)
        starts[k].record(stream)
        step()
        ends[k].record(stream)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def global_input(cfg, batch: int, info, dev):
    """(CPU tensor on rank 0 else None, device tensor of the whole seeded batch
    on every rank). Rank 0 draws the batch on its CPU; other ranks receive it
    by an NCCL broadcast (set-up only, outside every timed region)."""
    import torch
    import torch.distributed as dist

    from gpumode_qr_b200 import inputs

    if info.rank == 0:
        A_cpu = inputs.make_config_input(cfg, batch)
        A = A_cpu.to(dev)
    else:
        A_cpu = None
        A = torch.empty(batch, cfg.n, cfg.n, dtype=torch.float32, device=dev)
    if info.initialized:
        dist.broadcast(A, src=0)
    return A_cpu, A


def large_n_roofline(cfg, ms: float, rows: int, route: str, peaks: dict) -> dict:
    pk, bound, src = flop_peak(route, peaks)
    tf = 4.0 / 3.0 * cfg.n**3 * rows / (ms / 1e3) / 1e12
    return {"bound": bound, "achieved": tf, "peak": pk, "unit": "TFLOP/s", "frac": tf / pk,
            "peak_source": src, "frac_of_fp32_nominal": tf / FP32_FFMA_NOMINAL_TFLOPS}


def per_config_sweep(dev, flush_buf, cpu: bool, peaks: dict) -> dict:
    import torch

    from gpumode_qr_b200 import _lib, api, checker, inputs

    out = {}
    gpu_ms, cpu_ms = [], []
    stream = torch.cuda.current_stream(dev)
    for cfg in inputs.CONFIGS:
        A_cpu = inputs.make_config_input(cfg)
        A = A_cpu.to(dev)
        H = torch.empty_like(A)
        tau = torch.empty(cfg.batch, cfg.n, device=dev)
        fn = api.geqrf_into_fn(A, H, tau)
        route = api.route(cfg.batch, cfg.n)
        times = time_device_steps(fn, 10, 3, flush_buf, stream)
        med = statistics.median(times)
        gpu_ms.append(med)
        gate = checker.check(A, H, tau)
        rec = {
            "batch": cfg.batch,
            "n": cfg.n,
            "route": route,
            "median_ms": med,
            "min_ms": min(times),
            "matrices_per_s": cfg.batch / (med / 1e3),
            "gates": {"factor": gate.factor_residual, "factor_thr": gate.factor_threshold,
                      "orth": gate.orth_residual, "orth_thr": gate.orth_threshold,
                      "passed": gate.passed},
        }
        if cfg.n <= 64:
            gbs = cfg.bytes / (med / 1e3) / 1e9
            rec["roofline"] = {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"],
                               "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"]}
        else:
            rec["roofline"] = large_n_roofline(cfg, med, cfg.batch, route, peaks)
        if cpu:
            torch.set_num_threads(os.cpu_count() or 1)
            torch.geqrf(A_cpu[:1])
            ct = []
            for _ in range(3 if cfg.n < 4096 else 2):
                t0 = time.perf_counter()
                Hr, tr = torch.geqrf(A_cpu)
                ct.append((time.perf_counter() - t0) * 1e3)
            cmed = statistics.median(ct)
            cpu_ms.append(cmed)
            rec["cpu_geqrf_median_ms"] = cmed
            rec["speedup_vs_cpu"] = cmed / med
            if cfg.parity:
                par = checker.parity(H.cpu(), tau.cpu(), Hr, tr)
                rec["parity_vs_geqrf"] = {"h_rel": par.h_rel, "tau_rel": par.tau_rel,
                                          "col_rel": par.col_rel, "ok": par.ok()}
        if cfg.n >= 512:
            # the trailing-update pipe per n, whole factorization (median of 3 each)
            kinds = {}
            old_kind = _lib.get_config("larfb_kind")
            try:
                for kind, name in api.LARFB_KINDS.items():
                    _lib.set_config("larfb_kind", kind)
                    kinds[name] = statistics.median(time_device_steps(fn, 3, 1, flush_buf, stream))
            finally:
                _lib.set_config("larfb_kind", old_kind)
            rec["trailing_update_pipe_ms"] = kinds
        out[cfg.name] = rec
        del A, H, tau, A_cpu
        torch.cuda.empty_cache()
    gm = math.exp(sum(math.log(x) for x in gpu_ms) / len(gpu_ms))
    res = {"configs": out, "gpu_geomean_ms": gm}
    if cpu_ms:
        cg = math.exp(sum(math.log(x) for x in cpu_ms) / len(cpu_ms))
        res["cpu_geomean_ms"] = cg
        res["geomean_speedup_vs_cpu"] = cg / gm
        res["cpu_cores"] = torch.get_num_threads()
        res["cpu_model"] = _cpu_model()
    return res


def strong_sweep(info, dev, flush_buf, peaks: dict, skip: int) -> dict:
    """Strong scaling of the other configs at this N: each config's fixed batch
    sharded over the ranks, 10 timed steps, MAX over ranks of the per-rank
    median. Every rank runs the same steps and collectives."""
    import torch

    from gpumode_qr_b200 import api, inputs, sharding

    out = {}
    stream = torch.cuda.current_stream(dev)
    for cfg in inputs.CONFIGS:
        if cfg.index == skip:
            continue
        _, A_glob = global_input(cfg, cfg.batch, info, dev)
        s, e = sharding.shard_range(cfg.batch, info.rank, info.world)
        A = A_glob[s:e].contiguous()
        del A_glob
        H = torch.empty_like(A)
        tau = torch.empty(A.shape[0], cfg.n, device=dev)
        sharding.barrier(info)
        if e > s:
            med = statistics.median(
                time_device_steps(api.geqrf_into_fn(A, H, tau), 10, 3, flush_buf, stream))
        else:
            med = 0.0
        med = sharding.max_over_ranks(med, info)
        rec = {"global_batch": cfg.batch, "max_batch_per_gpu": -(-cfg.batch // info.world),
               "median_ms": med, "matrices_per_s": cfg.batch / (med / 1e3)}
        if cfg.n > 64:
            rec["roofline_per_gpu"] = large_n_roofline(
                cfg, med, -(-cfg.batch // info.world), api.route(max(e - s, 1), cfg.n), peaks)
        out[cfg.name] = rec
        del A, H, tau
        torch.cuda.empty_cache()
    return out


def gram_sweep(dev, flush_buf, b: int = 640) -> dict:
    """The statistics step in front of the factorization (S = G G^T, then QR of
    S) at the shape the reference's task statement singles out (batched
    512 x 512, contracted dimension 512): kernel time, FP32 roofline fraction
    of the Gram kernel (n (n + 1) k FLOPs per matrix, the symmetric count),
    Gram + factorization time, cuBLAS FP32 G @ G.mT (TF32 off) on the same GPU,
    and FP64 parity of S on four matrices."""
    import torch

    from gpumode_qr_b200 import api

    n, k = 512, 512
    g = torch.Generator().manual_seed(7)
    G_cpu = torch.randn(b, n, k, generator=g)
    G = G_cpu.to(dev)
    stream = torch.cuda.current_stream(dev)
    S = api.gram(G)
    ms = statistics.median(time_device_steps(lambda: api.gram(G), 10, 3, flush_buf, stream))
    ms_qr = statistics.median(time_device_steps(lambda: api.gram_geqrf(G), 5, 2, flush_buf, stream))
    old_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ms_torch = statistics.median(
            time_device_steps(lambda: torch.matmul(G, G.mT), 10, 3, flush_buf, stream))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old_tf32
    g64 = G_cpu[:4].double()
    want = g64 @ g64.transpose(-1, -2)
    err = float((S[:4].double().cpu() - want).abs().max() / want.abs().max())
    flops = b * n * (n + 1) * k
    tf = flops / (ms / 1e3) / 1e12
    del G, S
    torch.cuda.empty_cache()
    return {"workload": f"gram_b{b}_n{n}_k{k}", "gram_ms": ms, "gram_geqrf_ms": ms_qr,
            "torch_fp32_matmul_ms": ms_torch,
            "roofline": {"bound": "fp32_ffma", "achieved": tf, "peak": FP32_FFMA_NOMINAL_TFLOPS,
                         "unit": "TFLOP/s", "frac": tf / FP32_FFMA_NOMINAL_TFLOPS,
                         "flops_per_matrix": n * (n + 1) * k},
            "s_rel_err_vs_fp64": err}


def pcie_probe(A_host, H_host, A_dev, H_dev, dev, reps: int = 10) -> dict:
    """Copy-engine bandwidth of this box for the e2e step's buffers: one
    host-to-device copy, one device-to-host copy, and both at once on two
    streams (GB/s, median of ``reps``). Outside every timed region."""
    import torch

    s1 = torch.cuda.Stream(device=dev)
    s2 = torch.cuda.Stream(device=dev)

    def timed(fn):
        out = []
        for _ in range(reps + 2):
            cur = torch.cuda.current_stream(dev)
            a = torch.cuda.Event(enable_timing=True)
            z = torch.cuda.Event(enable_timing=True)
            a.record(cur)
            fn(cur)
            z.record(cur)
            torch.cuda.synchronize(dev)
            out.append(a.elapsed_time(z))
        return statistics.median(out[2:])

    def h2d(cur):
        s1.wait_stream(cur)
        with torch.cuda.stream(s1):
            A_dev.copy_(A_host, non_blocking=True)
        cur.wait_stream(s1)

    def d2h(cur):
        s2.wait_stream(cur)
        with torch.cuda.stream(s2):
            H_host.copy_(H_dev, non_blocking=True)
        cur.wait_stream(s2)

    nb = A_host.numel() * 4
    t_h, t_d = timed(h2d), timed(d2h)

    def both(cur):  # both directions in flight together
        s1.wait_stream(cur)
        s2.wait_stream(cur)
        with torch.cuda.stream(s1):
            A_dev.copy_(A_host, non_blocking=True)
        with torch.cuda.stream(s2):
            H_host.copy_(H_dev, non_blocking=True)
        cur.wait_stream(s1)
        cur.wait_stream(s2)

    t_b = timed(both)
    return {"h2d_gbs": nb / t_h / 1e6, "d2h_gbs": nb / t_d / 1e6, "both_gbs": 2 * nb / t_b / 1e6,
            "method": "pinned cudaMemcpyAsync of the step's A / H buffers, median of %d" % reps}


def run_gram_quick(args, info) -> int:
    """Profiling workload: the Gram kernel alone, device-timed."""
    import torch

    from gpumode_qr_b200 import api

    dev = torch.device("cuda", info.local_rank if info.initialized else 0)
    b = args.batch or 640
    G = torch.randn(b, 512, 512, generator=torch.Generator().manual_seed(7)).to(dev)
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    times = time_device_steps(lambda: api.gram(G), args.steps, args.warmup, flush_buf,
                              torch.cuda.current_stream(dev))
    if info.rank == 0:
        print(json.dumps({"quick": True, "workload": f"gram_b{b}_n512_k512",
                          "median_ms": statistics.median(times)}), flush=True)
    return 0


def run_ours(args, info) -> int:
    import torch

    from gpumode_qr_b200 import _lib, api, checker, inputs, sharding

    dev = torch.device("cuda", info.local_rank if info.initialized else 0)
    torch.cuda.set_device(dev)
    hooks = apply_hooks(args.set)
    if args.workload == "gram":
        return run_gram_quick(args, info)
    cfg = inputs.config(args.config)
    world = info.world
    gb = global_batch_of(args, cfg, world)
    A_glob_cpu, A_glob = global_input(cfg, gb, info, dev)
    s, e = sharding.shard_range(gb, info.rank, world)
    rows = e - s
    A = A_glob[s:e].contiguous()
    del A_glob
    H = torch.empty_like(A)
    tau = torch.empty(rows, cfg.n, device=dev)
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    step = api.geqrf_into_fn(A, H, tau) if rows > 0 else (lambda: None)
    route = api.route(max(rows, 1), cfg.n)

    # correctness gate on this rank's shard before timing
    step()
    torch.cuda.synchronize()
    gate = checker.check(A, H, tau) if (not args.quick and rows > 0) else None
    if gate is not None and not gate.passed:
        print(f"[bench] rank {info.rank}: gate FAILED {gate.as_dict()}", file=sys.stderr)

    # timed region: device-resident inputs
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sharding.barrier(info)
    torch.cuda.synchronize()
    _lib.set_config("launches", 0)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(dev.index) as clk:
        for k in range(args.steps):
            flush_buf.fill_(k & 0x7F)
            starts[k].record(stream)
            step()
            ends[k].record(stream)
        torch.cuda.synchronize()
    launches = _lib.get_config("launches")
    sharding.barrier(info)
    torch.cuda.synchronize()
    times = [a.elapsed_time(z) for a, z in zip(starts, ends)]
    my_med = statistics.median(times)
    total_ms = sharding.max_over_ranks(sum(times), info)
    med_ms = sharding.max_over_ranks(my_med, info)
    value = gb * args.steps / (total_ms / 1e3)
    launches_total = int(sharding.sum_over_ranks(launches, info))

    if args.quick:
        if info.rank == 0:
            print(json.dumps({"quick": True, "workload": f"cfg{cfg.index}_b{gb}_n{cfg.n}",
                              "route": route, "batch_per_gpu": rows, "median_ms": med_ms,
                              "value": value, "unit": UNIT, "hooks": hooks}), flush=True)
        return 0

    # e2e through the public API with pinned host buffers (copies in the timed region)
    A_host = A.cpu().pin_memory()
    H_host = torch.empty_like(A_host).pin_memory()
    tau_host = torch.empty(A_host.shape[0], cfg.n).pin_memory()
    e2e_steps = max(3, min(args.steps, 50))
    e2e_ws = torch.empty(max(api.host_workspace_bytes(max(rows, 1), cfg.n), 16), dtype=torch.uint8,
                         device=dev)

    def e2e_step():
        if rows > 0:
            api.geqrf_host(A_host, H_host, tau_host, device=dev, chunks=args.chunks,
                           workspace=e2e_ws)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    sharding.barrier(info)
    e_s = torch.cuda.Event(enable_timing=True)
    e_e = torch.cuda.Event(enable_timing=True)
    e_s.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e_e.record(stream)
    torch.cuda.synchronize()
    e2e_ms = sharding.max_over_ranks(e_s.elapsed_time(e_e), info)
    sharding.barrier(info)
    e2e_value = gb * e2e_steps / (e2e_ms / 1e3)
    h2d = A_host.numel() * 4
    d2h = H_host.numel() * 4 + tau_host.numel() * 4
    pcie = pcie_probe(A_host, H_host, A, H, dev) if rows > 0 else {}
    if pcie:
        pcie["bound_ms"] = max(h2d / (pcie["h2d_gbs"] * 1e6), d2h / (pcie["d2h_gbs"] * 1e6))
        pcie["e2e_frac"] = pcie["bound_ms"] / (e2e_ms / e2e_steps)

    peaks = measured_peaks()
    extra = {}
    if not args.no_configs:
        if world == 1:
            if info.rank == 0:
                extra["per_config"] = per_config_sweep(dev, flush_buf, not args.no_cpu, peaks)
                extra["gram"] = gram_sweep(dev, flush_buf)
        else:
            extra["strong"] = strong_sweep(info, dev, flush_buf, peaks, cfg.index)
    cpu = None
    if info.rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_geqrf_rate(A_glob_cpu, args.cpu_seconds)

    if info.rank == 0:
        rec = profile_record(f"cfg{cfg.index}_b{gb}_n{cfg.n}") or {}
        if cfg.n <= 64:
            alg_bytes = 2 * rows * cfg.n * cfg.n * 4
            ach = alg_bytes / (statistics.mean(times) / 1e3) / 1e9
            roof = {"bound": "hbm", "achieved": ach, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": ach / peaks["hbm_gbs"], "peak_source": peaks["source"],
                    "algorithmic_bytes_per_launch": alg_bytes}
        else:
            roof = large_n_roofline(cfg, statistics.mean(times), rows, route, peaks)
            roof["algorithmic_flops_per_step"] = 4.0 / 3.0 * cfg.n**3 * rows
            roof["scope"] = ("the whole factorization step on this GPU (panels and trailing "
                             "updates), CUDA events on the launching stream")
        roof["traffic"] = rec.get("traffic_bytes_per_launch")
        roof["kernel"] = rec.get("kernel") or route
        if rec:
            roof["profile"] = {k: v for k, v in rec.items() if k != "traffic_bytes_per_launch"}
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps,
            "median_ms": med_ms,
            "higher_is_better": True,
            "scaling": args.scaling,
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded torch.Generator on CPU, copied to HBM)",
            "config": config_dict(cfg, gb, args.scaling),
            "sharding": {"batch_per_gpu_rank0": rows, "max_batch_per_gpu": -(-gb // world),
                         "parallelism": f"batch-sharded dp{world}, no collective on the hot path",
                         "l2": "flushed between steps (256 MiB write, outside the step events)"},
            "route": route,
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                    "api": "qrb_geqrf_f32_host via gpumode_qr_b200.api.geqrf_host (pinned host in/out)",
                    "chunks": args.chunks,
                    "pcie": pcie},
            "gpu_launches": launches_total,
            "clocks": clk.summary(),
            "gates": ({"factor": gate.factor_residual, "orth": gate.orth_residual,
                       "passed": gate.passed} if gate is not None else None),
            "hooks": hooks,
            **extra,
        }
        print(json.dumps(line), flush=True)
    return 0


def main(argv=None) -> int:
    args = parse_args(argv)
    from gpumode_qr_b200 import sharding

    info = sharding.init_from_env()
    try:
        if args.impl == "reference":
            return run_reference(args, info)
        return run_ours(args, info)
    finally:
        sharding.destroy(info)


if __name__ == "__main__":
    raise SystemExit(main())
