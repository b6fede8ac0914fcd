"""Grid sweep over (batch, n) with a regime report.

Mirrors the reference's grid search (scripts/run_grid_search.py:34-36 grid,
:79-119 per point, :122-160 summary): every point is a column-scaled dense
problem with cond = 1 (src/qrbench/inputs.py:52-60, restated in
``inputs.make_benchmark_problem``), gated with the FP64 checker, then timed for
this library's ``impl`` and for the library baseline ``torch.geqrf`` on the
same GPU (cuSOLVER). Each point also records its regime: the path that runs
(the fused warp kernel for n <= 32, the fused CTA kernel for 32 < n <= 128 at the
sizes it is dispatched for, or the blocked panel / trailing-update route), the
bound (HBM traffic 2 b n^2 4 bytes against the measured copy bandwidth, or
(4/3) n^3 b FLOPs against the FP32 FFMA peak, whichever takes longer) and the
achieved fraction of that roofline.

    python -m gpumode_qr_b200.grid --out grid.json [--batches 2 8 --ns 32 64]
"""

from __future__ import annotations

import argparse
import json
import math
import statistics
import sys
import time
from pathlib import Path

GRID_BATCH = [2, 4, 8, 16, 32, 64, 128, 256]
GRID_N = [32, 64, 128, 256, 512, 1024, 2048, 4096]
FP32_FFMA_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # nominal: SMs x FMA lanes x 2 x max clock
L2_FLUSH_BYTES = 256 << 20


def _peaks() -> dict:
    p = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d.get("hbm_gbs")), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def regime(batch: int, n: int, ms: float, peaks: dict) -> dict:
    nbytes = 2 * batch * n * n * 4
    flops = 4.0 / 3.0 * n**3 * batch
    t_hbm = nbytes / (peaks["hbm_gbs"] * 1e9)
    t_flop = flops / (FP32_FFMA_TFLOPS * 1e12)
    bound = "hbm" if t_hbm >= t_flop else "flop"
    floor_ms = max(t_hbm, t_flop) * 1e3
    return {
        "path": ("fused" if n <= 32 else
                 "fused_cta" if n <= 128 and (n <= 64 or n > 96 or batch <= 592) else
                 "blocked"),
        "bound": bound,
        "floor_ms": floor_ms,
        "roofline_frac": floor_ms / ms if ms > 0 else None,
        "achieved": (nbytes / (ms / 1e3) / 1e9) if bound == "hbm" else (flops / (ms / 1e3) / 1e12),
        "achieved_unit": "GB/s" if bound == "hbm" else "TFLOP/s",
    }


def _time_device(fn, warmup: int, iters: int, flush) -> list[float]:
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(iters):
        flush.fill_(1)
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        out.append((s, e))
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in out]


def benchmark_point(batch: int, n: int, warmup: int, iters: int, torch_budget_s: float,
                    gate: bool, flush, peaks: dict) -> dict:
    import torch

    from . import api, checker, inputs

    prob = inputs.make_benchmark_problem({"batch": batch, "n": n, "cond": 1})
    A = prob.tensor.to("cuda")
    H, tau = api.impl(A)
    torch.cuda.synchronize()
    row = {"shape": {"batch": batch, "n": n, "cond": 1}, "name": prob.name}
    if gate:
        row["correctness"] = checker.check(A, H, tau).as_dict()
    del H, tau
    # our path: fewer iterations for long points
    t0 = time.perf_counter()
    api.impl(A)
    torch.cuda.synchronize()
    one = time.perf_counter() - t0
    its = max(3, min(iters, int(2.0 / max(one, 1e-6))))
    ours = _time_device(lambda: api.impl(A), min(warmup, its), its, flush)
    ms = statistics.median(ours)
    row["b200_geqrf"] = {"median_ms": ms, "iters": its, "matrices_per_s": batch / (ms / 1e3)}
    row["regime"] = regime(batch, n, ms, peaks)
    # library baseline on the same GPU, bounded in time
    if torch_budget_s > 0:
        t0 = time.perf_counter()
        torch.geqrf(A)
        torch.cuda.synchronize()
        one = time.perf_counter() - t0
        if one * 3 <= torch_budget_s:
            its_t = max(1, min(iters, int(torch_budget_s / max(one, 1e-6)) - 1))
            tt = _time_device(lambda: torch.geqrf(A), 1, its_t, flush)
            tms = statistics.median(tt)
        else:
            tms, its_t = one * 1e3, 1
        row["torch_geqrf_cuda"] = {"median_ms": tms, "iters": its_t}
        row["speedup_vs_torch_cuda"] = tms / ms
    return row


def summarize(rows: list[dict]) -> dict:
    sp = [r["speedup_vs_torch_cuda"] for r in rows if "speedup_vs_torch_cuda" in r]
    fr = [r["regime"]["roofline_frac"] for r in rows]
    fails = [r["name"] for r in rows if "correctness" in r and not r["correctness"]["passed"]]
    out = {
        "n_points": len(rows),
        "gate_failures": fails,
        "roofline_frac": {"min": min(fr), "max": max(fr),
                          "geomean": math.exp(sum(math.log(x) for x in fr) / len(fr))},
    }
    if sp:
        out["speedup_vs_torch_cuda"] = {
            "min": min(sp), "max": max(sp),
            "geomean": math.exp(sum(math.log(x) for x in sp) / len(sp)),
        }
    return out


def markdown(rows: list[dict]) -> str:
    ns = sorted({r["shape"]["n"] for r in rows})
    bs = sorted({r["shape"]["batch"] for r in rows})
    by = {(r["shape"]["batch"], r["shape"]["n"]): r for r in rows}
    lines = ["| batch \\ n | " + " | ".join(str(n) for n in ns) + " |",
             "|---" * (len(ns) + 1) + "|"]
    for b in bs:
        cells = []
        for n in ns:
            r = by.get((b, n))
            if r is None:
                cells.append("")
                continue
            ms = r["b200_geqrf"]["median_ms"]
            frac = r["regime"]["roofline_frac"]
            sp = r.get("speedup_vs_torch_cuda")
            cells.append(f"{ms:.3g} ms, {100 * frac:.0f}% {r['regime']['bound']}"
                         + (f", {sp:.0f}x" if sp is not None else ""))
        lines.append(f"| {b} | " + " | ".join(cells) + " |")
    return "\n".join(lines)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--batches", type=int, nargs="*", default=GRID_BATCH)
    ap.add_argument("--ns", type=int, nargs="*", default=GRID_N)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--torch-budget-s", type=float, default=3.0,
                    help="seconds of torch.geqrf timing per point (0 = skip the library baseline)")
    ap.add_argument("--no-gate", action="store_true")
    ap.add_argument("--out", default=None, help="write the rows and summary as JSON here")
    args = ap.parse_args(argv)

    import torch

    if not torch.cuda.is_available():
        print("grid: a CUDA device is required", file=sys.stderr)
        return 2
    peaks = _peaks()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    rows = []
    for b in args.batches:
        for n in args.ns:
            r = benchmark_point(b, n, args.warmup, args.iters, args.torch_budget_s,
                                not args.no_gate, flush, peaks)
            rows.append(r)
            g = r.get("correctness", {}).get("passed")
            print(f"[grid] {r['name']:>18} gate={'-' if g is None else ('PASS' if g else 'FAIL')} "
                  f"ours={r['b200_geqrf']['median_ms']:.4g}ms "
                  f"frac={r['regime']['roofline_frac']:.3f} ({r['regime']['bound']}) "
                  f"torch={r.get('torch_geqrf_cuda', {}).get('median_ms', float('nan')):.4g}ms",
                  flush=True)
            torch.cuda.empty_cache()
    summary = summarize(rows)
    doc = {"peaks": peaks, "fp32_ffma_tflops_nominal": FP32_FFMA_TFLOPS, "rows": rows,
           "summary": summary, "device": torch.cuda.get_device_name(0)}
    if args.out:
        Path(args.out).write_text(json.dumps(doc, indent=1))
    print(json.dumps(summary))
    print(markdown(rows))
    return 1 if summary["gate_failures"] else 0


if __name__ == "__main__":
    raise SystemExit(main())
