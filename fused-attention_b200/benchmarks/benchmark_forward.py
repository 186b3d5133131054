"""Forward benchmark (MHA) of the B200 kernels, in the reference's output schema.

Counterpart of the reference's `benchmarks/benchmark_forward.py`: the same command-line options,
configuration grid (D in {64, 128} x N in {128, 512, 2048, 8192}, fp16, B x H = 2 x 8 by default),
timing protocol (first call timed on its own, 10 warm-up calls, median of 30 CUDA-event runs) and
CSV columns, so B200 rows line up with the reference's `results/benchmarks/fused/...` files.

  fused    attention.fused.fused.fused_attention (sm_100a kernel; or any kernel file via --kernel)
  sdpa     torch.nn.functional.scaled_dot_product_attention(is_causal=True)
  unfused  attention.fused.unfused.unfused_attention, the reference's three-kernel baseline (S and
           P materialised in global memory) as sm_100a kernels

Run from the repository root:
    python fused-attention_b200/benchmarks/benchmark_forward.py --tile-m 64 --tile-n 128
Outputs: results/benchmarks/fused/<tag>/<tile>/bench_forward_{sep,agg}_<tag>_<tile>.csv
The per-configuration CSV has the reference's columns plus `kernel_tiles`, the tile shape the
sm_100a kernel ran (`q128_kv64` or `q128_kv128`; empty for other implementations): the kernel's
query tile is always 128 rows, so tile_m is not a kernel parameter here.
"""
import argparse
import csv
import importlib.util
import os
import re
import statistics
import time

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
DEFAULT_KERNEL = os.path.join(os.path.dirname(HERE), "attention", "fused", "fused.py")


def kernel_label(path):
    """The kernel file as written into the CSVs: relative to the repository root when inside it."""
    full = os.path.abspath(path)
    return os.path.relpath(full, REPO) if full.startswith(REPO + os.sep) else os.path.basename(full)


def kernel_tiles(tile_n):
    """Tile shape the sm_100a forward runs for the reference's (tile_m, tile_n) knobs: 128 query
    rows always (tile_m only takes part in the divisibility rule), 64 or 128 keys per K/V tile."""
    return f"q128_kv{64 if tile_n <= 64 else 128}"


def load_kernel(path, name="fused_attention"):
    """Import `name` from a kernel file by path (the reference's runners do the same)."""
    mod_name = "kernel_" + re.sub(r"\W", "_", os.path.splitext(os.path.basename(path))[0])
    spec = importlib.util.spec_from_file_location(mod_name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return getattr(mod, name)


UNFUSED = os.path.join(os.path.dirname(HERE), "attention", "fused", "unfused.py")


UNFUSED_GQA = os.path.join(os.path.dirname(HERE), "attention", "gqa", "unfused_gqa.py")
_loaded = {}


def unfused_attention(q, k, v, tm, tn):
    """The unfused baseline: unfused_attention for MHA, unfused_gqa_attention when K/V have fewer
    heads (both run the same three kernels)."""
    key = (UNFUSED, "unfused_attention") if k.shape == q.shape else (UNFUSED_GQA, "unfused_gqa_attention")
    if key not in _loaded:
        _loaded[key] = load_kernel(*key)
    return _loaded[key](q, k, v, tm, tn)


def time_call(fn, warmup=10, reps=30):
    """(median ms of `reps` CUDA-event timed calls, ms of the first call) for fn()."""
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    fn()
    torch.cuda.synchronize()
    first_ms = (time.perf_counter() - t0) * 1e3
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    return statistics.median(times), first_ms


def speedups(rows):
    """Append fused_speedup_vs_unfused / _vs_sdpa (other_ms / fused_ms) to each fused row."""
    lat = {(r[0], r[1], r[4]): float(r[7]) for r in rows if r[7] != ""}
    for r in rows:
        fused_ms = lat.get((r[0], r[1], "fused")) if r[4] == "fused" else None
        for other in ("unfused", "sdpa"):
            o = lat.get((r[0], r[1], other))
            r.append(f"{o / fused_ms:.3f}" if fused_ms and o else "")


def summary_rows(rows):
    """Mean latency / throughput per N, per D and overall for every impl, plus the geometric mean
    of per-configuration fused speedups (the reference's aggregate table)."""
    ok = [(r[0], r[1], r[4], float(r[7]), float(r[8])) for r in rows if r[7] != ""]
    impls = list(dict.fromkeys(r[4] for r in rows))

    def one(scope, value, sub):
        out = [scope, value]
        for name in impls:
            ms = [x[3] for x in sub if x[2] == name]
            tf = [x[4] for x in sub if x[2] == name]
            out += [f"{statistics.mean(ms):.4f}" if ms else "", f"{statistics.mean(tf):.3f}" if tf else ""]
        lat = {(x[0], x[1], x[2]): x[3] for x in sub}
        for other in ("unfused", "sdpa"):
            ratios = [lat[(d, n, other)] / ms for (d, n, name), ms in lat.items()
                      if name == "fused" and (d, n, other) in lat]
            out.append(f"{statistics.geometric_mean(ratios):.2f}" if ratios else "")
        return out

    body = [one("N", n, [x for x in ok if x[1] == n]) for n in sorted({x[1] for x in ok})]
    body += [one("D", d, [x for x in ok if x[0] == d]) for d in sorted({x[0] for x in ok})]
    body.append(one("all", "all", ok))
    header = (["scope", "value"] + [f"{name}_{m}" for name in impls for m in ("avg_median_ms", "avg_tflops")]
              + ["fused_speedup_vs_unfused", "fused_speedup_vs_sdpa"])
    return header, body


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--kernel", default=DEFAULT_KERNEL, help="file that defines fused_attention")
    p.add_argument("--tag", default=None, help="name used in output paths (default: b200_<kernel file>)")
    p.add_argument("--B", type=int, default=2)
    p.add_argument("--H", type=int, default=8)
    p.add_argument("--tile-m", type=int, default=64)
    p.add_argument("--tile-n", type=int, default=64)
    p.add_argument("--impls", default="fused,unfused,sdpa")
    p.add_argument("--Ds", default="64,128")
    p.add_argument("--Ns", default="128,512,2048,8192")
    p.add_argument("--out", default=None)
    p.add_argument("--summary-out", default=None)
    a = p.parse_args()

    fused = load_kernel(a.kernel)
    impls = {
        "fused": lambda q, k, v: fused(q, k, v, a.tile_m, a.tile_n),
        "unfused": lambda q, k, v: unfused_attention(q, k, v, a.tile_m, a.tile_n),
        "sdpa": lambda q, k, v: F.scaled_dot_product_attention(q, k, v, is_causal=True),
    }
    tag = a.tag or "b200_" + os.path.splitext(os.path.basename(a.kernel))[0]
    tile = f"{a.tile_m}x{a.tile_n}"
    base = f"results/benchmarks/fused/{tag}/{tile}"
    out = a.out or f"{base}/bench_forward_sep_{tag}_{tile}.csv"
    summary_out = a.summary_out or f"{base}/bench_forward_agg_{tag}_{tile}.csv"
    gpu = torch.cuda.get_device_name()
    print(f"kernel={a.kernel}  tag={tag}  tile={tile}  gpu={gpu}")

    torch.manual_seed(0)
    rows = []
    for D in map(int, a.Ds.split(",")):
        for N in map(int, a.Ns.split(",")):
            q, k, v = (torch.randn(a.B, a.H, N, D, device="cuda", dtype=torch.float16) for _ in range(3))
            flops = 4 * a.B * a.H * N * N * D / 2  # two GEMMs of 2 N^2 D, halved by the causal mask
            for name in a.impls.split(","):
                try:
                    ms, first_ms = time_call(lambda: impls[name](q, k, v))
                    tf = flops / (ms * 1e-3) / 1e12
                    print(f"D={D:<4} N={N:<5} {name:<8} {ms:8.3f} ms  {tf:7.2f} TFLOP/s  (first call {first_ms:.0f} ms)")
                    rows.append([D, N, a.B, a.H, name, a.tile_m, a.tile_n, f"{ms:.4f}", f"{tf:.3f}", f"{first_ms:.1f}"])
                except Exception as e:  # recorded like the reference records a failed configuration
                    print(f"D={D:<4} N={N:<5} {name:<8} FAILED: {type(e).__name__}: {e}")
                    rows.append([D, N, a.B, a.H, name, a.tile_m, a.tile_n, "", "", ""])
            del q, k, v
            torch.cuda.empty_cache()
    speedups(rows)
    label = kernel_label(a.kernel)
    for r in rows:
        r += [gpu, label, kernel_tiles(a.tile_n) if r[4] == "fused" and a.kernel == DEFAULT_KERNEL else ""]
    os.makedirs(os.path.dirname(out) or ".", exist_ok=True)
    with open(out, "w", newline="") as f:
        w = csv.writer(f)
        w.writerow(["D", "N", "B", "H", "impl", "tile_m", "tile_n", "median_ms", "tflops", "first_call_ms",
                    "fused_speedup_vs_unfused", "fused_speedup_vs_sdpa", "gpu", "kernel", "kernel_tiles"])
        w.writerows(rows)
    header, body = summary_rows(rows)
    os.makedirs(os.path.dirname(summary_out) or ".", exist_ok=True)
    with open(summary_out, "w", newline="") as f:
        w = csv.writer(f)
        w.writerow(header)
        w.writerows(body)
    print(f"wrote {out}\nwrote {summary_out}")


if __name__ == "__main__":
    main()
