"""Forward benchmark of the B200 GQA/MQA kernel, in the reference's output schema.

Counterpart of the reference's `benchmarks/benchmark_forward_gqa.py`: one run per K/V head count,
the same options (--H-kv, --tile-m, --tile-n, --kernel, --tag, --impls, --out, --summary-out), the
same timing protocol as benchmark_forward.py (first call timed on its own, 10 warm-up calls,
median of 30 CUDA-event runs) and the same CSV columns (the MHA columns plus H_kv), so B200 rows
line up with the reference's `results/benchmarks/fused_gqa/...` files.  FLOPs are the MHA count
(they depend on H, not on H_kv).

  fused    attention.gqa.fused_gqa.fused_gqa_attention (sm_100a kernel; or any kernel file via --kernel)
  sdpa     torch.nn.functional.scaled_dot_product_attention(is_causal=True, enable_gqa=True)
  unfused  attention.gqa.unfused_gqa.unfused_gqa_attention, the reference's three-kernel GQA
           baseline (S and P materialised in global memory) as sm_100a kernels

--dtype bf16 and --Ds/--Ns/--B/--H cover BASELINE config 3 (B=4 H=32 S=8192 D=128 bf16):
    python fused-attention_b200/benchmarks/benchmark_forward_gqa.py --B 4 --H 32 --H-kv 2 \\
        --Ds 128 --Ns 8192 --dtype bf16 --tile-m 128 --tile-n 128
Run from the repository root.  Outputs:
results/benchmarks/fused_gqa/<tag>/<tile>/Hkv<H_kv>/bench_forward_gqa_{sep,agg}_<tag>_<tile>_Hkv<H_kv>.csv
(the reference also draws a PNG of the same numbers; matplotlib is not installed here).
"""
import argparse
import csv
import importlib.util
import os

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_KERNEL = os.path.join(os.path.dirname(HERE), "attention", "gqa", "fused_gqa.py")
DTYPES = {"fp16": torch.float16, "bf16": torch.bfloat16}


def _forward_bench():
    """benchmark_forward.py (timing, speedup and aggregate helpers), loaded by path."""
    spec = importlib.util.spec_from_file_location("_fa_b200_benchmark_forward",
                                                  os.path.join(HERE, "benchmark_forward.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


SEP_COLUMNS = ["D", "N", "B", "H", "impl", "tile_m", "tile_n", "median_ms", "tflops", "first_call_ms",
               "H_kv", "fused_speedup_vs_unfused", "fused_speedup_vs_sdpa", "gpu", "kernel", "kernel_tiles"]


def output_paths(tag, tile_m, tile_n, h_kv):
    tile = f"{tile_m}x{tile_n}"
    base = f"results/benchmarks/fused_gqa/{tag}/{tile}/Hkv{h_kv}"
    return (f"{base}/bench_forward_gqa_sep_{tag}_{tile}_Hkv{h_kv}.csv",
            f"{base}/bench_forward_gqa_agg_{tag}_{tile}_Hkv{h_kv}.csv")


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--kernel", default=DEFAULT_KERNEL, help="file that defines fused_gqa_attention")
    p.add_argument("--tag", default=None, help="name used in output paths (default: b200_<kernel file>)")
    p.add_argument("--B", type=int, default=2)
    p.add_argument("--H", type=int, default=8)
    p.add_argument("--H-kv", type=int, default=8, help="K/V heads (must divide --H)")
    p.add_argument("--tile-m", type=int, default=64)
    p.add_argument("--tile-n", type=int, default=64)
    p.add_argument("--impls", default="fused,unfused,sdpa")
    p.add_argument("--Ds", default="32,64,128")
    p.add_argument("--Ns", default="128,512,2048,8192")
    p.add_argument("--dtype", choices=sorted(DTYPES), default="fp16")
    p.add_argument("--out", default=None)
    p.add_argument("--summary-out", default=None)
    a = p.parse_args(argv)
    if a.H % a.H_kv != 0:
        p.error(f"--H-kv={a.H_kv} must divide --H={a.H}")

    fb = _forward_bench()
    fused = fb.load_kernel(a.kernel, "fused_gqa_attention")
    impls = {
        "fused": lambda q, k, v: fused(q, k, v, a.tile_m, a.tile_n),
        "unfused": lambda q, k, v: fb.unfused_attention(q, k, v, a.tile_m, a.tile_n),
        "sdpa": lambda q, k, v: F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True),
    }
    tag = a.tag or "b200_" + os.path.splitext(os.path.basename(a.kernel))[0]
    out, summary_out = output_paths(tag, a.tile_m, a.tile_n, a.H_kv)
    out, summary_out = a.out or out, a.summary_out or summary_out
    gpu = torch.cuda.get_device_name()
    dt = DTYPES[a.dtype]
    print(f"kernel={a.kernel}  tag={tag}  tile={a.tile_m}x{a.tile_n}  H_kv={a.H_kv}  dtype={a.dtype}  gpu={gpu}")

    torch.manual_seed(0)
    rows = []
    for D in map(int, a.Ds.split(",")):
        for N in map(int, a.Ns.split(",")):
            q = torch.randn(a.B, a.H, N, D, device="cuda", dtype=dt)
            k, v = (torch.randn(a.B, a.H_kv, N, D, device="cuda", dtype=dt) for _ in range(2))
            flops = 4 * a.B * a.H * N * N * D / 2  # two GEMMs of 2 N^2 D per query head, halved by the mask
            for name in a.impls.split(","):
                try:
                    ms, first_ms = fb.time_call(lambda: impls[name](q, k, v))
                    tf = flops / (ms * 1e-3) / 1e12
                    print(f"Hkv={a.H_kv} D={D:<4} N={N:<5} {name:<8} {ms:8.3f} ms  {tf:7.2f} TFLOP/s  "
                          f"(first call {first_ms:.0f} ms)")
                    rows.append([D, N, a.B, a.H, name, a.tile_m, a.tile_n, f"{ms:.4f}", f"{tf:.3f}",
                                 f"{first_ms:.1f}", a.H_kv])
                except Exception as e:  # recorded like the reference records a failed configuration
                    print(f"Hkv={a.H_kv} D={D:<4} N={N:<5} {name:<8} FAILED: {type(e).__name__}: {e}")
                    rows.append([D, N, a.B, a.H, name, a.tile_m, a.tile_n, "", "", "", a.H_kv])
            del q, k, v
            torch.cuda.empty_cache()
    fb.speedups(rows)
    for r in rows:
        r += [gpu, fb.kernel_label(a.kernel),
              fb.kernel_tiles(a.tile_n) if r[4] == "fused" and a.kernel == DEFAULT_KERNEL else ""]
    os.makedirs(os.path.dirname(out) or ".", exist_ok=True)
    with open(out, "w", newline="") as f:
        w = csv.writer(f)
        w.writerow(SEP_COLUMNS)
        w.writerows(rows)
    header, body = fb.summary_rows(rows)
    os.makedirs(os.path.dirname(summary_out) or ".", exist_ok=True)
    with open(summary_out, "w", newline="") as f:
        w = csv.writer(f)
        w.writerow(header)
        w.writerows(body)
    print(f"wrote {out}\nwrote {summary_out}")


if __name__ == "__main__":
    main()
