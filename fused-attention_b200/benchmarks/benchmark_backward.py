"""Forward + backward benchmark of the B200 kernels, in the reference's output schema.

Counterpart of the reference's `benchmarks/benchmark_backward.py`: same options, grid
(D in {64, 128} x N in {128, 512, 2048, 8192}, fp16, B x H = 2 x 8), measurements (median of
CUDA-event timings of forward only, backward only with an untimed forward before it, and
forward + backward; peak extra memory of one forward + backward) and CSV / Markdown layout.

  fused  attention.backward.fused_backward.fused_attention_autograd (sm_100a kernels)
  naive  eager PyTorch: S = Q K^T / sqrt(D) in fp16 matmuls, fp32 masked softmax, P V; autograd
         keeps the N x N probabilities (the usual unfused training baseline)
  sdpa   torch.nn.functional.scaled_dot_product_attention(is_causal=True)
TFLOP/s counts causal FLOPs of fwd + bwd = 3.5 x (2 B H N^2 D), recomputation not counted.

Run from the repository root:
    python fused-attention_b200/benchmarks/benchmark_backward.py --tile-m 64 --tile-n 128
Outputs: results/benchmarks/backward/bench_backward_<tile>.{csv,md}
"""
import argparse
import csv
import math
import os
import statistics
import sys

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from attention.backward.fused_backward import fused_attention_autograd  # noqa: E402


def naive_attention(q, k, v):
    n, d = q.shape[-2], q.shape[-1]
    s = (q @ k.transpose(-1, -2)).float() / math.sqrt(d)
    s = s.masked_fill(torch.ones(n, n, device=q.device, dtype=torch.bool).triu(1), float("-inf"))
    return torch.softmax(s, dim=-1).to(q.dtype) @ v


class Timings:
    """CUDA-event timings of one implementation on one input set (fresh leaf copies of q, k, v)."""

    def __init__(self, fn, q, k, v, do):
        self.fn, self.do = fn, do
        self.leaves = [t.detach().clone().requires_grad_(True) for t in (q, k, v)]

    def _zero_grads(self):
        for t in self.leaves:
            t.grad = None

    def _timed(self, body, setup=None):
        """Device ms of body(); setup() (untimed) runs first and its result is passed on."""
        arg = setup() if setup is not None else None
        if setup is not None:
            torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        body(arg)
        stop.record()
        stop.synchronize()
        return start.elapsed_time(stop)

    def step(self):
        self._zero_grads()
        self.fn(*self.leaves).backward(self.do)

    def forward_ms(self, reps):
        with torch.no_grad():
            return statistics.median(self._timed(lambda _: self.fn(*self.leaves)) for _ in range(reps))

    def backward_ms(self, reps):
        def setup():
            self._zero_grads()
            return self.fn(*self.leaves)
        return statistics.median(self._timed(lambda o: o.backward(self.do), setup) for _ in range(reps))

    def step_ms(self, reps):
        return statistics.median(self._timed(lambda _: self.step()) for _ in range(reps))

    def peak_extra_mb(self):
        """Peak device memory above the resident inputs while one forward + backward runs."""
        self._zero_grads()
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        resident = torch.cuda.memory_allocated()
        torch.cuda.reset_peak_memory_stats()
        self.step()
        torch.cuda.synchronize()
        return (torch.cuda.max_memory_allocated() - resident) / float(1 << 20)


def measure(fn, q, k, v, do, warmup, reps):
    """Median ms of forward, backward and forward + backward; peak extra MB of one fwd + bwd."""
    t = Timings(fn, q, k, v, do)
    for _ in range(warmup):
        t.step()
    torch.cuda.synchronize()
    return t.forward_ms(reps), t.backward_ms(reps), t.step_ms(reps), t.peak_extra_mb()


def _cell(value, spec):
    return "" if value is None else format(value, spec)


def _over(a, b):
    return a / b if a and b else None


# The three report tables: (heading, column names, cells of one (D, N) row given a lookup
# get(impl, key) -> value or None).  Speedups are other_ms / fused_ms (>1 = fused faster).
IMPLS3 = ("fused", "naive", "sdpa")
TABLES = [
    ("Forward + backward",
     ["D", "N", "fused ms", "naive ms", "SDPA ms", "vs naive", "vs SDPA", "fused TFLOP/s", "SDPA TFLOP/s"],
     lambda get: [_cell(get("fused", "fwd_bwd_ms"), ".3f"), _cell(get("naive", "fwd_bwd_ms"), ".3f") or "OOM",
                  _cell(get("sdpa", "fwd_bwd_ms"), ".3f"),
                  _cell(_over(get("naive", "fwd_bwd_ms"), get("fused", "fwd_bwd_ms")), ".2f"),
                  _cell(_over(get("sdpa", "fwd_bwd_ms"), get("fused", "fwd_bwd_ms")), ".2f"),
                  _cell(get("fused", "tflops"), ".1f"), _cell(get("sdpa", "tflops"), ".1f")]),
    ("Backward only",
     ["D", "N", "fused bwd ms", "naive bwd ms", "SDPA bwd ms", "vs naive", "vs SDPA", "fused bwd / fused fwd"],
     lambda get: [_cell(get(i, "bwd_ms"), ".3f") for i in IMPLS3]
                 + [_cell(_over(get("naive", "bwd_ms"), get("fused", "bwd_ms")), ".2f"),
                    _cell(_over(get("sdpa", "bwd_ms"), get("fused", "bwd_ms")), ".2f"),
                    _cell(_over(get("fused", "bwd_ms"), get("fused", "fwd_ms")), ".2f")]),
    ("Peak extra memory (MB)",
     ["D", "N", "fused", "naive", "SDPA", "naive / fused"],
     lambda get: [_cell(get(i, "peak_mem_mb"), ".1f") for i in IMPLS3]
                 + [_cell(_over(get("naive", "peak_mem_mb"), get("fused", "peak_mem_mb")), ".1f")]),
]


def markdown(rows, tile, gpu, B, H, reps):
    """The report in the reference's Markdown layout (same headings and columns)."""
    done = {(r["D"], r["N"], r["impl"]): r for r in rows if r["status"] == "ok"}
    configs = sorted({(r["D"], r["N"]) for r in rows})
    out = [f"# Backward benchmark (fused tile {tile})", "",
           f"GPU: {gpu}; B={B}, H={H}; FP16 inputs; causal. Median of {reps} runs.  ",
           "Speedup = other_ms / fused_ms (>1 = fused faster). Memory = peak extra GPU memory during fwd+bwd."]
    for heading, columns, cells in TABLES:
        out += ["", f"## {heading}", "", "| " + " | ".join(columns) + " |", "|" + "---|" * len(columns)]
        for D, N in configs:
            def get(impl, key, D=D, N=N):
                r = done.get((D, N, impl))
                return None if r is None else r[key]
            out.append("| " + " | ".join([str(D), str(N)] + cells(get)) + " |")
    return "\n".join(out) + "\n"


def csv_row(r, B, H, tm, tn, gpu):
    """One result dict as a CSV row: floats with four decimals, plus the run's constants."""
    row = {key: (f"{val:.4f}" if isinstance(val, float) else val) for key, val in r.items()}
    row.update(B=B, H=H, tile_m=tm, tile_n=tn, gpu=gpu)
    return row


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--B", type=int, default=2)
    p.add_argument("--H", type=int, default=8)
    p.add_argument("--tile-m", type=int, default=64)
    p.add_argument("--tile-n", type=int, default=64)
    p.add_argument("--Ds", default="64,128")
    p.add_argument("--Ns", default="128,512,2048,8192")
    p.add_argument("--impls", default="fused,naive,sdpa")
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--reps", type=int, default=20)
    p.add_argument("--out-dir", default="results/benchmarks/backward")
    a = p.parse_args()

    tm, tn = a.tile_m, a.tile_n
    impls = {
        "fused": lambda q, k, v: fused_attention_autograd(q, k, v, tm, tn),
        "naive": naive_attention,
        "sdpa": lambda q, k, v: F.scaled_dot_product_attention(q, k, v, is_causal=True),
    }
    gpu = torch.cuda.get_device_name()
    print(f"GPU: {gpu}  B={a.B} H={a.H}  fused tile {tm}x{tn}")
    rows = []
    for D in map(int, a.Ds.split(",")):
        for N in map(int, a.Ns.split(",")):
            torch.manual_seed(0)
            q, k, v, do = (torch.randn(a.B, a.H, N, D, device="cuda", dtype=torch.float16) for _ in range(4))
            total = 3.5 * 4 * a.B * a.H * N * N * D / 2
            for name in a.impls.split(","):
                if name == "fused" and (N % tm or N % tn):
                    continue
                try:
                    f_ms, b_ms, fb_ms, mem = measure(impls[name], q, k, v, do, a.warmup, a.reps)
                    tf = total / (fb_ms * 1e-3) / 1e12
                    print(f"{D:>4} {N:>5} {name:<6} | {f_ms:8.3f} {b_ms:8.3f} {fb_ms:8.3f} | {tf:7.2f} | {mem:9.1f}")
                    rows.append(dict(D=D, N=N, impl=name, fwd_ms=f_ms, bwd_ms=b_ms, fwd_bwd_ms=fb_ms,
                                     tflops=tf, peak_mem_mb=mem, status="ok"))
                except torch.cuda.OutOfMemoryError:
                    rows.append(dict(D=D, N=N, impl=name, status="OOM"))
                except Exception as e:
                    print(f"{D:>4} {N:>5} {name:<6} | FAILED: {type(e).__name__}: {e}")
                    rows.append(dict(D=D, N=N, impl=name, status=f"FAILED: {type(e).__name__}"))
                torch.cuda.empty_cache()
            del q, k, v, do
    os.makedirs(a.out_dir, exist_ok=True)
    tile = f"{tm}x{tn}"
    fields = ["D", "N", "B", "H", "impl", "tile_m", "tile_n", "fwd_ms", "bwd_ms", "fwd_bwd_ms", "tflops",
              "peak_mem_mb", "status", "gpu"]
    csv_path = os.path.join(a.out_dir, f"bench_backward_{tile}.csv")
    with open(csv_path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=fields)
        w.writeheader()
        w.writerows(csv_row(r, a.B, a.H, tm, tn, gpu) for r in rows)
    md_path = os.path.join(a.out_dir, f"bench_backward_{tile}.md")
    with open(md_path, "w") as f:
        f.write(markdown(rows, tile, gpu, a.B, a.H, a.reps))
    print(f"wrote {csv_path}\nwrote {md_path}")


if __name__ == "__main__":
    main()
