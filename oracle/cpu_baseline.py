"""CPU baseline: the reference's PyTorch path for causal attention, timed on the host cores.

TEST / MEASUREMENT INFRASTRUCTURE ONLY (used by bench.py's cpu_baseline leg and by
`bench.py --impl reference`; never by the product).

It restates, with torch on the CPU, the reference's fp32 explicit attention
(attention/fused/reference.py:16-23 in the reference) and, for fwd+bwd, autograd through that
naive path (benchmarks/benchmark_backward.py:31-37, tests/backward/run_correctness_backward.py:
25-32); and torch's causal scaled_dot_product_attention, the reference benchmarks' SDPA path, on
the same cores.  The workload is a bounded sample (a few (batch, head) pairs of the configuration) so
that it finishes in seconds; throughput is reported with the same causal FLOP convention as the
GPU numbers: fwd = 2 * S^2 * D per head, fwd+bwd = 3.5x that.
"""
import math
import os
import time

import torch


def naive_attention(q, k, v):
    """fp32 explicit causal attention (autograd-capable)."""
    n, d = q.shape[-2], q.shape[-1]
    s = (q @ k.transpose(-1, -2)) / math.sqrt(d)
    mask = torch.ones(n, n, dtype=torch.bool).triu(1)
    return torch.softmax(s.masked_fill(mask, float("-inf")), dim=-1) @ v


def time_fwd_bwd(S, D, heads=1, reps=3, threads=None, seed=0):
    """Median wall time of fwd+bwd on `heads` heads of length S, dim D (fp32 on the CPU).
    Returns (seconds, flops_counted, threads_used)."""
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    q, k, v, do = (torch.randn(1, heads, S, D, generator=g) for _ in range(4))
    q.requires_grad_(True)
    k.requires_grad_(True)
    v.requires_grad_(True)
    times = []
    for _ in range(reps):
        q.grad = k.grad = v.grad = None
        t0 = time.perf_counter()
        naive_attention(q, k, v).backward(do)
        times.append(time.perf_counter() - t0)
    times.sort()
    flops = 3.5 * 2 * heads * S * S * D
    return times[len(times) // 2], flops, threads


def time_sdpa_fwd_bwd(S, D, heads=1, reps=3, threads=None, seed=0):
    """Median wall time of fwd+bwd through torch's scaled_dot_product_attention(is_causal=True) on
    the CPU in fp32 (the reference benchmarks' SDPA comparison path, benchmarks/
    benchmark_backward.py:44 in the reference, run on the host).  Returns (seconds, flops_counted,
    threads_used)."""
    import torch.nn.functional as F
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    q, k, v, do = (torch.randn(1, heads, S, D, generator=g) for _ in range(4))
    for t in (q, k, v):
        t.requires_grad_(True)
    times = []
    for _ in range(reps):
        q.grad = k.grad = v.grad = None
        t0 = time.perf_counter()
        F.scaled_dot_product_attention(q, k, v, is_causal=True).backward(do)
        times.append(time.perf_counter() - t0)
    times.sort()
    return times[len(times) // 2], 3.5 * 2 * heads * S * S * D, threads
