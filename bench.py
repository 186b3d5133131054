#!/usr/bin/env python
"""Benchmark of the B200 fused causal attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...           (N > 1, one rank per GPU)

Workload (default, BASELINE config 2 at the metric's point): causal MHA, B=4, H=32, S=8192,
D=128, fp16, Q/K/V/dO i.i.d. N(0,1) (synthetic, seeded).  One step = forward + backward through
the public autograd API (fused_attention_autograd: LSE-saving forward, delta, dK/dV, dQ kernels).
With N GPUs every rank owns the same per-GPU work (weak scaling: global batch 4N) through
attention.dist.sharded_attention_autograd, which all-gathers O and dQ/dK/dV over NCCL.
--workload c5: BASELINE config 5, causal GQA fwd+bwd, B=8, H=32, H_kv=8, D=128, bf16, S=32768
(--seq 8192 / 16384 for the other points), the same global job on every N (strong scaling).

value  = fwd+bwd causal TFLOP/s of the whole job (3.5 * 2 * B * H * S^2 * D per step, the
         reference's convention), device time, max over ranks, inputs resident in HBM.
e2e    = the same metric with pinned-host inputs copied in and O/dQ/dK/dV copied out every step
         (batch slices pipelined: copy-in, compute and copy-out of different slices overlap).
roofline: the dominant kernel, timed alone with CUDA events on its launch stream, in rounds
         interleaved with untimed steps (so the kernels run in the step loop's clock state).
cpu_baseline: the reference's PyTorch fp32 path on the host cores, on a bounded sample (plus
         torch's causal SDPA on the same sample).
--impl reference: the reference's CPU implementation (oracle port) timed the same way.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "fused-attention_b200")
for _p in (PKG, REPO):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "causal fwd & fwd+bwd TFLOP/s at S=8k,D=128 fp16; % of B200 tensor peak"
UNIT = "TFLOP/s"
SPEC_PEAK = 2250.0
FALLBACK_PEAK = 1590.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c2", "c5"], default="c2",
                    help="c2: B=4/GPU H=32 S=8192 D=128 fp16 MHA, weak scaling (the metric's point); "
                         "c5: B=8 H=32 H_kv=8 D=128 bf16 S=32768, strong scaling")
    ap.add_argument("--batch", type=int, default=None, help="per-GPU batch (c2) / global batch (c5)")
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=None, help="0 = MHA")
    ap.add_argument("--seq", type=int, default=None)
    ap.add_argument("--dim", type=int, default=128)
    ap.add_argument("--dtype", choices=["fp16", "bf16"], default=None)
    ap.add_argument("--tile-m", type=int, default=64)
    ap.add_argument("--tile-n", type=int, default=128)
    ap.add_argument("--e2e-steps", type=int, default=None, help="default: --steps")
    ap.add_argument("--e2e-slices", type=int, default=32,
                    help="pipeline slices per end-to-end step on one GPU (upper bound)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    a = ap.parse_args()
    c5 = a.workload == "c5"
    defaults = {"batch": 8 if c5 else 4, "kv_heads": 8 if c5 else 0, "seq": 32768 if c5 else 8192,
                "dtype": "bf16" if c5 else "fp16"}
    for key, val in defaults.items():
        if getattr(a, key) is None:
            setattr(a, key, val)
    a.strong = c5
    if a.e2e_steps is None:
        a.e2e_steps = a.steps
    return a


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d.get("hbm_gbs", 0)) or None, "measured"
    except (OSError, ValueError, KeyError):
        return FALLBACK_PEAK, 6650.0, "fallback"


def load_sustained_peak():
    """cuBLAS bf16 TFLOP/s back to back for seconds under the power cap (MEASURED_PEAKS.json)."""
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops_sustained"])
    except (OSError, ValueError, KeyError):
        return None


def load_traffic():
    """Per-launch DRAM bytes of each kernel from the committed ncu summary (or None)."""
    path = os.path.join(REPO, "profiles", "traffic.txt")
    out = {}
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 3 and not line.startswith("#"):
                out[(parts[0], parts[1])] = float(parts[2])
    except OSError:
        pass
    return out


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.dev)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for name, flag in zip(names, parts[3:7]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# Longest sequence the CPU sample runs: the explicit path keeps S x S fp32 matrices for autograd
# (4 GiB each at S=32768), so longer configurations are sampled at this length.
CPU_SAMPLE_MAX_S = 8192


def cpu_baseline_sample(S, D, reps=3):
    from oracle.cpu_baseline import time_fwd_bwd, time_sdpa_fwd_bwd
    Ss = min(S, CPU_SAMPLE_MAX_S)
    secs, flops, threads = time_fwd_bwd(Ss, D, heads=1, reps=reps)
    time_sdpa_fwd_bwd(min(Ss, 1024), D, heads=1, reps=1)  # first call: one-time set-up, untimed
    s_secs, s_flops, _ = time_sdpa_fwd_bwd(Ss, D, heads=1, reps=reps)
    note = "" if Ss == S else f" (the workload's S={S} sampled at S={Ss})"
    return {"value": flops / secs / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"1 (batch, head) pair of the workload (S={Ss}, D={D}){note}, fp32 fwd+bwd through "
                      f"torch autograd of the explicit reference path, median of {reps}",
            "sdpa": {"value": s_flops / s_secs / 1e12, "unit": UNIT, "cores": threads,
                     "sample": f"the same (batch, head) pair through torch.nn.functional."
                               f"scaled_dot_product_attention(is_causal=True), fp32 fwd+bwd, median of {reps}"}}


def run_reference_arm(a, rank):
    """--impl reference: the reference's CPU implementation on the host cores, rank 0 only."""
    if rank != 0:
        return
    from oracle.cpu_baseline import time_fwd_bwd
    S, D = min(a.seq, CPU_SAMPLE_MAX_S), a.dim
    for _ in range(a.warmup):
        time_fwd_bwd(S, D, heads=1, reps=1)
    times = []
    flops = None
    threads = None
    for _ in range(a.steps):
        t, flops, threads = time_fwd_bwd(S, D, heads=1, reps=1)
        times.append(t)
    total = sum(times)
    value = flops * a.steps / total / 1e12
    sample = (f"per step: 1 (batch, head) pair of B={a.batch} H={a.heads} S={a.seq} D={D}"
              + ("" if S == a.seq else f" sampled at S={S}")
              + ", fp32 fwd+bwd via torch autograd of the reference's explicit path on the CPU")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1000 * total / a.steps,
            "higher_is_better": True, "scaling": "strong" if a.strong else "weak", "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic", "config": workload_config(a, 1),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def e2e_slices(B, H, H_kv, world, max_slices):
    """The end-to-end leg's pipeline slices: [(q/o/dq/do index, k/v/dk/dv index)], each a pair of
    (batch slice, head slice).  A slice is `world` batch entries; on one GPU each batch entry is
    also cut into 2^k runs of whole K/V-head groups (query heads [g*grp, (g+1)*grp) go with K/V
    head g), as many as keep the step at or under `max_slices` slices."""
    bs = world
    hsplit = 1
    if world == 1:
        while hsplit * 2 * (B // bs) <= max_slices and H_kv % (hsplit * 2) == 0:
            hsplit *= 2
    kvh = H_kv // hsplit
    qh = kvh * (H // H_kv)
    return [((slice(c * bs, (c + 1) * bs), slice(p * qh, (p + 1) * qh)),
             (slice(c * bs, (c + 1) * bs), slice(p * kvh, (p + 1) * kvh)))
            for c in range(B // bs) for p in range(hsplit)]


def workload_config(a, world):
    kind = "GQA" if a.kv_heads and a.kv_heads != a.heads else "MHA"
    if a.strong:
        name = (f"BASELINE config 5: causal {kind} fwd+bwd, B={a.batch} (global) H={a.heads} "
                f"H_kv={a.kv_heads or a.heads} S={a.seq} D={a.dim} {a.dtype}")
        global_b, per_gpu = a.batch, a.batch / world
    else:
        name = (f"causal {kind} fwd+bwd, B={a.batch}/GPU H={a.heads} H_kv={a.kv_heads or a.heads} "
                f"S={a.seq} D={a.dim} {a.dtype}")
        global_b, per_gpu = a.batch * world, a.batch
    return {"workload": name, "global_batch": global_b, "per_gpu_batch": per_gpu, "heads": a.heads,
            "kv_heads": a.kv_heads or a.heads, "seq_len": a.seq, "head_dim": a.dim,
            "tiles": f"{a.tile_m}x{a.tile_n} (kernel: 128-row query tiles, {64 if a.tile_n <= 64 else 128}-key K/V tiles)",
            "parallelism": f"(batch, K/V head) shards over {world} GPU(s)",
            "l2": "inputs larger than L2 (4 x B*H*S*D*2 bytes per step vs 126 MB)"}


def main():
    a = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        run_reference_arm(a, rank)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        # NCCL's blocks must get SMs while the attention kernels are queued, or the gathers of
        # one chunk cannot overlap the kernels of the next
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = True
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev, pg_options=opts)
        group = dist.group.WORLD

    from attention.backward.fused_backward import fused_attention_autograd, _forward, _native
    from attention.dist import plan_chunks, sharded_attention_autograd

    dt = torch.float16 if a.dtype == "fp16" else torch.bfloat16
    B = a.batch if a.strong else a.batch * world
    H, S, D = a.heads, a.seq, a.dim
    H_kv = a.kv_heads or H
    g = torch.Generator(device=dev).manual_seed(1234)
    q = torch.randn(B, H, S, D, device=dev, generator=g, dtype=torch.float32).to(dt).requires_grad_(True)
    k = torch.randn(B, H_kv, S, D, device=dev, generator=g, dtype=torch.float32).to(dt).requires_grad_(True)
    v = torch.randn(B, H_kv, S, D, device=dev, generator=g, dtype=torch.float32).to(dt).requires_grad_(True)
    do = torch.randn(B, H, S, D, device=dev, generator=g, dtype=torch.float32).to(dt)
    nat = _native()

    def attn(q_, k_, v_):
        if world > 1:
            return sharded_attention_autograd(q_, k_, v_, a.tile_m, a.tile_n, group)
        return fused_attention_autograd(q_, k_, v_, a.tile_m, a.tile_n)

    def step():
        q.grad = k.grad = v.grad = None
        attn(q, k, v).backward(do)

    def fwd_only():
        with torch.no_grad():
            attn(q, k, v)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, iters):
        barrier()
        torch.cuda.synchronize()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(s.elapsed_time(e))

    launch_chunks = plan_chunks(B * H_kv, world) if world > 1 else 1
    flops_fwd = 2.0 * B * H * S * S * D
    flops_step = 3.5 * flops_fwd

    # clocks are sampled from before the warm-up until the timed region ends (nvidia-smi needs a
    # few hundred ms to start; the timed region alone can be shorter than that)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.5)
    for _ in range(a.warmup):
        step()
    nat.check_status(dev)
    ms = timed(step, a.steps)
    clocks = sampler.stop()
    nat.check_status(dev)
    value = flops_step * a.steps / (ms / 1e3) / 1e12

    for _ in range(a.warmup):
        fwd_only()
    ms_fwd = timed(fwd_only, a.steps)
    fwd_tflops = flops_fwd * a.steps / (ms_fwd / 1e3) / 1e12

    # ---- per-kernel device times (this rank's shard, each kernel timed alone on its stream)
    units = B * H_kv // world
    grp = H // H_kv
    qs = q.detach().view(B * H_kv, grp, S, D)[:units]
    ks = k.detach().view(B * H_kv, 1, S, D)[:units]
    vs = v.detach().view(B * H_kv, 1, S, D)[:units]
    dos = do.view(B * H_kv, grp, S, D)[:units]
    o_s, lse_s = _forward(qs, ks, vs, a.tile_m, a.tile_n)
    delta = torch.empty_like(lse_s)
    dq_s, dk_s, dv_s = torch.empty_like(qs), torch.empty_like(ks), torch.empty_like(vs)
    kern = {
        "fwd": (lambda: nat.fwd(qs, ks, vs, o_s, lse_s, a.tile_m, a.tile_n), 2.0),
        "bwd_preprocess": (lambda: nat.bwd_preprocess(o_s, dos, delta), 0.0),
        "bwd_dkdv": (lambda: nat.bwd_dkdv(qs, ks, vs, dos, lse_s, delta, dk_s, dv_s, a.tile_m, a.tile_n), 4.0),
        "bwd_dq": (lambda: nat.bwd_dq(qs, ks, vs, dos, lse_s, delta, dq_s, a.tile_m, a.tile_n), 3.0),
    }
    # Each round runs one untimed step (which keeps the GPU in the step loop's clock and power
    # state) and then times every kernel once; a kernel's time is its median over the rounds.
    for fn, _ in kern.values():
        fn()
    samples = {name: [] for name in kern}
    for _ in range(max(3, min(10, a.steps))):
        step()
        for name, (fn, _) in kern.items():
            samples[name].append(timed(fn, 1))
    kt = {name: statistics.median(v) for name, v in samples.items()}
    nat.check_status(dev)
    shard_unit_flops = units * grp * S * S * D  # one causal S x S x D GEMM over the shard
    dominant = max(kt, key=kt.get)
    peak, hbm_peak, peak_kind = load_peaks()
    dom_flops = kern[dominant][1] * shard_unit_flops
    achieved = dom_flops / (kt[dominant] / 1e3) / 1e12
    traffic = load_traffic().get((dominant, f"S{S}_D{D}"))
    sustained = load_sustained_peak()
    roofline = {"bound": "tensor", "kernel": dominant, "achieved": achieved, "peak": peak, "unit": UNIT,
                "frac": achieved / peak, "peak_kind": peak_kind, "traffic": traffic,
                # the power-capped cuBLAS figure: what a tensor-bound kernel inside a long step meets
                "peak_sustained": sustained, "frac_sustained": (achieved / sustained) if sustained else None,
                "algorithmic_flops_per_launch": dom_flops, "launch_ms": kt[dominant],
                "kernels_ms": kt,
                "kernels_tflops": {n: (kern[n][1] * shard_unit_flops / (kt[n] / 1e3) / 1e12) if kern[n][1] else None
                                   for n in kt}}

    # ---- end to end through the public API with pinned host buffers
    hq, hk, hv, hdo = (t.detach().cpu().pin_memory() for t in (q, k, v, do))
    ho = torch.empty(q.shape, dtype=dt).pin_memory()
    hdq = torch.empty(q.shape, dtype=dt).pin_memory()
    hdk = torch.empty(k.shape, dtype=dt).pin_memory()
    hdv = torch.empty(v.shape, dtype=dt).pin_memory()

    # The host-resident job streams through the public API one slice at a time (attention is
    # independent per batch entry and per K/V head with its query-head group): slice c+1 copies in
    # on one stream while slice c computes and slice c-1 copies out on another (PCIe is full
    # duplex).  Every byte of Q, K, V, dO goes in and every byte of O, dQ, dK, dV comes out inside
    # the timed region.  A slice is `world` batch entries, so with N GPUs each rank still gets a
    # full share of every call; on one GPU each batch entry is also cut into runs of whole K/V-head
    # groups (contiguous in every tensor), up to --e2e-slices slices per step: small slices shorten
    # the copy-in of the first slice and the copy-out of the last, the parts no compute can hide
    # (the PCIe copies, not the kernels, bound this leg).
    h2d_stream = torch.cuda.Stream(device=dev)
    d2h_stream = torch.cuda.Stream(device=dev)
    comp = torch.cuda.current_stream(dev)
    slices = e2e_slices(B, H, H_kv, world, a.e2e_slices)
    nslices = len(slices)

    def e2e_step():
        h2d_stream.wait_stream(comp)
        ins = []
        for slq, slk in slices:
            with torch.cuda.stream(h2d_stream):
                tens = [hq[slq].to(dev, non_blocking=True), hk[slk].to(dev, non_blocking=True),
                        hv[slk].to(dev, non_blocking=True), hdo[slq].to(dev, non_blocking=True)]
                ready = torch.cuda.Event()
                ready.record(h2d_stream)
            ins.append((slq, slk, tens, ready))
        keep = []
        for slq, slk, (tq, tk, tv, tdo), ready in ins:
            comp.wait_event(ready)
            q_, k_, v_ = (t.requires_grad_(True) for t in (tq, tk, tv))
            o = attn(q_, k_, v_)
            o.backward(tdo)
            done = torch.cuda.Event()
            done.record(comp)
            with torch.cuda.stream(d2h_stream):
                d2h_stream.wait_event(done)
                ho[slq].copy_(o.detach(), non_blocking=True)
                hdq[slq].copy_(q_.grad, non_blocking=True)
                hdk[slk].copy_(k_.grad, non_blocking=True)
                hdv[slk].copy_(v_.grad, non_blocking=True)
            keep.append((tq, tk, tv, tdo, o))  # no buffer is reused before the copies end
        comp.wait_stream(d2h_stream)

    e2e_step()
    ms_e2e = timed(e2e_step, a.e2e_steps)
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hdo))
    d2h = sum(t.numel() * t.element_size() for t in (ho, hdq, hdk, hdv))
    e2e = {"value": flops_step * a.e2e_steps / (ms_e2e / 1e3) / 1e12, "unit": UNIT,
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": a.e2e_steps,
           "slices_per_step": nslices,
           "ms_per_step": ms_e2e / a.e2e_steps}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline_sample(S, D)

    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": ms / a.steps, "higher_is_better": True,
                "scaling": "strong" if a.strong else "weak", "vs_baseline": None,
                "dtype": "f16" if a.dtype == "fp16" else "bf16",
                "data": "synthetic (i.i.d. N(0,1), seeded)", "config": workload_config(a, world),
                "fwd_tflops": fwd_tflops, "fwd_ms_per_step": ms_fwd / a.steps,
                "frac_of_spec_peak": {"fwd+bwd": value / (SPEC_PEAK * world), "fwd": fwd_tflops / (SPEC_PEAK * world)},
                "frac_of_measured_peak": {"fwd+bwd": value / (peak * world), "fwd": fwd_tflops / (peak * world),
                                          "peak_kind": peak_kind},
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks,
                # per step: forward, delta, dK/dV and dQ kernels, once per chunk of this rank's units
                "gpu_launches": 4 * launch_chunks * a.steps}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
