"""Correctness records of the B200 kernels in the reference's CSV schemas.

    python tests/runners/run_correctness.py --suite fused [--tile-m 64 --tile-n 64] [--filter N512]
    python tests/runners/run_correctness.py --suite gqa
    python tests/runners/run_correctness.py --suite backward

For every case of the reference's grids (its 84 MHA and 96 GQA forward cases with their crc32
seeds, and its 7 backward cases with their CUDA-generator inputs), run the drop-in function
(`fused_attention`, `fused_gqa_attention`, `fused_attention_autograd`; with `--impl unfused` the
three-kernel baseline `unfused_attention` / `unfused_gqa_attention`), compare it with the fp32
PyTorch ground truth computed on the same device, and write one CSV row per case with the
reference's columns:

  fused:    results/correctness/fused/b200/<tile>/correctness_fused_b200_<tile>.csv
  gqa:      results/correctness/fused_gqa/b200/<tile>/correctness_fused_gqa_b200_<tile>.csv
  backward: results/correctness/backward/backward_b200_<tile>.csv

so each case's error sits next to the reference's own record for its cuTile kernels.  Forward
rule: PASS if the output is finite and |out - ref| <= 2e-2 + 2e-2 |ref| everywhere (tol_ratio is
the largest |out - ref| / (2e-2 + 2e-2 |ref|)); backward rule: relative Frobenius error of O, dQ,
dK, dV each <= 2e-2.  `--impl reference` runs the fp32 ground truth through the same harness (a
self-check of the harness, also on `--device cpu`).  Exit status: 0 all cases pass, 1 any case
fails, 2 setup error.  Test infrastructure: it uses the oracle's restatement of the case grids.
"""
import argparse
import csv
import math
import os
import sys
import time

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
for _p in (os.path.join(REPO, "fused-attention_b200"), REPO):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

from oracle import attention_oracle as ora  # noqa: E402

ATOL, RTOL, REL_FLOOR = ora.ATOL, ora.RTOL, ora.REL_FLOOR
BWD_REL = 2e-2
# the reference's 7 backward cases (B, H, N, D, sigma); inputs from a CUDA generator seeded N + D
BACKWARD_CASES = [(1, 1, 128, 64, 1.0), (2, 4, 256, 64, 1.0), (2, 4, 512, 128, 1.0), (1, 2, 1024, 64, 3.0),
                  (2, 8, 2048, 64, 1.0), (2, 8, 2048, 128, 1.0), (1, 4, 512, 64, 7.0)]
ROW_CHUNK = 2048  # query rows per reference block (bounds the fp32 score matrix)

FWD_COLUMNS = ["case", "B", "H", "N", "D", "magnitude", "seed", "max_abs_err", "max_rel_err", "tol_ratio",
               "time_s", "result", "note"]
GQA_COLUMNS = ["case", "B", "H", "H_kv", "group", "N", "D", "magnitude", "seed", "max_abs_err", "max_rel_err",
               "tol_ratio", "time_s", "result", "note"]
BWD_COLUMNS = ["test", "B", "H", "N", "D", "sigma", "relerr_O", "relerr_dQ", "relerr_dK", "relerr_dV", "result",
               "fused_ms", "sdpa_ms", "fused_speedup_vs_sdpa"]


def reference_forward(q, k, v):
    """fp32 causal attention (query head h reads K/V head h // (H / H_kv)), in row blocks."""
    B, H, N, D = q.shape
    grp = H // k.shape[1]
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    for b in range(B):
        for h in range(H):
            kf, vf = k[b, h // grp].float(), v[b, h // grp].float()
            for r0 in range(0, N, ROW_CHUNK):
                r1 = min(N, r0 + ROW_CHUNK)
                s = (q[b, h, r0:r1].float() @ kf[:r1].T) / math.sqrt(D)
                qi = torch.arange(r0, r1, device=q.device)[:, None]
                ki = torch.arange(0, r1, device=q.device)[None, :]
                s = s.masked_fill(ki > qi, float("-inf"))
                out[b, h, r0:r1] = torch.softmax(s, dim=-1) @ vf[:r1]
    return out


def reference_autograd(q, k, v, do):
    """fp32 autograd of causal attention: (O, dQ, dK, dV)."""
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    N, D = q.shape[-2], q.shape[-1]
    mask = torch.ones(N, N, dtype=torch.bool, device=q.device).triu(1)
    s = (qf @ kf.transpose(-1, -2)) / math.sqrt(D)
    o = torch.softmax(s.masked_fill(mask, float("-inf")), dim=-1) @ vf
    o.backward(do.float())
    return o.detach(), qf.grad, kf.grad, vf.grad


def forward_errors(out, ref):
    """(max_abs_err, max_rel_err, tol_ratio, finite) of out against ref."""
    out = out.float()
    finite = bool(torch.isfinite(out).all())
    d = (out - ref).abs()
    return (float(d.max()), float((d / ref.abs().clamp_min(REL_FLOOR)).max()),
            float((d / (ATOL + RTOL * ref.abs())).max()), finite)


def rel_fro(x, ref):
    return float(torch.linalg.vector_norm(x.float() - ref) / torch.linalg.vector_norm(ref).clamp_min(1e-30))


def _sync(device):
    if device.type == "cuda":
        torch.cuda.synchronize(device)


def run_forward(a, device):
    gqa = a.suite == "gqa"
    cases = ora.gqa_cases() if gqa else ora.mha_cases()
    cases = [c for c in cases if a.filter in c.id]
    if a.impl == "fused":
        if gqa:
            from attention.gqa.fused_gqa import fused_gqa_attention as fn
        else:
            from attention.fused.fused import fused_attention as fn
    elif a.impl == "unfused":
        if gqa:
            from attention.gqa.unfused_gqa import unfused_gqa_attention as fn
        else:
            from attention.fused.unfused import unfused_attention as fn
    else:
        fn = lambda q, k, v, tm, tn: reference_forward(q, k, v)  # noqa: E731
    rows, failed = [], 0
    for c in cases:
        q, k, v = (torch.from_numpy(x).to(device) for x in ora.make_inputs(c))
        note = ""
        _sync(device)
        t0 = time.perf_counter()
        try:
            out = fn(q, k, v, a.tile_m, a.tile_n)
            _sync(device)
        except Exception as e:  # recorded as a failed case, like the reference's runner
            out, note = None, f"{type(e).__name__}: {e}"
        elapsed = time.perf_counter() - t0
        if out is not None:
            mx, rel, ratio, finite = forward_errors(out, reference_forward(q, k, v))
            ok = finite and ratio <= 1.0
            if not finite:
                note = "non-finite output"
        else:
            mx = rel = ratio = float("nan")
            ok = False
        failed += not ok
        head = [c.id, c.B, c.H] + ([c.H_kv, c.H // c.H_kv] if gqa else []) + [c.N, c.D, c.magnitude, c.seed]
        rows.append(head + [mx, rel, ratio, elapsed, "PASS" if ok else "FAIL", note])
        print(f"{c.id:32s} max_abs {mx:.3e}  tol_ratio {ratio:.3f}  {'PASS' if ok else 'FAIL'} {note}")
        del q, k, v, out
    return (GQA_COLUMNS if gqa else FWD_COLUMNS), rows, failed


def run_backward(a, device):
    if a.impl == "fused":
        from attention.backward.fused_backward import fused_attention_autograd
        fn = lambda q, k, v: fused_attention_autograd(q, k, v, a.tile_m, a.tile_n)  # noqa: E731
    else:
        fn = None
    rows, failed = [], 0
    for (B, H, N, D, sigma) in BACKWARD_CASES:
        name = f"B{B}_H{H}_N{N}_D{D}_s{sigma:g}"
        if a.filter not in name:
            continue
        gen = torch.Generator(device=device).manual_seed(N + D)
        q, k, v = (torch.randn(B, H, N, D, device=device, generator=gen) * sigma for _ in range(3))
        do = torch.randn(B, H, N, D, device=device, generator=gen)
        q, k, v, do = (t.half() for t in (q, k, v, do))
        ref = reference_autograd(q, k, v, do)
        if fn is None:
            got = ref
        else:
            qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
            o = fn(qg, kg, vg)
            o.backward(do)
            got = (o.detach(), qg.grad, kg.grad, vg.grad)
        errs = [rel_fro(x, r) for x, r in zip(got, ref)]
        ok = all(math.isfinite(e) and e <= BWD_REL for e in errs)
        failed += not ok
        rows.append(["correctness", B, H, N, D, sigma] + [f"{e:.3e}" for e in errs] + ["PASS" if ok else "FAIL", "", "", ""])
        print(f"{name:24s} " + "  ".join(f"{n} {e:.2e}" for n, e in zip(("O", "dQ", "dK", "dV"), errs)) + ("  PASS" if ok else "  FAIL"))
    return BWD_COLUMNS, rows, failed


def default_csv(a):
    tile = f"{a.tile_m}x{a.tile_n}"
    if a.impl == "unfused":  # the reference's layout for its non-fused implementations
        name = "unfused" if a.suite == "fused" else "unfused_gqa"
        return f"results/correctness/{name}/b200/correctness_{name}_b200_{tile}.csv"
    tag = "b200" if a.impl == "fused" else "reference"
    if a.suite == "fused":
        return f"results/correctness/fused/{tag}/{tile}/correctness_fused_{tag}_{tile}.csv"
    if a.suite == "gqa":
        return f"results/correctness/fused_gqa/{tag}/{tile}/correctness_fused_gqa_{tag}_{tile}.csv"
    return f"results/correctness/backward/backward_{tag}_{tile}.csv"


def main(argv=None):
    p = argparse.ArgumentParser(description="B200 kernels against the fp32 PyTorch ground truth, reference CSV schema")
    p.add_argument("--suite", required=True, choices=("fused", "gqa", "backward"))
    p.add_argument("--impl", default="fused", choices=("fused", "unfused", "reference"))
    p.add_argument("--tile-m", type=int, default=64)
    p.add_argument("--tile-n", type=int, default=64)
    p.add_argument("--filter", default="", help="only cases whose id contains this text")
    p.add_argument("--csv", default=None)
    p.add_argument("--device", default="cuda")
    a = p.parse_args(argv)
    try:
        device = torch.device(a.device)
        if device.type == "cuda" and not torch.cuda.is_available():
            raise RuntimeError("no CUDA device (use --impl reference --device cpu for a harness self-check)")
        if a.impl != "reference" and device.type != "cuda":
            raise RuntimeError(f"--impl {a.impl} needs a CUDA device")
        if a.impl == "unfused" and a.suite == "backward":
            raise RuntimeError("the unfused baseline is forward only")
    except RuntimeError as e:
        print(f"setup error: {e}", file=sys.stderr)
        return 2
    columns, rows, failed = (run_backward if a.suite == "backward" else run_forward)(a, device)
    path = a.csv or default_csv(a)
    os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
    with open(path, "w", newline="") as f:
        w = csv.writer(f)
        w.writerow(columns)
        w.writerows(rows)
    print(f"{len(rows) - failed}/{len(rows)} passed; wrote {path}")
    return 1 if failed else 0


if __name__ == "__main__":
    sys.exit(main())
